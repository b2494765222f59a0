// Device side of the context-parallel key/value streaming (KvPeers in
// attention.cuh): one TMA map per owner rank over that rank's symmetric
// key/value buffer, the owner and local row of a key position, and the
// bounded wait for an owner's publish flag. Shared by the tensor-core forward
// (attention_tc.cu) and backward (attention_bwd_tc.cu) kernels, which take a
// KvPeerMaps kernel argument in their streaming instantiation and a NoKvPeers
// (empty) one otherwise, so the single-GPU instantiation is unchanged.
//
// The loads are plain TMA tile loads (no cluster multicast) whose source is
// another GPU's memory reached over NVLink through its CUDA IPC mapping.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "attention.cuh"
#include "common.cuh"

namespace g2b {

struct KvPeerMaps {
  CUtensorMap k[kKvMaxOwners];  // owner q's keys:   {64, Hkv, Tl, B}
  CUtensorMap v[kKvMaxOwners];  // owner q's values: same dims
  const uint32_t* flags;
  uint32_t epoch;
  int world, zigzag, Tl;
};
struct NoKvPeers {};

template <class KV>
struct KvStreaming {
  static constexpr bool on = false;
};
template <>
struct KvStreaming<KvPeerMaps> {
  static constexpr bool on = true;
};

// Owner rank of natural key position k and its row in the owner's buffer
// (host-callable too, for the CPU check of this arithmetic).
__host__ __device__ __forceinline__ int kv_owner_row(const KvPeerMaps& kv, int k, int* local_row) {
  if (kv.zigzag) {
    const int h = kv.Tl >> 1;
    const int c = k / h;
    const bool first = c < kv.world;
    *local_row = (first ? 0 : h) + (k - c * h);
    return first ? c : 2 * kv.world - 1 - c;
  }
  const int q = k / kv.Tl;
  *local_row = k - q * kv.Tl;
  return q;
}

__device__ __forceinline__ uint32_t kv_ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Returns once owner q has published this call's epoch (bit q of *seen caches
// that for the rest of the launch). The rows were written by the owner's
// generic stores and are read here by TMA (the async proxy), hence the proxy
// fence after the acquire. Bounded: on expiry (or when another role already
// gave up) reports ERR_TIMEOUT_PEER, raises *abort and returns false.
__device__ __forceinline__ bool kv_owner_ready(const KvPeerMaps& kv, int q, uint32_t* seen,
                                               uint32_t* err, volatile int* abort) {
  if (*seen & (1u << q)) return true;
  const uint32_t* f = kv.flags + q;
  const uint64_t t0 = globaltimer_ns();
  while ((int32_t)(kv_ld_acquire_sys(f) - kv.epoch) < 0) {
    if (*abort) return false;
    if (globaltimer_ns() - t0 > kWaitBudgetNs) {
      report_error(err, ERR_TIMEOUT_PEER);
      *abort = 1;
      return false;
    }
    __nanosleep(128);
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
  *seen |= 1u << q;
  return true;
}

// Host: the per-owner maps, boxes of `rows` rows of one head (128B swizzle,
// K-major), over dims {64, Hkv, Tl, B} of each owner's buffer.
inline bool make_kv_peer_maps(KvPeerMaps* m, const KvPeers& p, int Hkv, int B, int rows,
                              PFN_cuTensorMapEncodeTiled_v12000 enc) {
  if (!enc || p.world < 1 || p.world > kKvMaxOwners || p.Tl % rows) return false;
  if (p.zigzag && (p.Tl / 2) % rows) return false;
  if ((p.sb * 2) % 16 || (p.st * 2) % 16 || (p.v_off * 2) % 16) return false;
  *m = KvPeerMaps{};
  for (int q = 0; q < p.world; ++q) {
    if (!p.base[q] || (reinterpret_cast<uintptr_t>(p.base[q]) & 15)) return false;
    for (int which = 0; which < 2; ++which) {
      void* base = static_cast<__nv_bfloat16*>(p.base[q]) + (which ? p.v_off : 0);
      cuuint64_t dims[4] = {64, (cuuint64_t)Hkv, (cuuint64_t)p.Tl, (cuuint64_t)B};
      cuuint64_t strides[3] = {64 * 2, (cuuint64_t)p.st * 2, (cuuint64_t)p.sb * 2};
      cuuint32_t box[4] = {64, 1, (cuuint32_t)rows, 1};
      cuuint32_t estr[4] = {1, 1, 1, 1};
      if (enc(which ? &m->v[q] : &m->k[q], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, base, dims,
              strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    }
  }
  m->flags = p.flags;
  m->epoch = p.epoch;
  m->world = p.world;
  m->zigzag = p.zigzag;
  m->Tl = p.Tl;
  return p.flags != nullptr;
}

}  // namespace g2b
