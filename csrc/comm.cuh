// Host-side interface of the peer-memory collectives (csrc/comm.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <string>

namespace g2b {

constexpr int kCommMaxBlocks = 160;  // flag slots per (phase, rank)
constexpr int kCommMaxRanks = 8;
// A rank's flag buffer: [2][kCommMaxRanks][kCommMaxBlocks] handshake words,
// then the device epoch counter and the launch's finished-CTA count (used
// when a launch passes epoch 0), then the record of the first handshake that
// gave up on this rank: {recorded, phase, CTA, peer, epoch waited for, flag
// value seen, this rank, 0}.
constexpr int kCommEpochWord = 2 * kCommMaxRanks * kCommMaxBlocks;
constexpr int kCommTimeoutWord = kCommEpochWord + 2;
constexpr int kCommFlagWords = kCommTimeoutWord + 8;

// One fused all-reduce over NVLink peer memory. Every rank owns a symmetric
// buffer (same size, same element offsets on every rank); peer_bufs[q] is rank
// q's buffer mapped into this process, peer_flags[q] rank q's flag array
// ([2][kCommMaxRanks][kCommMaxBlocks] uint32). The kernel reduces elements
// [offset, offset + n) across ranks, multiplies by `scale` and leaves the
// result in every rank's buffer.
struct CommArgs {
  void** peer_bufs = nullptr;       // device array [world]
  uint32_t** peer_flags = nullptr;  // device array [world]
  int rank = 0, world = 1;
  int64_t offset = 0, n = 0;        // elements
  int dtype = 0;                    // 0 = fp32 buffer, 1 = bf16 buffer
  float scale = 1.f;
  // strictly increasing per call, same on all ranks; 0 = take it from the
  // device counter in this rank's flag buffer (previous launch's + 1), so a
  // captured CUDA graph replays with fresh epochs
  uint32_t epoch = 0;
  unsigned long long* byte_counter = nullptr;  // payload bytes (reference convention)
  uint32_t* err = nullptr;
  int nblocks = 32;
  int64_t wait_budget_ns = 2000000000ll;
  // Threads per CTA: 512 (the wide kernel, for a GPU with nothing else to
  // run) or 128 (the slim kernel: <= 80 registers a thread and no dynamic
  // shared memory, so one CTA fits on an SM beside a resident persistent GEMM
  // or attention CTA and the reduction overlaps backward without taking SMs
  // away from it).
  int threads = 512;
  // Payload elements charged to byte_counter (the reference convention: the
  // parameters of the bucket, alignment padding excluded); < 0 = n.
  int64_t count = -1;
  // NVLink SHARP form (comm_allreduce_mc_launch): the multicast address of
  // the same symmetric buffer, bound to every rank's copy.
  void* mc_base = nullptr;
};

int comm_allreduce_launch(const CommArgs& a, cudaStream_t s);

// The same all-reduce through the NVSwitch (multimem): CTA j of rank r reads
// part j of slice r already summed over all ranks by the switch
// (multimem.ld_reduce on the multicast address), scales it and writes it to
// every rank's copy with one multimem.st. Each rank moves S/p in and S/p out
// of its own slice plus (p-1)/p * S of the others' results arriving: about
// half the NVLink bytes of the P2P form, with no reduction arithmetic on the
// SMs. Same flags, epochs and bounded handshakes as the P2P form.
int comm_allreduce_mc_launch(const CommArgs& a, cudaStream_t s);

// Launch a single-thread kernel that waits (bounded) for *flag == value and
// records ERR_TIMEOUT_PEER in *err when the budget expires. Used to test the
// bounded-wait path: a flag nobody sets must time out and leave the context
// usable.
int comm_flag_wait_test_launch(uint32_t* flag, uint32_t value, int64_t budget_ns, uint32_t* err,
                               cudaStream_t s);

// CUDA IPC helpers: export a device allocation, open a peer's, close it.
std::string comm_ipc_handle(void* ptr);
void* comm_ipc_open(const std::string& handle);
void comm_ipc_close(void* ptr);
int comm_enable_peer(int peer);

// A zero-filled device allocation of its own (cudaMalloc), so that one CUDA
// IPC handle covers exactly this buffer; released with comm_symm_free.
void* comm_symm_alloc(int64_t bytes);
void comm_symm_free(void* p);

}  // namespace g2b
