// Python bindings of the gpt2_harness_b200 native library.
//
// The launchers take raw device addresses (Python ints from Tensor.data_ptr())
// and a CUDA stream handle: validation of shapes, dtypes and devices happens
// once in gpt2_harness_b200/ops/*.py, so a launch from Python costs one
// pybind call and nothing else, and every call is capturable in a CUDA graph.
#include <pybind11/pybind11.h>
#include <cuda_runtime.h>
#include <stdexcept>
#include <string>

#include "attention.cuh"
#include "comm.cuh"
#include "decode.cuh"
#include "elementwise.cuh"
#include "gemm.cuh"
#include "launch_count.h"
#include "zero.cuh"
#include "tp.cuh"

namespace py = pybind11;
using namespace g2b;

namespace {

template <typename T>
T* P(int64_t v) {
  return reinterpret_cast<T*>(static_cast<uintptr_t>(v));
}
cudaStream_t S(int64_t v) { return reinterpret_cast<cudaStream_t>(static_cast<uintptr_t>(v)); }

void check(int rc, const char* what) {
  if (rc != 0) {
    cudaError_t e = last_launch_error();
    last_launch_error() = cudaSuccess;
    if (e == cudaSuccess) e = cudaPeekAtLastError();
    throw std::runtime_error(std::string(what) + " failed (code " + std::to_string(rc) +
                             ", cuda: " + cudaGetErrorString(e) + ")");
  }
}

HeadView hv(int64_t base, int64_t sb, int64_t st, int64_t sh) {
  HeadView v;
  v.base = P<void>(base);
  v.sb = sb;
  v.st = st;
  v.sh = sh;
  return v;
}

}  // namespace

PYBIND11_MODULE(_C, m) {
  m.doc() = "sm_100a kernels of gpt2_harness_b200";
  m.def("launch_count", []() { return (long long)launch_counter().load(); },
        "Number of kernels this library has launched in this process.");

  m.def(
      "gemm",
      [](int64_t A, int64_t lda, int a_mn, int64_t B, int64_t ldb, int b_mn, int M, int N, int K,
         int epi, int64_t out, int64_t ldo, int64_t aux, int64_t ldaux, int64_t bias, float alpha,
         int64_t alpha_ptr, int accumulate, int splits, int64_t workspace, int bn, int max_ctas,
         int pair, int64_t ce_stats, int64_t ce_targets, int64_t ce_tgt_logit, int ce_vocab_offset,
         int64_t owner_out, int owner_rows, int owner_self, int64_t err, int64_t stream) {
        GemmArgs g;
        g.A = P<void>(A);
        g.lda = lda;
        g.a_mn_major = a_mn;
        g.B = P<void>(B);
        g.ldb = ldb;
        g.b_mn_major = b_mn;
        g.M = M;
        g.N = N;
        g.K = K;
        g.epilogue = epi;
        g.out = P<void>(out);
        g.ldo = ldo;
        g.aux = P<void>(aux);
        g.ldaux = ldaux;
        g.bias = P<void>(bias);
        g.alpha = alpha;
        g.alpha_ptr = P<float>(alpha_ptr);
        g.accumulate = accumulate;
        g.splits = splits;
        g.workspace = P<void>(workspace);
        g.bn = bn;
        g.max_ctas = max_ctas;
        g.pair = pair;
        g.ce_stats = P<void>(ce_stats);
        g.ce_targets = P<int64_t>(ce_targets);
        g.ce_tgt_logit = P<float>(ce_tgt_logit);
        g.ce_vocab_offset = ce_vocab_offset;
        g.owner_out = P<void*>(owner_out);
        g.owner_rows = owner_rows;
        g.owner_self = owner_self;
        g.err = P<uint32_t>(err);
        check(gemm_bf16_launch(g, S(stream)), "gemm_bf16");
      });

  m.def("attn_fwd", [](int64_t q, int64_t k, int64_t v, int64_t o, int64_t sb, int64_t st,
                       int64_t sh, int64_t osb, int64_t ost, int64_t osh, int64_t lse, int B,
                       int H, int Hkv, int Tq, int Tk, int q_offset, int causal, float scale,
                       int64_t kv_sb, int64_t kv_st, int64_t kv_sh, int64_t err, int64_t stream) {
    AttnArgs a;
    a.q = hv(q, sb, st, sh);
    a.k = hv(k, kv_sb, kv_st, kv_sh);
    a.v = hv(v, kv_sb, kv_st, kv_sh);
    a.o = hv(o, osb, ost, osh);
    a.lse = P<float>(lse);
    a.B = B;
    a.H = H;
    a.Hkv = Hkv;
    a.Tq = Tq;
    a.Tk = Tk;
    a.q_offset = q_offset;
    a.causal = causal;
    a.scale = scale;
    a.err = P<uint32_t>(err);
    check(attn_fwd_launch(a, S(stream)), "attn_fwd");
  });

  m.def("attn_bwd",
        [](int64_t q, int64_t k, int64_t v, int64_t o, int64_t dout, int64_t dq, int64_t dk,
           int64_t dv, int64_t sb, int64_t st, int64_t sh, int64_t osb, int64_t ost, int64_t osh,
           int64_t dsb, int64_t dst, int64_t dsh, int64_t lse, int64_t delta, int B, int H,
           int Hkv, int Tq, int Tk, int q_offset, int causal, float scale, int64_t kv_sb, int64_t kv_st,
           int64_t kv_sh, int64_t dkv_sb, int64_t dkv_st, int64_t dkv_sh, int64_t err,
           int64_t stream) {
          AttnArgs a;
          a.q = hv(q, sb, st, sh);
          a.k = hv(k, kv_sb, kv_st, kv_sh);
          a.v = hv(v, kv_sb, kv_st, kv_sh);
          a.o = hv(o, osb, ost, osh);
          a.dout = hv(dout, osb, ost, osh);
          a.dq = hv(dq, dsb, dst, dsh);
          a.dk = hv(dk, dkv_sb, dkv_st, dkv_sh);
          a.dv = hv(dv, dkv_sb, dkv_st, dkv_sh);
          a.lse = P<float>(lse);
          a.delta = P<float>(delta);
          a.B = B;
          a.H = H;
          a.Hkv = Hkv;
          a.Tq = Tq;
          a.Tk = Tk;
          a.q_offset = q_offset;
          a.causal = causal;
          a.scale = scale;
          a.err = P<uint32_t>(err);
          check(attn_bwd_launch(a, S(stream)), "attn_bwd");
        });

  // Context-parallel streaming forms: keys and values read in place from
  // every owner's compact [B, Tl, 2C] buffer (peer_bases[q], this process's
  // mapping), after owner q's publish word flags[q] reaches `epoch`.
  auto kv_peers = [](const py::sequence& bases, int64_t kv_sb, int64_t kv_st, int64_t v_off,
                     int Tl, int zigzag, int64_t flags, int64_t epoch) {
    const size_t n = py::len(bases);
    if (n == 0 || n > (size_t)kKvMaxOwners)
      throw std::runtime_error("attention peers: 1 to 8 owner buffers");
    KvPeers kp;
    kp.world = (int)n;
    for (size_t q = 0; q < n; ++q) kp.base[q] = reinterpret_cast<void*>(bases[q].cast<int64_t>());
    kp.sb = kv_sb;
    kp.st = kv_st;
    kp.v_off = v_off;
    kp.Tl = Tl;
    kp.zigzag = zigzag;
    kp.flags = P<const uint32_t>(flags);
    kp.epoch = (uint32_t)epoch;
    return kp;
  };
  m.def("attn_fwd_peers", [kv_peers](int64_t q, int64_t o, int64_t sb, int64_t st, int64_t sh, int64_t osb,
                                     int64_t ost, int64_t osh, int64_t lse, int B, int H, int Hkv, int Tq,
                                     int Tk, int q_offset, float scale, const py::sequence& bases,
                                     int64_t kv_sb, int64_t kv_st, int64_t v_off, int Tl, int zigzag,
                                     int64_t flags, int64_t epoch, int64_t err, int64_t stream) {
    const KvPeers kp = kv_peers(bases, kv_sb, kv_st, v_off, Tl, zigzag, flags, epoch);
    AttnArgs a;
    a.q = hv(q, sb, st, sh);
    a.o = hv(o, osb, ost, osh);
    a.lse = P<float>(lse);
    a.B = B;
    a.H = H;
    a.Hkv = Hkv;
    a.Tq = Tq;
    a.Tk = Tk;
    a.q_offset = q_offset;
    a.causal = 1;
    a.scale = scale;
    a.err = P<uint32_t>(err);
    a.peers = &kp;
    check(attn_fwd_launch(a, S(stream)), "attn_fwd_peers");
  });
  m.def("attn_bwd_peers",
        [kv_peers](int64_t q, int64_t o, int64_t dout, int64_t dq, int64_t dk, int64_t dv, int64_t sb,
                   int64_t st, int64_t sh, int64_t osb, int64_t ost, int64_t osh, int64_t dsb, int64_t dst,
                   int64_t dsh, int64_t lse, int64_t delta, int B, int H, int Hkv, int Tq, int Tk,
                   int q_offset, float scale, int64_t dkv_sb, int64_t dkv_st, int64_t dkv_sh,
                   const py::sequence& bases, int64_t kv_sb, int64_t kv_st, int64_t v_off, int Tl,
                   int zigzag, int64_t flags, int64_t epoch, int64_t err, int64_t stream) {
          const KvPeers kp = kv_peers(bases, kv_sb, kv_st, v_off, Tl, zigzag, flags, epoch);
          AttnArgs a;
          a.q = hv(q, sb, st, sh);
          a.o = hv(o, osb, ost, osh);
          a.dout = hv(dout, osb, ost, osh);
          a.dq = hv(dq, dsb, dst, dsh);
          a.dk = hv(dk, dkv_sb, dkv_st, dkv_sh);
          a.dv = hv(dv, dkv_sb, dkv_st, dkv_sh);
          a.lse = P<float>(lse);
          a.delta = P<float>(delta);
          a.B = B;
          a.H = H;
          a.Hkv = Hkv;
          a.Tq = Tq;
          a.Tk = Tk;
          a.q_offset = q_offset;
          a.causal = 1;
          a.scale = scale;
          a.err = P<uint32_t>(err);
          a.peers = &kp;
          check(attn_bwd_launch(a, S(stream)), "attn_bwd_peers");
        });

  m.def("attn_set_impl", [](int impl) { attn_set_impl(impl); },
        "0: tensor-core forward when the layout allows (default); 1: mma.sync forward");
  m.def("attn_get_impl", []() { return attn_get_impl(); });

  m.def("layernorm_fwd", [](int64_t x, int64_t ldx, int64_t g, int64_t b, int64_t y, int64_t ldy,
                            int64_t mean, int64_t rstd, int M, int C, float eps, int64_t push_bases,
                            int push_n, int64_t push_local, int64_t stream) {
    RowPush push;
    push.bases = P<void*>(push_bases);
    push.n = push_n;
    push.local = P<void>(push_local);
    check(layernorm_fwd_launch(P<float>(x), ldx, P<void>(g), P<void>(b), P<void>(y), ldy,
                               P<float>(mean), P<float>(rstd), M, C, eps, S(stream), push),
          "layernorm_fwd");
  });

  m.def("layernorm_bwd", [](int64_t dy, int64_t x, int64_t mean, int64_t rstd, int64_t g,
                            int64_t dres, int64_t dres_bf16, int64_t partials, int64_t dgamma,
                            int64_t dbeta, int64_t dsum, int M, int C, int accumulate,
                            int acc_params, int acc_sum, int64_t push_bases, int push_n,
                            int64_t push_local, int64_t stream) {
    RowPush push;
    push.bases = P<void*>(push_bases);
    push.n = push_n;
    push.local = P<void>(push_local);
    check(layernorm_bwd_launch(P<void>(dy), P<float>(x), P<float>(mean), P<float>(rstd),
                               P<void>(g), P<float>(dres), P<void>(dres_bf16), P<float>(partials),
                               P<float>(dgamma), P<float>(dbeta), P<float>(dsum), M, C,
                               accumulate, acc_params, acc_sum, S(stream), push),
          "layernorm_bwd");
  });

  m.def("layernorm_bwd_partial_rows", [](int M) { return layernorm_bwd_partial_rows(M); });

  m.def("colsum_f32", [](int64_t in, int R, int C, int64_t out, int acc, int64_t stream) {
    check(colsum_f32_launch(P<float>(in), R, C, P<float>(out), acc, S(stream)), "colsum_f32");
  });

  m.def("colsum_bf16", [](int64_t in, int64_t ld, int M, int C, int64_t ws, int64_t out, int acc,
                          int64_t stream) {
    check(colsum_bf16_launch(P<void>(in), ld, M, C, P<float>(ws), P<float>(out), acc, S(stream)),
          "colsum_bf16");
  });

  m.def("embedding_fwd", [](int64_t idx, int64_t wte, int64_t wpe, int64_t x, int B, int T, int C,
                            int pos0, int split, int pos1, int64_t stream) {
    check(embedding_fwd_launch(P<int64_t>(idx), P<void>(wte), P<void>(wpe), P<float>(x), B, T, C,
                               pos0, split, pos1, S(stream)),
          "embedding_fwd");
  });

  m.def("embedding_bwd", [](int64_t idx, int64_t dx, int64_t wte_grad, int64_t wpe_grad, int B,
                            int T, int C, int V, int pos0, int split, int pos1, int64_t det_part,
                            int64_t det_slots, int64_t stream) {
    check(embedding_bwd_launch(P<int64_t>(idx), P<float>(dx), P<float>(wte_grad),
                               P<float>(wpe_grad), B, T, C, V, pos0, split, pos1, S(stream),
                               P<float>(det_part), P<int>(det_slots)),
          "embedding_bwd");
  });
  m.def("embedding_wte_det_chunks", [](int64_t M) { return embedding_wte_det_chunks(M); });

  m.def("cross_entropy", [](int64_t logits, int64_t ld, int64_t targets, int64_t loss_rows, int M,
                            int V, int vocab_offset, int64_t stream) {
    check(cross_entropy_fwd_bwd_launch(P<void>(logits), ld, P<int64_t>(targets),
                                       P<float>(loss_rows), M, V, vocab_offset, S(stream)),
          "cross_entropy");
  });

  m.def("exp2_fma_test", [](int64_t x, int64_t y, int n, int64_t stream) {
    check(exp2_fma_test_launch(P<float>(x), P<float>(y), n, S(stream)), "exp2_fma_test");
  });
  m.def("ce_combine", [](int64_t stats, int nparts, int M, int64_t targets, int64_t tgt_logit,
                         int64_t lse, int64_t loss_rows, int64_t stream) {
    check(ce_combine_launch(P<void>(stats), nparts, M, P<int64_t>(targets), P<float>(tgt_logit),
                            P<float>(lse), P<float>(loss_rows), S(stream)),
          "ce_combine");
  });
  m.def("ce_grad", [](int64_t logits, int64_t ld, int M, int V, int64_t lse, int64_t targets,
                      int vocab_offset, int64_t stream) {
    check(ce_grad_launch(P<void>(logits), ld, M, V, P<float>(lse), P<int64_t>(targets),
                         vocab_offset, S(stream)),
          "ce_grad");
  });
  m.def("loss_reduce", [](int64_t loss_rows, int64_t targets, int M, int64_t out, int64_t stream) {
    check(loss_reduce_launch(P<float>(loss_rows), P<int64_t>(targets), M, P<float>(out),
                             S(stream)),
          "loss_reduce");
  });

  m.def("adamw", [](int64_t p, int64_t g, int64_t mm, int64_t v, int64_t pb, int64_t n,
                    int64_t n_decay, int64_t ranges, int nr, int64_t hp, int64_t clip,
                    int64_t stream) {
    check(adamw_launch(P<float>(p), P<float>(g), P<float>(mm), P<float>(v), P<void>(pb), n,
                       n_decay, P<int64_t>(ranges), nr, P<float>(hp), P<float>(clip), S(stream)),
          "adamw");
  });

  m.def("sumsq", [](int64_t g, int64_t n, int64_t ws, int64_t out, int64_t stream) {
    check(sumsq_launch(P<float>(g), n, P<float>(ws), P<float>(out), S(stream)), "sumsq");
  });

  m.def("clip_coef", [](int64_t sumsq, float scale2, float max_norm, int64_t clip,
                        int64_t norm_out, int64_t stream) {
    check(clip_coef_launch(P<float>(sumsq), scale2, max_norm, P<float>(clip), P<float>(norm_out),
                           S(stream)),
          "clip_coef");
  });

  m.def("cast_f32_bf16", [](int64_t in, int64_t out, int64_t n, int64_t stream) {
    check(cast_f32_bf16_launch(P<float>(in), P<void>(out), n, S(stream)), "cast_f32_bf16");
  });
  m.def("cast_bf16_f32", [](int64_t in, int64_t out, int64_t n, int64_t stream) {
    check(cast_bf16_f32_launch(P<void>(in), P<float>(out), n, S(stream)), "cast_bf16_f32");
  });
  m.def("scale_f32", [](int64_t x, int64_t n, float a, int64_t stream) {
    check(scale_f32_launch(P<float>(x), n, a, S(stream)), "scale_f32");
  });

  // ----------------------------------------------------- peer-memory comm ---
  m.def("ipc_handle", [](int64_t ptr) { return py::bytes(comm_ipc_handle(P<void>(ptr))); });
  m.def("ipc_open", [](py::bytes h) {
    void* p = comm_ipc_open(std::string(h));
    if (!p) throw std::runtime_error("ipc_open: cudaIpcOpenMemHandle failed");
    return (int64_t)(uintptr_t)p;
  });
  m.def("ipc_close", [](int64_t ptr) { comm_ipc_close(P<void>(ptr)); });
  m.def("enable_peer_access", [](int peer) { return comm_enable_peer(peer); });
  m.def("symm_alloc", [](int64_t bytes) {
    void* p = comm_symm_alloc(bytes);
    if (!p) throw std::runtime_error("symm_alloc: cudaMalloc failed");
    return (int64_t)(uintptr_t)p;
  });
  m.def("symm_free", [](int64_t p) { comm_symm_free(P<void>(p)); });
  // The three all-reduce forms share one argument list; `count` is the
  // payload (elements) charged to the byte counter, < 0 = n.
  auto comm_args = [](int64_t peer_bufs, int64_t peer_flags, int rank, int world, int64_t offset,
                      int64_t n, int dtype, float scale, uint32_t epoch, int64_t counter,
                      int64_t err, int nblocks, int64_t wait_budget_ns, int64_t count) {
    CommArgs c;
    c.peer_bufs = P<void*>(peer_bufs);
    c.peer_flags = P<uint32_t*>(peer_flags);
    c.rank = rank;
    c.world = world;
    c.offset = offset;
    c.n = n;
    c.dtype = dtype;
    c.scale = scale;
    c.epoch = epoch;
    c.byte_counter = P<unsigned long long>(counter);
    c.err = P<uint32_t>(err);
    c.nblocks = nblocks;
    c.wait_budget_ns = wait_budget_ns;
    c.count = count;
    return c;
  };
  m.def("allreduce_p2p",
        [comm_args](int64_t peer_bufs, int64_t peer_flags, int rank, int world, int64_t offset,
                    int64_t n, int dtype, float scale, uint32_t epoch, int64_t counter, int64_t err,
                    int nblocks, int64_t wait_budget_ns, int64_t count, int64_t stream) {
          CommArgs c = comm_args(peer_bufs, peer_flags, rank, world, offset, n, dtype, scale, epoch,
                                 counter, err, nblocks, wait_budget_ns, count);
          check(comm_allreduce_launch(c, S(stream)), "allreduce_p2p");
        });
  m.def("allreduce_p2p_slim",
        [comm_args](int64_t peer_bufs, int64_t peer_flags, int rank, int world, int64_t offset,
                    int64_t n, int dtype, float scale, uint32_t epoch, int64_t counter, int64_t err,
                    int nblocks, int64_t wait_budget_ns, int64_t count, int64_t stream) {
          CommArgs c = comm_args(peer_bufs, peer_flags, rank, world, offset, n, dtype, scale, epoch,
                                 counter, err, nblocks, wait_budget_ns, count);
          c.threads = 128;
          check(comm_allreduce_launch(c, S(stream)), "allreduce_p2p_slim");
        });
  m.def("allreduce_mc",
        [comm_args](int64_t peer_bufs, int64_t peer_flags, int64_t mc_base, int rank, int world,
                    int64_t offset, int64_t n, int dtype, float scale, uint32_t epoch,
                    int64_t counter, int64_t err, int nblocks, int64_t wait_budget_ns,
                    int64_t count, int64_t stream) {
          CommArgs c = comm_args(peer_bufs, peer_flags, rank, world, offset, n, dtype, scale, epoch,
                                 counter, err, nblocks, wait_budget_ns, count);
          c.mc_base = P<void>(mc_base);
          check(comm_allreduce_mc_launch(c, S(stream)), "allreduce_mc");
        });
  // ZeRO-2 kernels: every argument is passed by name in a dict (int pointers,
  // ints, floats); see csrc/zero.cuh for their meaning.
  auto zero_args = [](const py::dict& d) {
    auto I = [&](const char* k) { return d[k].cast<int64_t>(); };
    ZeroArgs z;
    z.peer_grad = P<float*>(I("peer_grad"));
    z.peer_grad16 = P<__nv_bfloat16*>(d.contains("peer_grad16") ? I("peer_grad16") : 0);
    z.peer_shadow = P<__nv_bfloat16*>(I("peer_shadow"));
    z.peer_flags = P<uint32_t*>(I("peer_flags"));
    z.peer_norm = P<unsigned long long*>(I("peer_norm"));
    z.rank = (int)I("rank");
    z.world = (int)I("world");
    z.buckets = P<int64_t>(I("buckets"));
    z.nb = (int)I("nb");
    z.bucket = (int)I("bucket");
    z.rs_blocks = (int)I("rs_blocks");
    z.gsh = P<float>(I("gsh"));
    z.master = P<float>(I("master"));
    z.exp_avg = P<float>(I("exp_avg"));
    z.exp_avg_sq = P<float>(I("exp_avg_sq"));
    z.sumsq_parts = P<float>(I("sumsq_parts"));
    z.decay_ranges = P<int64_t>(I("decay_ranges"));
    z.nr = (int)I("nr");
    z.hp = P<float>(I("hp"));
    z.max_norm = d["max_norm"].cast<float>();
    z.scale = d["scale"].cast<float>();
    z.epoch = (uint32_t)I("epoch");
    z.byte_counter = P<unsigned long long>(I("byte_counter"));
    z.norm_out = P<float>(I("norm_out"));
    z.err = P<uint32_t>(I("err"));
    z.wait_budget_ns = I("wait_budget_ns");
    if (d.contains("done_handshake")) z.done_handshake = (int)I("done_handshake");
    if (d.contains("peer_shard")) {
      z.peer_shard = P<__nv_bfloat16*>(I("peer_shard"));
      z.gather_dst = P<__nv_bfloat16>(I("gather_dst"));
      z.ag_span = I("ag_span");
      z.ag_slice = I("ag_slice");
      z.ag_offset = I("ag_offset");
    }
    return z;
  };
  m.def("zero_rs", [zero_args](const py::dict& d, int64_t stream) {
    check(zero_rs_launch(zero_args(d), S(stream)), "zero_rs");
  });
  m.def("zero_adamw_ag", [zero_args](const py::dict& d, int nblocks, int64_t stream) {
    check(zero_adamw_ag_launch(zero_args(d), nblocks, S(stream)), "zero_adamw_ag");
  });
  m.def("zero_ag", [zero_args](const py::dict& d, int nblocks, int64_t stream) {
    check(zero_ag_launch(zero_args(d), nblocks, S(stream)), "zero_ag");
  });
  // Tensor-parallel kernels: arguments by name (see csrc/tp.cuh).
  auto tp_args = [](const py::dict& d) {
    auto I = [&](const char* k) -> int64_t { return d.contains(k) ? d[k].cast<int64_t>() : 0; };
    TpArgs t;
    t.peer_bufs = P<void*>(I("peer_bufs"));
    t.peer_flags = P<uint32_t*>(I("peer_flags"));
    t.rank = (int)I("rank");
    t.world = (int)I("world");
    t.rows = I("rows");
    t.cols = (int)I("cols");
    t.nblocks = d.contains("nblocks") ? (int)I("nblocks") : 64;
    t.epoch = (uint32_t)I("epoch");
    t.bias = P<const __nv_bfloat16>(I("bias"));
    t.resid = P<const float>(I("resid"));
    t.out_f32 = P<float>(I("out_f32"));
    t.out_bf16 = P<__nv_bfloat16>(I("out_bf16"));
    t.idx = P<const int64_t>(I("idx"));
    t.wpe = P<const __nv_bfloat16>(I("wpe"));
    t.T = d.contains("T") ? (int)I("T") : 1;
    t.vocab_per_rank = I("vocab_per_rank");
    t.logits = P<__nv_bfloat16>(I("logits"));
    t.ld = I("ld");
    t.vocab_valid = (int)I("vocab_valid");
    t.vocab_start = I("vocab_start");
    t.stats = P<float>(I("stats"));
    t.loss_rows = P<float>(I("loss_rows"));
    t.byte_counter = P<unsigned long long>(I("byte_counter"));
    t.err = P<uint32_t>(I("err"));
    if (d.contains("wait_budget_ns")) t.wait_budget_ns = I("wait_budget_ns");
    t.src = P<const __nv_bfloat16>(I("src"));
    t.src_ld = I("src_ld");
    t.B = (int)I("B");
    t.Tl = (int)I("Tl");
    t.zigzag = (int)I("zigzag");
    t.pushed = (int)I("pushed");
    t.inbox = P<const __nv_bfloat16>(I("inbox"));
    t.peer_bufs2 = P<void*>(I("peer_bufs2"));
    return t;
  };
  m.def("cp_kv_gather", [tp_args](const py::dict& d, int64_t st) {
    check(cp_kv_gather_launch(tp_args(d), S(st)), "cp_kv_gather");
  });
  m.def("cp_kv_publish", [tp_args](const py::dict& d, int64_t st) {
    check(cp_kv_publish_launch(tp_args(d), S(st)), "cp_kv_publish");
  });
  m.def("kv_publish_words", []() { return kKvPublishWords; });
  m.def("cp_kv_reduce", [tp_args](const py::dict& d, int64_t st) {
    check(cp_kv_reduce_launch(tp_args(d), S(st)), "cp_kv_reduce");
  });
  m.def("tp_ag_rows", [tp_args](const py::dict& d, int64_t st) {
    check(tp_ag_rows_launch(tp_args(d), S(st)), "tp_ag_rows");
  });
  m.def("tp_rs_rows", [tp_args](const py::dict& d, int64_t st) {
    check(tp_rs_rows_launch(tp_args(d), S(st)), "tp_rs_rows");
  });
  m.def("tp_embed_fwd", [tp_args](const py::dict& d, int64_t st) {
    check(tp_embed_fwd_launch(tp_args(d), S(st)), "tp_embed_fwd");
  });
  m.def("tp_embed_bwd", [tp_args](const py::dict& d, int64_t st) {
    check(tp_embed_bwd_launch(tp_args(d), S(st)), "tp_embed_bwd");
  });
  m.def("tp_ce_stats", [tp_args](const py::dict& d, int64_t st) {
    check(tp_ce_stats_launch(tp_args(d), S(st)), "tp_ce_stats");
  });
  m.def("tp_ce_finish", [tp_args](const py::dict& d, int64_t st) {
    check(tp_ce_finish_launch(tp_args(d), S(st)), "tp_ce_finish");
  });
  m.def("tp_flag_words", []() { return 2 * kTpMaxRanks * kTpMaxBlocks; });
  m.def("zero_flag_words", []() { return 2 * kCommMaxRanks * kZeroMaxBlocks; });
  m.def("zero_norm_words", []() { return 2 * kZeroMaxBlocks * kCommMaxRanks; });
  m.def("zero_max_blocks", []() { return kZeroMaxBlocks; });
  m.def("comm_flag_words", []() { return kCommFlagWords; });
  m.def("flag_wait_test", [](int64_t flag, uint32_t value, int64_t budget_ns, int64_t err,
                             int64_t stream) {
    check(comm_flag_wait_test_launch(P<uint32_t>(flag), value, budget_ns, P<uint32_t>(err),
                                     S(stream)),
          "flag_wait_test");
  });
m.def("decode_embed", [](int64_t tok, int64_t lens, int64_t wte, int64_t wpe, int64_t x, int B, int C,
                           int64_t stream) {
    check(decode_embed_launch(P<int64_t>(tok), P<int>(lens), P<void>(wte), P<void>(wpe), P<float>(x), B, C,
                              S(stream)),
          "decode_embed");
  });
  m.def("decode_attn", [](int64_t qkv, int64_t ld, int64_t kc, int64_t vc, int64_t lens, int64_t part_o,
                          int64_t part_ml, int64_t out, int64_t ld_out, int B, int H, int Hkv, int Tmax,
                          float scale, int64_t stream) {
    check(decode_attn_launch(P<void>(qkv), ld, P<void>(kc), P<void>(vc), P<int>(lens), P<float>(part_o),
                             P<float>(part_ml), P<void>(out), ld_out, B, H, Hkv, Tmax, scale, S(stream)),
          "decode_attn");
  });
  m.def("decode_partials_numel", [](int B, int H, int Tmax) { return decode_partials_numel(B, H, Tmax); });
  m.def("decode_set_impl", [](int impl) { decode_set_impl(impl); },
        "decode attention kernel: 1 = one position a warp (default), 2 = four positions a warp");
  m.def("decode_get_impl", []() { return decode_get_impl(); });
  m.def("decode_argmax", [](int64_t logits, int64_t ld, int V, int64_t tok, int64_t lens, int64_t hist,
                            int Tmax, int B, int64_t stream) {
    check(decode_argmax_launch(P<void>(logits), ld, V, P<int64_t>(tok), P<int>(lens), P<int64_t>(hist), Tmax,
                               B, S(stream)),
          "decode_argmax");
  });
}
