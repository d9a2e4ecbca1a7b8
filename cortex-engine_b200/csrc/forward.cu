// Whole-forward driver: CortexModel.forward (cortex/models/cortex.py:90-122),
// return_aux=False, launched as one stream of kernels with no host sync.
//
//   pack+tokenize   window offsets and the gather-sum straight into packed order,
//                   norm_kv fused (_pack_events, :125-165): sorted batch indices
//                   are packed inside the tokenizer; a second launch repacks
//                   unsorted ones (stable counting sort) and tokenizes again
//   LN_q, q_proj    batch-invariant latent queries, computed once per forward
//   kv_proj         packed (E, 2D) keys|values                 (perceiver.py:67-69)
//   cross attention varlen keys per sample, no padding          (perceiver.py:71-80)
//   out_proj+resid  latents param broadcast as the residual      (perceiver.py:82)
//   N x block       LN, qkv, attention, out+resid, LN, mlp0+GELU, mlp2+resid; each
//                   LN rides the residual GEMM before it as a second output
//   final LN + head LN, head q, head kv_proj, 2-query attention, out_proj D->1
//                   (cortex.py:29-53): bf16 models run it as one fused kernel on a
//                   weight-only matrix built per forward (head.cu); otherwise
//                   row_norm2, two linears, attention and a GEMV
#include <cstdlib>
#include <cstring>

#include <vector>

#include "common.cuh"
#include "kernels.h"

namespace ck {
int linear_dispatch(const void* A, int dtype, int64_t M, int64_t K, int64_t lda, const void* W,
                    int w_dtype, int w_layout, int64_t N, int64_t ldw, const float* w_scale,
                    int epi, const void* aux, int64_t ld_aux, int64_t aux_row_mod, void* Y,
                    int64_t ldy, cudaStream_t st, bool w_static);
int attention_dispatch(const ck_attention_args& a, cudaStream_t st);
}  // namespace ck

using namespace ck;

namespace {

constexpr float kLnEps = 1e-5f;

size_t al(size_t x) { return (x + 255) & ~size_t(255); }

struct Layout {
  size_t counts, offsets, dest, emax, packws, tokslots, wdeq, xkv, kv, xq, qc, lat, x, qkv, att, hbuf, qh, oh,
      qall, total;
};

// The fused behaviour head (head.cu) runs whenever the model qualifies;
// CK_HEAD_FUSED=0 in the environment selects the composed head instead.
bool use_fused_head(const ck_model* m) {
  const char* v = std::getenv("CK_HEAD_FUSED");
  return (v == nullptr || std::strcmp(v, "0") != 0) && head_fused_supported(m);
}

// The INT8 linears of the self-attention blocks that the forward dequantises
// to bf16 once per call (bf16 models; K a multiple of 16 and 16-byte aligned
// weights), in block order qkv, out, mlp.0, mlp.2, with their (N, K).
struct DeqPlan {
  int n = 0;
  size_t bytes = 0;
};

int64_t block_lin_n(const ck_model* m, int j) {
  const int64_t D = m->latent_dim, Hm = m->mlp_hidden;
  return j == 0 ? 3 * D : (j == 2 ? Hm : D);
}
int64_t block_lin_k(const ck_model* m, int j) {
  return j == 3 ? (int64_t)m->mlp_hidden : (int64_t)m->latent_dim;
}
const ck_linear_weight& block_lin(const ck_block_weights& w, int j) {
  return j == 0 ? w.qkv : (j == 1 ? w.out : (j == 2 ? w.mlp0 : w.mlp2));
}
bool dequantised(const ck_model* m, const ck_linear_weight& lw, int64_t N, int64_t K) {
  if (m->dtype != CK_BF16 || lw.dtype != CK_I8 || lw.w == nullptr || lw.scale == nullptr)
    return false;
  DequantSeg g{reinterpret_cast<const int8_t*>(lw.w), lw.scale,
               reinterpret_cast<void*>(uintptr_t(256)), N, K, K, K};
  return dequant_seg_ok(g);
}
DeqPlan deq_plan(const ck_model* m) {
  DeqPlan d;
  for (int i = 0; i < m->num_layers && m->blocks != nullptr; ++i)
    for (int j = 0; j < 4; ++j) {
      const int64_t N = block_lin_n(m, j), K = block_lin_k(m, j);
      if (dequantised(m, block_lin(m->blocks[i], j), N, K)) {
        ++d.n;
        d.bytes += (size_t)N * K * 2;
      }
    }
  return d;
}

Layout plan(const ck_model* m, int64_t E, int32_t B) {
  const size_t es = m->dtype == CK_F32 ? 4 : 2;
  const size_t D = m->latent_dim, Dh_in = m->hidden_dim, L = m->num_latents;
  const size_t BL = (size_t)B * L;
  Layout o;
  size_t p = 0;
  auto take = [&](size_t bytes) {
    size_t at = p;
    p += al(bytes);
    return at;
  };
  o.counts = take((size_t)B * 4);
  o.offsets = take((size_t)(B + 1) * 4);
  o.dest = take((size_t)(E > 0 ? E : 1) * 4);
  o.emax = take(4);
  o.packws = take(pack_workspace_bytes(E, B));
  o.tokslots = take(tokenize_packed_slots() * 4);
  o.wdeq = take(deq_plan(m).bytes + 256);
  o.xkv = take((size_t)(E > 0 ? E : 1) * Dh_in * es);
  o.kv = take((size_t)(E > 0 ? E : 1) * 2 * D * es);
  o.xq = take(L * D * es);
  o.qc = take(L * D * es);
  o.lat = take(BL * D * es);
  o.x = take(BL * D * es);
  o.qkv = take(BL * 3 * D * es);
  o.att = take(BL * D * es);
  o.hbuf = take(BL * (size_t)m->mlp_hidden * es);
  o.qh = take((size_t)m->behavior_dim * D * es);
  o.oh = take((size_t)B * m->behavior_dim * D * es);
  o.qall = take(use_fused_head(m) ? head_qall_bytes(m) : 1);
  o.total = p;
  return o;
}

int lin(const ck_model* m, const void* A, int64_t M, int64_t K, int64_t lda,
        const ck_linear_weight& w, int64_t N, int epi, const void* aux, int64_t ld_aux,
        int64_t mod, void* Y, int64_t ldy, cudaStream_t st) {
  if (w.w == nullptr) return CK_ERR_INVALID_ARG;
  if (w.bias != nullptr) return CK_ERR_UNSUPPORTED;  // every linear on this path is bias-free
  const int wd = w.dtype;
  if (wd != m->dtype && wd != CK_I8) return CK_ERR_UNSUPPORTED;
  // (the model's weights: no kernel of the forward writes them)
  return linear_dispatch(A, m->dtype, M, K, lda, w.w, wd, CK_W_NK, N, K, w.scale, epi, aux,
                         ld_aux, mod, Y, ldy, st, true);
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// The batch-invariant prologue (LayerNorm of the latent parameter, the cross
// attention's q_proj, the head's weight-only matrix) runs on a side stream
// forked from the caller's stream at the start of the forward and joined
// before the cross attention, so it overlaps packing, the tokenizer and
// kv_proj instead of preceding them. One side stream and event pair per host
// thread and device (a stream that joins a graph capture is captured with it).
// CK_SIDE=0 in the environment runs the prologue on the caller's stream.
struct SideStream {
  cudaStream_t s = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
  cudaEvent_t deq = nullptr;  // the INT8 weights' dequantisation is done
};

// A host thread's side streams, released when the thread exits (errors are
// ignored: at process exit the runtime may already be gone).
struct SideStreams {
  static constexpr int kMaxDev = 16;
  SideStream dev[kMaxDev];
  ~SideStreams() {
    for (SideStream& ss : dev) {
      if (ss.s) cudaStreamDestroy(ss.s);
      if (ss.fork) cudaEventDestroy(ss.fork);
      if (ss.join) cudaEventDestroy(ss.join);
      if (ss.deq) cudaEventDestroy(ss.deq);
    }
  }
};

SideStream* side_stream() {
  const char* v = std::getenv("CK_SIDE");
  if (v != nullptr && std::strcmp(v, "0") == 0) return nullptr;
  constexpr int kMaxDev = SideStreams::kMaxDev;
  thread_local SideStreams streams;
  SideStream* cache = streams.dev;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return nullptr;
  SideStream& ss = cache[dev];
  if (ss.s == nullptr) {
    SideStream n;
    if (cudaStreamCreateWithFlags(&n.s, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&n.fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&n.join, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&n.deq, cudaEventDisableTiming) != cudaSuccess) {
      (void)cudaGetLastError();
      if (n.s) cudaStreamDestroy(n.s);
      if (n.fork) cudaEventDestroy(n.fork);
      if (n.join) cudaEventDestroy(n.join);
      if (n.deq) cudaEventDestroy(n.deq);
      return nullptr;
    }
    ss = n;
  }
  return &ss;
}

// LayerNorm fused into the residual GEMM before it (gemm_tc FUSE_LN) is on by
// default; CK_LN_FUSE=0 in the environment runs separate LayerNorm kernels.
bool ln_fuse_enabled() {
  const char* v = std::getenv("CK_LN_FUSE");
  return v == nullptr || std::strcmp(v, "0") != 0;
}

// Residual linear Y = aux + A W^T whose output feeds a LayerNorm X = LN(Y).
// With bf16 activations and N = 512 (the two 256-column halves of a row block
// on a CTA pair) one GEMM writes both Y and X; otherwise a LayerNorm kernel
// follows the GEMM.
int lin_resid_ln(const ck_model* m, const void* A, int64_t M, int64_t K,
                 const ck_linear_weight& w, int64_t N, const void* aux, int64_t ld_aux,
                 int64_t mod, void* Y, const void* g, const void* b, void* X, cudaStream_t st) {
  if (ln_fuse_enabled() && m->dtype == CK_BF16 && w.w != nullptr && w.bias == nullptr &&
      (w.dtype == CK_BF16 || w.dtype == CK_I8) && N == 512 && g != nullptr && al16(g) &&
      (mod <= 0 || mod % 32 == 0) &&
      (b == nullptr || al16(b)) && al16(X) &&
      gemm_tc_supported(M, K, K, w.dtype, CK_W_NK, N, K, A, w.w, N, Y, CK_EPI_RESID, aux,
                        ld_aux)) {
    GemmFusion fz;
    fz.eps = kLnEps;
    fz.ln_out = X;
    fz.ln_ld = N;
    fz.ln_gamma = g;
    fz.ln_beta = b;
    fz.w_static = true;
    return gemm_tc(A, M, K, K, w.w, w.dtype, CK_W_NK, N, K, w.scale, CK_EPI_RESID, aux, ld_aux,
                   mod, Y, N, st, &fz);
  }
  const int rc = lin(m, A, M, K, K, w, N, CK_EPI_RESID, aux, ld_aux, mod, Y, N, st);
  if (rc != CK_OK) return rc;
  return row_norm(Y, m->dtype, M, (int32_t)N, N, g, b, kLnEps, CK_NORM_LAYER, X, N, st);
}

ck_attention_args attn_base(const ck_model* m) {
  ck_attention_args a;
  memset(&a, 0, sizeof(a));
  a.dtype = m->dtype;
  return a;
}

}  // namespace

extern "C" size_t ck_forward_workspace_bytes(const ck_model* m, int64_t E, int32_t B) {
  if (m == nullptr || B <= 0 || E < 0) return 0;
  return plan(m, E, B).total + 256;
}

namespace {

// Which part of the forward runs, split at the packed keys|values of the
// events (the streaming K|V cache reuses those rows across calls).
enum Stage { kFull = 0, kKvOnly = 1, kFromKv = 2 };

struct KvIo {
  Stage stage;
  void* kv;          // kKvOnly: destination rows; kFromKv: source rows (else NULL)
  int32_t* offsets;  // window offsets (B + 1), written / read like kv
};

// The forward over E events, of which events *n_valid..E-1 are padding when
// n_valid (a device word) is given. With io.stage == kFromKv, E is the number
// of K|V rows in io.kv and no event arrays are read.
int forward_impl(const ck_model* m, const void* nid, const void* tb, const void* val,
                 const void* bidx, int idx_dt, int64_t E, int32_t B, const int32_t* n_valid,
                 void* out, void* ws, size_t ws_bytes, void* stream,
                 KvIo io = {kFull, nullptr, nullptr}) {
  if (m == nullptr || B <= 0 || E < 0) return CK_ERR_INVALID_ARG;
  if (io.stage != kKvOnly && out == nullptr) return CK_ERR_INVALID_ARG;
  if (io.stage != kFull && (io.kv == nullptr || io.offsets == nullptr)) return CK_ERR_INVALID_ARG;
  if (m->dtype != CK_BF16 && m->dtype != CK_F32) return CK_ERR_UNSUPPORTED;
  if (m->latent_dim <= 0 || m->hidden_dim <= 0 || m->num_latents <= 0 || m->num_heads <= 0 ||
      m->cross_heads <= 0 || m->head_dim <= 0 || m->mlp_hidden <= 0 || m->behavior_dim <= 0 ||
      m->num_layers < 0)
    return CK_ERR_INVALID_ARG;
  if (m->num_heads * m->head_dim != m->latent_dim) return CK_ERR_INVALID_ARG;
  if (m->latent_dim % m->cross_heads != 0) return CK_ERR_INVALID_ARG;
  if (m->num_layers > 0 && m->blocks == nullptr) return CK_ERR_INVALID_ARG;
  if (io.stage != kFromKv && E > 0 && (!nid || !tb || !val || !bidx)) return CK_ERR_INVALID_ARG;
  const Layout lay = plan(m, E, B);
  if (ws == nullptr || ws_bytes < lay.total + 256) return CK_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ws) + 255) & ~uintptr_t(255));
  auto P = [&](size_t off) { return reinterpret_cast<void*>(base + off); };
  int32_t* counts = reinterpret_cast<int32_t*>(P(lay.counts));
  int32_t* offsets = io.offsets ? io.offsets : reinterpret_cast<int32_t*>(P(lay.offsets));
  void* kv = io.kv ? io.kv : P(lay.kv);
  int32_t* dest = reinterpret_cast<int32_t*>(P(lay.dest));
  int32_t* emax = reinterpret_cast<int32_t*>(P(lay.emax));
  const int64_t D = m->latent_dim, Din = m->hidden_dim, L = m->num_latents;
  const int64_t BL = (int64_t)B * L;
  const int64_t H = m->num_heads, Dh = m->head_dim;
  const int64_t Hc = m->cross_heads, Dhc = D / Hc;
  const int64_t nq = m->behavior_dim;
  int rc;
#define CK_TRY(expr)           \
  do {                         \
    rc = (expr);               \
    if (rc != CK_OK) return rc; \
  } while (0)

  cudaEvent_t join_ev = nullptr;  // the side stream's prologue is done
  cudaEvent_t deq_ev = nullptr;   // the side stream's dequantisation is done

  // The blocks' INT8 linears as bf16 weights in the workspace (dequantised
  // below, once per forward), or the module's own weights.
  std::vector<ck_linear_weight> bw((size_t)m->num_layers * 4);
  std::vector<DequantSeg> deq;
  {
    uint8_t* wq = reinterpret_cast<uint8_t*>(P(lay.wdeq));
    for (int i = 0; i < m->num_layers; ++i)
      for (int j = 0; j < 4; ++j) {
        const ck_linear_weight& lw = block_lin(m->blocks[i], j);
        const int64_t N = block_lin_n(m, j), K = block_lin_k(m, j);
        ck_linear_weight& o = bw[(size_t)i * 4 + j];
        o = lw;
        if (dequantised(m, lw, N, K)) {
          deq.push_back(DequantSeg{reinterpret_cast<const int8_t*>(lw.w), lw.scale, wq, N, K, K, K});
          o.w = wq;
          o.dtype = CK_BF16;
          o.scale = nullptr;
          wq += (size_t)N * K * 2;
        }
      }
  }

  const bool fused_head = use_fused_head(m);
  if (io.stage != kKvOnly) {
    // 3. latent queries (batch-invariant), on the side stream when there is one
    SideStream* side = side_stream();
    cudaStream_t ps = st;
    if (side != nullptr) {
      if (cudaEventRecord(side->fork, st) != cudaSuccess ||
          cudaStreamWaitEvent(side->s, side->fork, 0) != cudaSuccess)
        return record_cuda_error();
      ps = side->s;
    }
    CK_TRY(row_norm(m->latents, m->dtype, L, (int32_t)D, D, m->norm_q_w, m->norm_q_b, kLnEps,
                    CK_NORM_LAYER, P(lay.xq), D, ps));
    CK_TRY(lin(m, P(lay.xq), L, D, D, m->cross_q, D, CK_EPI_STORE, nullptr, 0, 0, P(lay.qc), D,
               ps));
    if (fused_head) CK_TRY(head_prep(m, P(lay.qall), ps));
    if (side != nullptr) {
      if (cudaEventRecord(side->join, ps) != cudaSuccess) return record_cuda_error();
      join_ev = side->join;
    }
    // the INT8 weights of the blocks, widened and scaled to bf16 as
    // QuantizedLinear.forward does per call (cortex/quantization/calibrate.py:225-228);
    // joined before the first block, after the cross attention
    if (!deq.empty()) {
      CK_TRY(dequant_int8(deq.data(), (int)deq.size(), ps));
      if (side != nullptr) {
        if (cudaEventRecord(side->deq, ps) != cudaSuccess) return record_cuda_error();
        deq_ev = side->deq;
      }
    }
  }

  if (io.stage != kFromKv) {
    if (E > 0 && E <= kTokPackMaxE && B <= kTokPackMaxB) {
      // 1+2. packing inside the tokenizer (+ norm_kv): sorted batch indices
      // need no separate packing launches; a second launch repacks otherwise
      CK_TRY(tokenize_packed(m->neuron_emb, m->time_emb, m->value_emb, m->dtype, (int32_t)Din,
                             m->n_vocab, m->t_vocab, m->v_vocab, nid, tb, val, bidx, idx_dt, E, B,
                             m->norm_kv_w, m->norm_kv_b, kLnEps, P(lay.xkv), Din, offsets,
                             reinterpret_cast<int32_t*>(P(lay.tokslots)), st, n_valid));
    } else {
      // 1. packing
      CK_TRY(pack_events(bidx, idx_dt, 1, E, B, n_valid, counts, offsets, dest, emax,
                         P(lay.packws), pack_workspace_bytes(E, B), st));
      // 2. tokenizer + norm_kv, written in packed order
      CK_TRY(tokenize(m->neuron_emb, m->time_emb, m->value_emb, m->dtype, (int32_t)Din,
                      m->n_vocab, m->t_vocab, m->v_vocab, Din, Din, Din, nid, tb, val, idx_dt, 1,
                      1, 1, E, dest, m->norm_kv_w, m->norm_kv_b, kLnEps, P(lay.xkv), Din, st,
                      n_valid));
    }
  }
  // 4. packed keys|values
  if (io.stage != kFromKv && E > 0)
    CK_TRY(lin(m, P(lay.xkv), E, Din, Din, m->cross_kv, 2 * D, CK_EPI_STORE, nullptr, 0, 0, kv,
               2 * D, st));
  if (io.stage == kKvOnly) return CK_OK;
  // the prologue's results (and the side stream) join the caller's stream
  if (join_ev != nullptr && cudaStreamWaitEvent(st, join_ev, 0) != cudaSuccess)
    return record_cuda_error();
  // 5. cross attention over each sample's own events
  {
    const size_t es_b = m->dtype == CK_F32 ? 4 : 2;
    ck_attention_args a = attn_base(m);
    a.B = B;
    a.H = (int32_t)Hc;
    a.Dh = (int32_t)Dhc;
    a.Lq = (int32_t)L;
    a.key_offsets = offsets;
    a.q = P(lay.qc);
    a.q_ld = D;
    a.q_rows = L;
    a.q_col_per_h = Dhc;
    a.k = kv;
    a.k_ld = 2 * D;
    a.k_rows = E > 0 ? E : 1;
    a.k_col_per_h = Dhc;
    a.v = reinterpret_cast<uint8_t*>(kv) + D * es_b;
    a.v_ld = 2 * D;
    a.v_rows = E > 0 ? E : 1;
    a.v_col_per_h = Dhc;
    a.o = P(lay.att);
    a.o_ld = D;
    a.o_rows_per_b = L;
    a.o_col_per_h = Dhc;
    a.scale = 1.0f / sqrtf((float)Dhc);
    CK_TRY(attention_dispatch(a, st));
  }
  // Self-attention of a block over its fused (BL, 3D) q|k|v rows.
  const size_t es_b = m->dtype == CK_F32 ? 4 : 2;
  auto self_attention = [&]() {
    ck_attention_args a = attn_base(m);
    a.B = B;
    a.H = (int32_t)H;
    a.Dh = (int32_t)Dh;
    a.Lq = (int32_t)L;
    a.n_keys = (int32_t)L;
    a.q = P(lay.qkv);
    a.q_ld = 3 * D;
    a.q_rows = BL;
    a.q_rows_per_b = L;
    a.q_col_per_h = Dh;
    a.k = reinterpret_cast<uint8_t*>(P(lay.qkv)) + D * es_b;
    a.k_ld = 3 * D;
    a.k_rows = BL;
    a.k_rows_per_b = L;
    a.k_col_per_h = Dh;
    a.v = reinterpret_cast<uint8_t*>(P(lay.qkv)) + 2 * D * es_b;
    a.v_ld = 3 * D;
    a.v_rows = BL;
    a.v_rows_per_b = L;
    a.v_col_per_h = Dh;
    a.o = P(lay.att);
    a.o_ld = D;
    a.o_rows_per_b = L;
    a.o_col_per_h = Dh;
    a.scale = 1.0f / sqrtf((float)Dh);
    return attention_dispatch(a, st);
  };
  const int64_t Hm = m->mlp_hidden;
  {
    // 6. out_proj + broadcast latent residual (and block 0's norm_attn of it)
    bool x_ready = false;  // lay.x already holds norm_attn(lat) for the next block
    if (m->num_layers > 0) {
      CK_TRY(lin_resid_ln(m, P(lay.att), BL, D, m->cross_out, D, m->latents, D, L, P(lay.lat),
                          m->blocks[0].norm_attn_w, m->blocks[0].norm_attn_b, P(lay.x), st));
      x_ready = true;
    } else {
      CK_TRY(lin(m, P(lay.att), BL, D, D, m->cross_out, D, CK_EPI_RESID, m->latents, D, L,
                 P(lay.lat), D, st));
    }
    // 7. self-attention blocks (their dequantised weights join here)
    if (deq_ev != nullptr && cudaStreamWaitEvent(st, deq_ev, 0) != cudaSuccess)
      return record_cuda_error();
    for (int i = 0; i < m->num_layers; ++i) {
      const ck_block_weights& w = m->blocks[i];
      const ck_linear_weight& w_qkv = bw[(size_t)i * 4];
      const ck_linear_weight& w_out = bw[(size_t)i * 4 + 1];
      const ck_linear_weight& w_mlp0 = bw[(size_t)i * 4 + 2];
      const ck_linear_weight& w_mlp2 = bw[(size_t)i * 4 + 3];
      if (!x_ready)
        CK_TRY(row_norm(P(lay.lat), m->dtype, BL, (int32_t)D, D, w.norm_attn_w, w.norm_attn_b,
                        kLnEps, CK_NORM_LAYER, P(lay.x), D, st));
      CK_TRY(lin(m, P(lay.x), BL, D, D, w_qkv, 3 * D, CK_EPI_STORE, nullptr, 0, 0, P(lay.qkv),
                 3 * D, st));
      x_ready = false;
      CK_TRY(self_attention());
      CK_TRY(lin_resid_ln(m, P(lay.att), BL, D, w_out, D, P(lay.lat), D, 0, P(lay.lat),
                          w.norm_mlp_w, w.norm_mlp_b, P(lay.x), st));
      CK_TRY(lin(m, P(lay.x), BL, D, D, w_mlp0, Hm, CK_EPI_GELU, nullptr, 0, 0, P(lay.hbuf), Hm,
                 st));
      if (i + 1 < m->num_layers) {
        CK_TRY(lin_resid_ln(m, P(lay.hbuf), BL, Hm, w_mlp2, D, P(lay.lat), D, 0, P(lay.lat),
                            m->blocks[i + 1].norm_attn_w, m->blocks[i + 1].norm_attn_b, P(lay.x),
                            st));
        x_ready = true;
      } else {
        CK_TRY(lin(m, P(lay.hbuf), BL, Hm, Hm, w_mlp2, D, CK_EPI_RESID, P(lay.lat), D, 0,
                   P(lay.lat), D, st));
      }
    }
  }
  // 8-9. final_norm, head norm and the behaviour head in one kernel
  if (fused_head) {
    CK_TRY(head_fused(m, P(lay.lat), B, P(lay.qall), out, st));
    return CK_OK;
  }
  // 8. final_norm then the head's norm
  CK_TRY(row_norm2(P(lay.lat), m->dtype, BL, (int32_t)D, D, m->final_norm_w, m->final_norm_b,
                   m->head_norm_w, m->head_norm_b, kLnEps, P(lay.x), D, st));
  // 9. behaviour head
  CK_TRY(lin(m, m->head_query, nq, D, D, m->head_q, D, CK_EPI_STORE, nullptr, 0, 0, P(lay.qh), D,
             st));
  CK_TRY(lin(m, P(lay.x), BL, D, D, m->head_kv, 2 * D, CK_EPI_STORE, nullptr, 0, 0, P(lay.qkv),
             2 * D, st));
  {
    ck_attention_args a = attn_base(m);
    a.B = B;
    a.H = (int32_t)H;
    a.Dh = (int32_t)Dh;
    a.Lq = (int32_t)nq;
    a.n_keys = (int32_t)L;
    a.q = P(lay.qh);
    a.q_ld = D;
    a.q_rows = nq;
    a.q_col_per_h = Dh;
    a.k = P(lay.qkv);
    a.k_ld = 2 * D;
    a.k_rows = BL;
    a.k_rows_per_b = L;
    a.k_col_per_h = Dh;
    a.v = reinterpret_cast<uint8_t*>(P(lay.qkv)) + D * es_b;
    a.v_ld = 2 * D;
    a.v_rows = BL;
    a.v_rows_per_b = L;
    a.v_col_per_h = Dh;
    a.o = P(lay.oh);
    a.o_ld = D;
    a.o_rows_per_b = nq;
    a.o_col_per_h = Dh;
    a.scale = 1.0f / sqrtf((float)Dh);
    CK_TRY(attention_dispatch(a, st));
  }
  CK_TRY(lin(m, P(lay.oh), (int64_t)B * nq, D, D, m->head_out, 1, CK_EPI_STORE, nullptr, 0, 0,
             out, 1, st));
#undef CK_TRY
  return CK_OK;
}

}  // namespace

extern "C" int ck_forward(const ck_model* m, const void* nid, const void* tb, const void* val,
                          const void* bidx, int idx_dt, int64_t E, int32_t B, void* out, void* ws,
                          size_t ws_bytes, void* stream) {
  return forward_impl(m, nid, tb, val, bidx, idx_dt, E, B, nullptr, out, ws, ws_bytes, stream);
}

extern "C" int ck_forward_kv(const ck_model* m, const int32_t* batch, int64_t capacity, int32_t B,
                             void* kv, int32_t* offsets, void* ws, size_t ws_bytes, void* stream) {
  if (batch == nullptr || capacity < 0 || capacity % 4 != 0) return CK_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(batch) & 15u) != 0) return CK_ERR_INVALID_ARG;
  const int32_t* a = batch + CK_BATCH_HEADER_WORDS;
  return forward_impl(m, a, a + capacity, a + 2 * capacity, a + 3 * capacity, CK_I32, capacity, B,
                      batch, nullptr, ws, ws_bytes, stream, KvIo{kKvOnly, kv, offsets});
}

extern "C" int ck_forward_from_kv(const ck_model* m, const void* kv, int64_t n_rows,
                                  const int32_t* offsets, int32_t B, void* out, void* ws,
                                  size_t ws_bytes, void* stream) {
  return forward_impl(m, nullptr, nullptr, nullptr, nullptr, CK_I32, n_rows, B, nullptr, out, ws,
                      ws_bytes, stream,
                      KvIo{kFromKv, const_cast<void*>(kv), const_cast<int32_t*>(offsets)});
}

extern "C" int ck_forward_batch(const ck_model* m, const int32_t* batch, int64_t capacity,
                                int32_t B, void* out, void* ws, size_t ws_bytes, void* stream) {
  if (batch == nullptr || capacity < 0 || capacity % 4 != 0) return CK_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(batch) & 15u) != 0) return CK_ERR_INVALID_ARG;
  const int32_t* a = batch + CK_BATCH_HEADER_WORDS;
  return forward_impl(m, a, a + capacity, a + 2 * capacity, a + 3 * capacity, CK_I32, capacity, B,
                      batch, out, ws, ws_bytes, stream);
}
