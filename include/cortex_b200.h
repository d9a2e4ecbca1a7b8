/*
 * cortex_b200.h — C ABI of the B200 (sm_100a) Cortex decoder forward hot path.
 *
 * Every entry point takes raw device pointers, element strides and an explicit
 * cudaStream_t (passed as void*), allocates nothing, and returns an int status
 * (CK_OK = 0, negative on error). Kernels that find bad data on the device
 * (an index out of range, a bounded wait that gave up) record a code in a
 * per-device status word that ck_get_last_status() reads back.
 *
 * The entry points replace the reference (peterajhgraham/cortex-engine) call
 * sites cited beside each one; the Python package in cortex-engine_b200/cortex
 * binds them with ctypes behind the reference's unchanged Python signatures.
 */
#ifndef CORTEX_B200_H_
#define CORTEX_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ── status codes ─────────────────────────────────────────────────────────── */
#define CK_OK 0
#define CK_ERR_INVALID_ARG -1 /* bad shape, stride, alignment or pointer */
#define CK_ERR_UNSUPPORTED -2 /* dtype / layout combination not built */
#define CK_ERR_CUDA -3        /* a CUDA runtime call failed (see ck_last_cuda_error) */
#define CK_ERR_INDEX -4       /* device: an event index is outside its table / batch */
#define CK_ERR_TIMEOUT -5     /* device: a bounded pipeline wait gave up */
#define CK_ERR_WORKSPACE -6   /* workspace smaller than the *_workspace_bytes query */

/* ── element types ────────────────────────────────────────────────────────── */
#define CK_F32 0
#define CK_BF16 1
#define CK_I8 2
#define CK_I32 3
#define CK_I64 4

/* ── norm modes and GEMM epilogues ────────────────────────────────────────── */
#define CK_NORM_NONE 0
#define CK_NORM_LAYER 1 /* (x - mean) * rstd * gamma + beta (nn.LayerNorm) */
#define CK_NORM_RMS 2   /* x / sqrt(mean(x^2) + eps) * gamma              */

#define CK_EPI_STORE 0 /* y = dtype(acc)                                  */
#define CK_EPI_GELU 1  /* y = dtype(gelu_erf(dtype(acc)))                 */
#define CK_EPI_RESID 2 /* y = dtype(aux[m % mod] + dtype(acc))            */
#define CK_EPI_BIAS 3  /* y = dtype(dtype(acc) + aux[n])                  */

#define CK_W_NK 0 /* weight stored (N, K): nn.Linear / QuantizedLinear */
#define CK_W_KN 1 /* weight stored (K, N): rms_norm_linear's w        */

/* Status word of the current device. Synchronises the device, copies the word
 * (and 4 info ints, may be NULL) out and clears it. Returns the code. */
int ck_get_last_status(int* info4);
/* Last CUDA runtime error recorded by an entry point that returned CK_ERR_CUDA. */
int ck_last_cuda_error(void);
const char* ck_status_string(int code);
/* Number of SMs of the current device (0 if none). */
int ck_num_sms(void);
/* Kernel launches issued by this library since it was loaded (all threads). */
long long ck_launch_count(void);

/* Launch trace, for measurement: between ck_trace_begin and ck_trace_end every
 * kernel the library launches outside a stream capture is bracketed by two
 * CUDA events on its own stream (up to `capacity` launches; later ones are
 * not timed). ck_trace_end synchronises on the events and writes one record
 * per traced launch, in launch order, to out[0 .. min(n, capacity)), with *n
 * the number traced. The events sit between launches, so a traced kernel does
 * not overlap its predecessor: each figure is that kernel's own device time.
 * No reference counterpart (the reference times kernels with torch profilers,
 * benchmarks/profiling/). */
typedef struct ck_trace_record {
  char name[96]; /* kernel name with template arguments, no namespaces */
  void* stream;  /* cudaStream_t the kernel ran on */
  float ms;      /* device time between the two events (-1 on error) */
} ck_trace_record;
int ck_trace_begin(int32_t capacity);
int ck_trace_end(ck_trace_record* out, int32_t capacity, int32_t* n);

/* ── 1. event packing ───────────────────────────────────────────────────────
 * Replaces _pack_events' index work (cortex/models/cortex.py:125-165):
 * bincount (:141), E_max (:142), stable argsort (:149), exclusive cumsum (:155-160),
 * pos_within (:161). Outputs counts[B], offsets[B+1] (offsets[B] = E),
 * dest[E] (packed row of every input event = offsets[b] + pos_within) and
 * e_max[1]. B must equal max(batch_indices)+1 (the reference's :140); an index
 * outside [0, B) sets CK_ERR_INDEX. */
size_t ck_pack_workspace_bytes(int64_t E, int32_t B);
int ck_pack_events(const void* batch_indices, int idx_dtype, int64_t idx_stride, int64_t E,
                   int32_t B, int32_t* counts, int32_t* offsets, int32_t* dest, int32_t* e_max,
                   void* workspace, size_t workspace_bytes, void* stream);

/* Padded layout of _pack_events (cortex/models/cortex.py:146-165): out[b, pos, :]
 * = flat[e, :], mask[b, pos] = 1, with pos = dest[e] - offsets[b]. `out` and
 * `mask` must be zeroed by the caller, as the reference's torch.zeros are. */
int ck_pack_scatter(const void* flat, int dtype, int64_t E, int32_t D, int64_t flat_stride,
                    const void* batch_indices, int idx_dtype, int64_t idx_stride,
                    const int32_t* dest, const int32_t* offsets, int32_t e_max, void* out,
                    uint8_t* mask, void* stream);

/* ── 2. tokenizer ───────────────────────────────────────────────────────────
 * Replaces fused_tokenizer (cortex/kernels/tokenizer.py:177-249) and the eager
 * sum of SpikeTokenizer.forward (cortex/models/tokenizer.py:90-93):
 * out[dest[e]] = n_emb[nid[e]] + t_emb[tb[e]] + v_emb[val[e]], left to right in
 * the table dtype. dest may be NULL (identity). With gamma != NULL the row is
 * then LayerNorm-ed (eps, gamma, beta) before it is stored (fuses
 * CrossAttentionBlock.norm_kv, cortex/models/perceiver.py:68). */
int ck_tokenize(const void* n_emb, const void* t_emb, const void* v_emb, int dtype, int32_t D,
                int64_t n_vocab, int64_t t_vocab, int64_t v_vocab, int64_t n_ld, int64_t t_ld,
                int64_t v_ld, const void* nid, const void* tb, const void* val, int idx_dtype,
                int64_t s_nid, int64_t s_tb, int64_t s_val, int64_t E, const int32_t* dest,
                const void* gamma, const void* beta, float eps, void* out, int64_t out_ld,
                void* stream);

/* Packing fused into the tokenizer: _pack_events' window offsets
 * (cortex/models/cortex.py:125-165) and the tokens in packed order in one
 * call, for contiguous tables (row stride D) and index arrays. Sorted
 * batch_indices (collate_events' layout) are packed inside the tokenizer
 * launch: tokens of event e go to row e, offsets[b] is the first event of
 * window b. A second launch checks the tokenizer blocks' flags and, when an
 * index is out of order or outside [0, B), redoes the packing as a stable
 * counting sort and tokenizes every event into its packed row (out-of-range
 * events are dropped with CK_ERR_INDEX in the status word, as ck_pack_events
 * does). offsets has B + 1 entries. workspace: at least
 * ck_tokenize_packed_workspace_bytes() bytes, contents arbitrary. Batches of
 * more than 2^20 events or 4096 windows return CK_ERR_UNSUPPORTED (use
 * ck_pack_events + ck_tokenize). */
size_t ck_tokenize_packed_workspace_bytes(void);
int ck_tokenize_packed(const void* n_emb, const void* t_emb, const void* v_emb, int dtype,
                       int32_t D, int64_t n_vocab, int64_t t_vocab, int64_t v_vocab,
                       const void* nid, const void* tb, const void* val, const void* batch_indices,
                       int idx_dtype, int64_t E, int32_t B, const void* gamma, const void* beta,
                       float eps, void* out, int64_t out_ld, int32_t* offsets, void* workspace,
                       size_t workspace_bytes, void* stream);

/* QuantizedLinear's weight (cortex/quantization/calibrate.py:225-228):
 * out[n, k] = bf16(float(w_int8[n, k]) * scale[n]), the fp32 product rounded
 * once, as (w.float() * s[:, None]).to(torch.bfloat16). w_int8 (N, K) with row
 * stride ldw, out (N, K) bf16 with row stride ldo; K a multiple of 16, both
 * 16-byte aligned (ldw a multiple of 16, ldo of 8). ck_forward applies it to
 * the INT8 linears of the self-attention blocks once per call. */
int ck_dequantize_int8(const void* w_int8, const float* scale, int64_t N, int64_t K, int64_t ldw,
                       void* out, int64_t ldo, void* stream);

/* ── 3. row norm ────────────────────────────────────────────────────────────
 * nn.LayerNorm (cortex/models/perceiver.py:51-52,97-98,143) or the RMSNorm of
 * rms_norm_linear_reference (cortex/kernels/fused_rmsnorm.py:86-108), fp32
 * statistics, output rounded to dtype. */
int ck_row_norm(const void* x, int dtype, int64_t M, int32_t D, int64_t ldx, const void* gamma,
                const void* beta, float eps, int mode, void* y, int64_t ldy, void* stream);

/* ── 4. linear ──────────────────────────────────────────────────────────────
 * y = epi(A @ W^T) for W (N,K) [nn.Linear, QuantizedLinear: cortex/quantization/
 * calibrate.py:225-228] or y = epi(A @ W) for W (K,N) [rms_norm_linear's w,
 * cortex/kernels/fused_rmsnorm.py:239]. W may be int8 with per-output-channel
 * fp32 scales (w_scale[N]); it is widened to bf16 inside the kernel and the
 * scale applied to the fp32 accumulator. bf16 problems whose strides are
 * 16-byte aligned run on the tcgen05 tensor-core kernel; fp32 problems (and
 * unaligned bf16 ones) on an fp32-accumulating CUDA-core kernel. */
int ck_linear(const void* A, int dtype, int64_t M, int64_t K, int64_t lda, const void* W,
              int w_dtype, int w_layout, int64_t N, int64_t ldw, const float* w_scale, int epi,
              const void* aux, int64_t ld_aux, int64_t aux_row_mod, void* Y, int64_t ldy,
              void* stream);

/* Norm then linear: replaces rms_norm_linear (cortex/kernels/fused_rmsnorm.py:239-301)
 * with norm_mode = CK_NORM_RMS, and LayerNorm->Linear pairs of the model with
 * CK_NORM_LAYER. RMSNorm of bf16 rows runs as ONE launch when the tensor-core
 * GEMM takes the shapes (16-byte aligned rows and gamma, K a multiple of 8) and the epilogue is
 * CK_EPI_STORE or CK_EPI_BIAS: the GEMM scales every A tile by gamma in shared
 * memory, sums x^2 per row on the way, and multiplies each output row by
 * 1 / sqrt(sum / K + eps) in its epilogue, so x is read once and no normalised
 * copy exists (the reference's kernel reads x twice, :130-233). That path
 * needs no workspace (NULL is fine). Every other call normalises into the
 * workspace (M*K elements of dtype; ck_norm_linear_workspace_bytes) and runs
 * the linear after it; it returns CK_ERR_WORKSPACE, launching nothing, when the
 * workspace is missing or too small. gamma is required. */
size_t ck_norm_linear_workspace_bytes(int dtype, int64_t M, int64_t K);
int ck_norm_linear(const void* x, int dtype, int64_t M, int64_t K, int64_t ldx, const void* gamma,
                   const void* beta, float eps, int norm_mode, const void* W, int w_dtype,
                   int w_layout, int64_t N, int64_t ldw, const float* w_scale, int epi,
                   const void* aux, int64_t ld_aux, int64_t aux_row_mod, void* Y, int64_t ldy,
                   void* workspace, size_t workspace_bytes, void* stream);

/* ck_norm_linear without a caller-provided workspace, for callers that cannot
 * allocate device memory (a host runtime binding this ABI without a CUDA
 * allocator of its own, or a serving loop that must not allocate once running).
 * No counterpart in the reference: it is an addition of this library. Calls
 * that ck_norm_linear runs as one launch need no scratch; on the two-launch
 * path the normalised activations go to a fixed 8 MiB array in device memory
 * that the library defines (held by every GPU that loads it until the process
 * exits): M*K elements of dtype must fit in CK_NORM_LINEAR_STATIC_SCRATCH_BYTES,
 * or the call returns CK_ERR_INVALID_ARG without launching anything. All calls
 * on a device share that array, so calls that overlap on the GPU race and must
 * be serialised by the caller. Each call looks the array's address up on the
 * current device; the first call on a device also loads the library's device
 * code there, so make it before any stream capture. Same arguments and results
 * as ck_norm_linear otherwise (CK_NORM_NONE runs the plain linear). */
#define CK_NORM_LINEAR_STATIC_SCRATCH_BYTES (8u << 20)
int ck_norm_linear_static(const void* x, int dtype, int64_t M, int64_t K, int64_t ldx,
                          const void* gamma, const void* beta, float eps, int norm_mode,
                          const void* W, int w_dtype, int w_layout, int64_t N, int64_t ldw,
                          const float* w_scale, int epi, const void* aux, int64_t ld_aux,
                          int64_t aux_row_mod, void* Y, int64_t ldy, void* stream);

/* ── 5. attention ───────────────────────────────────────────────────────────
 * softmax(q k^T * scale + mask) v per (batch b, head h), fp32 statistics.
 * Row r of (b, h) for tensor X in {q, k, v, o} lives at
 *   X + (b*X_rows_per_b + h*X_rows_per_h + r) * X_ld + h*X_col_per_h
 * except that with key_offsets != NULL the k/v rows of batch b start at
 * key_offsets[b] (packed varlen events, n_keys(b) = key_offsets[b+1]-key_offsets[b]).
 * key_mask (uint8, may be NULL) drops key e of batch b when key_mask[b*key_mask_ld + e]
 * is 0: the (B, 1, 1, E) bool attn_mask of cortex/models/perceiver.py:74-80.
 * block_mask (n_q_tiles x n_k_tiles, uint8, may be NULL) skips (BLOCK_L x BLOCK_E)
 * tiles as sparse_cross_attention does (cortex/kernels/sparse_xattn.py:340-434);
 * a query row with no unmasked key returns 0 (the kernel's l = 0 guard, :326-328,
 * and torch SDPA's fully-masked-row result on CPU). Replaces the SDPA calls of
 * cortex/models/perceiver.py:80,121 and cortex/models/cortex.py:49. */
typedef struct ck_attention_args {
  int dtype;
  int32_t B, H, Dh, Lq;
  int32_t n_keys;
  const int32_t* key_offsets;
  const void* q;
  int64_t q_ld, q_rows, q_rows_per_b, q_rows_per_h, q_col_per_h;
  const void* k;
  int64_t k_ld, k_rows, k_rows_per_b, k_rows_per_h, k_col_per_h;
  const void* v;
  int64_t v_ld, v_rows, v_rows_per_b, v_rows_per_h, v_col_per_h;
  void* o;
  int64_t o_ld, o_rows_per_b, o_rows_per_h, o_col_per_h;
  const uint8_t* block_mask;
  int32_t n_q_tiles, n_k_tiles, block_l, block_e;
  const uint8_t* key_mask;
  int64_t key_mask_ld;
  float scale;
} ck_attention_args;

int ck_attention(const ck_attention_args* args, void* stream);

/* ── 6. whole forward ───────────────────────────────────────────────────────
 * CortexModel.forward (cortex/models/cortex.py:90-122) for return_aux=False:
 * tokenizer + packing + Perceiver encoder + behaviour head, all on the device,
 * no host synchronisation. Weights are the module's parameters in place
 * (bf16 or fp32); QuantizedLinear layers pass int8 weights and fp32 scales. */
typedef struct ck_linear_weight {
  const void* w;       /* (N, K) */
  int dtype;           /* CK_BF16, CK_F32 or CK_I8 */
  const float* scale;  /* (N,) for CK_I8, else NULL */
  const void* bias;    /* (N,) or NULL */
} ck_linear_weight;

typedef struct ck_block_weights {
  const void *norm_attn_w, *norm_attn_b;
  ck_linear_weight qkv, out;
  const void *norm_mlp_w, *norm_mlp_b;
  ck_linear_weight mlp0, mlp2;
} ck_block_weights;

typedef struct ck_model {
  int dtype; /* CK_BF16 or CK_F32: activations and float parameters */
  int32_t hidden_dim, latent_dim, num_latents, num_layers, num_heads, head_dim;
  int32_t cross_heads, mlp_hidden, behavior_dim;
  int64_t n_vocab, t_vocab, v_vocab;
  const void *neuron_emb, *time_emb, *value_emb;
  const void* latents;
  const void *norm_q_w, *norm_q_b, *norm_kv_w, *norm_kv_b;
  ck_linear_weight cross_q, cross_kv, cross_out;
  const ck_block_weights* blocks; /* host array of num_layers entries */
  const void *final_norm_w, *final_norm_b;
  const void* head_query; /* (behavior_dim, latent_dim) */
  const void *head_norm_w, *head_norm_b;
  ck_linear_weight head_q, head_kv, head_out;
} ck_model;

/* The workspace holds the forward's intermediates and, for bf16 models whose
 * self-attention blocks carry INT8 linears, their weights dequantised to bf16
 * (bf16(float(w_int8) * scale), QuantizedLinear's rounding) once per call, on
 * which the blocks' GEMMs run. Contents arbitrary on entry. */
size_t ck_forward_workspace_bytes(const ck_model* m, int64_t E, int32_t B);
int ck_forward(const ck_model* m, const void* neuron_ids, const void* time_bins,
               const void* values, const void* batch_indices, int idx_dtype, int64_t E,
               int32_t B, void* behavior_out, void* workspace, size_t workspace_bytes,
               void* stream);

/* ── packed event batches ─────────────────────────────────────────────────
 * One batch of events in one int32 buffer, so that a batch crosses to the
 * device in a single copy and one captured launch sequence serves every batch
 * with the same (B, capacity):
 *
 *   int32 n_valid, reserved[3];
 *   int32 neuron_ids[capacity], time_bins[capacity], values[capacity],
 *         batch_indices[capacity];
 *
 * capacity is a multiple of 4, so every array starts 16-byte aligned. Events
 * n_valid..capacity-1 are padding; their entries are never read. The buffer
 * replaces the per-request list building and the four int64 tensors of
 * InferenceWorker._run_batch_sync (cortex/serve/worker.py:166-200). */
#define CK_BATCH_HEADER_WORDS 4
#define CK_BATCH_WORDS(capacity) (CK_BATCH_HEADER_WORDS + 4 * (int64_t)(capacity))

/* HOST memory only, no device work. Writes E events from four host index
 * arrays (idx_dtype CK_I32 or CK_I64, unit stride) into a batch buffer:
 * n_valid = E, ids narrowed to int32 (saturating, so an id outside int32
 * stays out of its table and the device reports CK_ERR_INDEX, where the
 * reference's embedding lookup raises), and *batch_size = max(batch_indices)
 * + 1, the B of cortex/models/cortex.py:137 (1 when E == 0). Returns
 * CK_ERR_INDEX for a negative batch index or one that does not fit int32
 * (torch.bincount rejects negative input, cortex/models/cortex.py:141). */
int ck_batch_stage(const void* neuron_ids, const void* time_bins, const void* values,
                   const void* batch_indices, int idx_dtype, int64_t E, int32_t* batch,
                   int64_t capacity, int32_t* batch_size);

/* ck_forward over a device batch buffer (16-byte aligned): capacity event
 * slots, of which the first n_valid (read on the device) are events. Size the
 * workspace with ck_forward_workspace_bytes(m, capacity, B). */
int ck_forward_batch(const ck_model* m, const int32_t* batch, int64_t capacity, int32_t B,
                     void* behavior_out, void* workspace, size_t workspace_bytes, void* stream);

/* ── native serving runner ────────────────────────────────────────────────
 * Owns, for one device: two pinned staging slots, the device batch buffer, the
 * forward workspace and one CUDA graph of ck_forward_batch per (B, capacity)
 * bucket (captured on the bucket's first batch). The one place where the
 * library allocates: ck_runner_create / the first batches of a size allocate,
 * ck_runner_destroy frees. All launches of one runner use one stream.
 *   ck_runner_stage   host index arrays -> pinned packed batch (ck_batch_stage);
 *                     B = batch_size if > 0, else max(batch_indices) + 1
 *   ck_runner_launch  one host-to-device copy, the bucket's graph, and a device
 *                     copy of the (B, behavior_dim) result to behavior_out
 *   ck_runner_launch_batch  the same from a packed batch already on the device
 *   ck_runner_invalidate    drop the graphs (and take m's weights if m != NULL)
 * Replaces the per-batch tensor building and the eager forward of
 * InferenceWorker._run_batch_sync (cortex/serve/worker.py:166-214). */
typedef struct ck_runner ck_runner;
int ck_runner_create(const ck_model* m, int32_t max_graphs, ck_runner** runner);
void ck_runner_destroy(ck_runner* runner);
int ck_runner_stage(ck_runner* runner, const void* neuron_ids, const void* time_bins,
                    const void* values, const void* batch_indices, int idx_dtype, int64_t E,
                    int32_t batch_size, int32_t* B);
int ck_runner_launch(ck_runner* runner, void* behavior_out, void* stream);
int ck_runner_launch_batch(ck_runner* runner, const int32_t* batch, int64_t capacity, int32_t B,
                           void* behavior_out, void* stream);
int ck_runner_invalidate(ck_runner* runner, const ck_model* m);
int ck_runner_counters(ck_runner* runner, long long* captures, long long* replays);

/* ── streaming K|V reuse ──────────────────────────────────────────────────
 * ck_forward split at the packed keys|values of the events, so that kv_proj
 * rows of windows seen before can come from a cache (the StreamingKVCache of
 * cortex/cache/streaming.py:79-236, wired to kv_proj outputs).
 *
 * ck_forward_kv: packing, tokenizer + norm_kv and kv_proj of a packed event
 * batch; writes kv (capacity, 2 * latent_dim) rows grouped by window (window b
 * at rows offsets[b] .. offsets[b+1]-1) and offsets (B + 1, device int32).
 * ck_forward_from_kv: the rest of the forward (latent queries, cross
 * attention over each window's rows, the self-attention stack, the head) from
 * n_rows such rows. Workspace: ck_forward_workspace_bytes(m, rows, B).
 * ck_copy_rows: segments (device int32, n x 3: src_row, dst_row, rows) copied
 * between two row buffers of src_rows / dst_rows rows of row_bytes (a
 * multiple of 16) each; a segment outside its buffer records CK_ERR_INDEX and
 * is skipped. */
int ck_forward_kv(const ck_model* m, const int32_t* batch, int64_t capacity, int32_t B, void* kv,
                  int32_t* offsets, void* workspace, size_t workspace_bytes, void* stream);
int ck_forward_from_kv(const ck_model* m, const void* kv, int64_t n_rows, const int32_t* offsets,
                       int32_t B, void* behavior_out, void* workspace, size_t workspace_bytes,
                       void* stream);
int ck_copy_rows(const void* src, int64_t src_rows, void* dst, int64_t dst_rows,
                 int64_t row_bytes, const int32_t* segments, int32_t n_segments, void* stream);

/* ── event ingest from bin-count matrices ─────────────────────────────────
 * events_from_bin_matrix + bucket_values + collate_events
 * (cortex/data/nlb.py:74-114, 249-280, 492-512) on the device: B windows of
 * window_bins rows each, every nonzero bin one event, in (window, time bin,
 * neuron) order, written as a packed event batch. */
typedef struct {
  const int32_t* counts; /* (n_rows, ld) int32 spike counts of one session, device */
  int64_t ld;            /* row stride in elements (>= n_neurons) */
  int64_t n_rows;        /* rows (time bins) of the matrix */
  int64_t start;         /* first row of the window */
  int32_t n_neurons;     /* columns (units of the session) */
  int32_t neuron_offset; /* added to the column (SessionData.neuron_id_offset) */
} ck_bin_window;

size_t ck_collate_bins_workspace_bytes(int32_t B, int32_t window_bins);
/* windows: (B,) ck_bin_window in device memory. Writes the batch (capacity
 * slots, n_valid = min(events, capacity)) and, when n_total != NULL, the
 * uncapped event count to the device int32 *n_total. Events past capacity
 * are dropped and record CK_ERR_INVALID_ARG; capacity 0 only counts (the
 * batch needs its header words only). A neuron id >= max_neurons or a window
 * outside its matrix records CK_ERR_INDEX (the window is skipped). */
int ck_collate_bins(const ck_bin_window* windows, int32_t B, int32_t window_bins,
                    int32_t n_buckets, int32_t max_neurons, int32_t* batch, int64_t capacity,
                    void* workspace, size_t workspace_bytes, int32_t* n_total, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CORTEX_B200_H_ */
