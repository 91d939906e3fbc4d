/*
 * dcinfer.h -- C ABI of the B200 verified INT8 W8A8 library (libdcinfer.so).
 *
 * The library replaces the WebGPU dispatch layer of DaisyChain-Infer
 * (public/webgpu.js) behind the same compute-core contract that
 * public/verified_core.js and public/infer.js call.  Plain C types only:
 * pointers, sizes and integer status codes.  Every pointer argument says
 * whether it is host or device memory.  A dc_ctx is bound to one CUDA device
 * and one stream and is not thread safe (the reference runs on one JS thread).
 *
 * Arithmetic contract (bit-exact with the reference CPU mirror):
 *   rows:    s[r] = f32(max(absmax/127, 1e-8)) computed in double; q uses the
 *            double scale and ECMAScript Math.round (verified_core.js:108-121)
 *   columns: s[c] = f32(max(absmax/127, 1e-8)); q uses the f32-rounded scale
 *            (verified_core.js:122-136)
 *   GEMM:    int32 sum of exact int8 products (= the mul LUT), k <= 131071,
 *            epilogue f32(f32(f32(acc) * rs[row]) * cs[col]), ReLU keeps -0
 *            (verified_core.js:227-228, 241-266)
 *   requant: out8 = requant_lut[(uint16)sat16(acc)], then relu_lut when DC_RELU
 *            (a rule this library declares; the reference defines none)
 */
#ifndef DCINFER_H
#define DCINFER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes --------------------------------------------------------- */
#define DC_OK 0
#define DC_E_ACCBOUND 1    /* AccumulatorBoundError, verified_core.js:41-49 */
#define DC_E_NONFINITE 2   /* NonFiniteError, verified_core.js:16-27 */
#define DC_E_INVAL 3       /* bad argument (shape, null pointer, range) */
#define DC_E_NOMEM 4       /* device or host allocation failed */
#define DC_E_CUDA 5        /* a CUDA runtime call failed; see dc_last_error */
#define DC_E_TIMEOUT 6     /* a bounded device wait gave up */
#define DC_E_LUT 7         /* LUT self-test or sha256 check failed (app.js:1074-1075) */
#define DC_E_GATE 8        /* init gate: a kernel disagreed with the LUT kernel (webgpu.js:470-492) */

/* ---- GEMM flags (the reference's d.relu / d.acc, plus the requant unit) ---- */
#define DC_RELU 1u         /* d.relu: v < 0 ? 0 : v after the epilogue */
#define DC_ACC 2u          /* d.acc: return the raw int32 accumulator */
#define DC_REQUANT 4u      /* int8 output through requant_lut (and relu_lut) */

#define DC_MAX_INT32_K 131071 /* floor((2^31-1)/(128*128)), verified_core.js:41 */

typedef struct dc_ctx dc_ctx;
typedef struct dc_weight dc_weight;

/* ---- context (replaces Compute.initCompute / loadLUTs, webgpu.js:247-648) --- */
/* Binds to `device`, creates a stream, builds the three LUT units, checks their
 * sha256 against the reference's LFS object ids and the mul[7,-3] == -21
 * self-test (app.js:1074-1075), uploads them, and gates every GEMM kernel
 * against the LUT kernel at the reference's gate shapes, clean and on poisoned
 * buffers (webgpu.js:470-516).  Returns DC_E_LUT / DC_E_GATE on failure. */
int dc_init(int device, dc_ctx** out);
void dc_destroy(dc_ctx* ctx);
/* compute.label (webgpu.js:616-618). */
const char* dc_backend_label(const dc_ctx* ctx);
/* Message of the last failing call on this context. */
const char* dc_last_error(const dc_ctx* ctx);
/* The context's cudaStream_t, as an opaque pointer. */
void* dc_stream(const dc_ctx* ctx);
/* Message of the last dc_init that failed on this thread (no context exists). */
const char* dc_init_error(void);
/* Run the context's work on an existing cudaStream_t (NULL = the context's own
 * stream; (void*)1 = cudaStreamLegacy, the legacy default stream).  Lets a
 * caller order the library's launches with its own work. */
int dc_set_stream(dc_ctx* ctx, void* stream);
/* Live GEMM timing: while on, every GEMM launch is bracketed by CUDA events on
 * its stream.  dc_timing(ctx, 1) resets and starts, dc_timing(ctx, 0) stops;
 * dc_timing_read sums the launches of one kernel kind (1 GEMV, 2 SIMT dp4a,
 * 3 tcgen05): total device ms, launch count, algorithmic bytes
 * (M·K + K·N + 4M + 4N + output) and ops (2·M·N·K). */
int dc_timing(dc_ctx* ctx, int on);
int dc_timing_read(dc_ctx* ctx, int kind, double* ms, long long* launches, double* bytes, double* ops);
/* Number of kernels this library has launched in this process (all contexts). */
unsigned long long dc_launch_count(void);
/* 1 when the tcgen05 tensor-core GEMM passed its init gate and is in use. */
int dc_tc_enabled(const dc_ctx* ctx);
/* Copy the LUT units out (host buffers of 65536 int16, 65536 int8, 256 int8). */
int dc_luts(const dc_ctx* ctx, int16_t* mul, int8_t* requant, int8_t* relu);
/* Wait for the context's stream; report (and clear) a device-side status such
 * as a non-finite input seen by a quantiser. */
int dc_sync(dc_ctx* ctx);

/* ---- the GEMM unit (compute.bgemm, webgpu.js:836-857) ------------------------
 * Host buffers, exactly the reference's argument meaning:
 *   Xq (batch*m) x k int8 row-major, Wq batch x (k x n) int8 row-major,
 *   rs[batch*m], cs[batch*n] f32.  out is int32 (DC_ACC), int8 (DC_REQUANT) or
 *   f32, (batch*m) x n row-major, owned by the caller.
 * Refuses k > 131071 with DC_E_ACCBOUND before any launch (webgpu.js:838). */
int dc_bgemm(dc_ctx* ctx, const int8_t* Xq, const int8_t* Wq, const float* rs, const float* cs, int m, int k, int n,
             int batch, unsigned flags, void* out);

/* Device-resident variant.  Wt is the weight in the library's layout: per batch
 * n rows of ldw bytes (K-major, i.e. Wᵀ), zero past k; Xq is (batch*m) rows of
 * ldx bytes, zero past k.  ldw and ldx are multiples of 16.  Asynchronous on the
 * context's stream. */
int dc_bgemm_dev(dc_ctx* ctx, const int8_t* Xq, int ldx, const int8_t* Wt, int ldw, const float* rs, const float* cs,
                 int m, int k, int n, int batch, unsigned flags, void* out);

/* dc_bgemm_dev with one kernel forced (1 GEMV, 2 SIMT dp4a, 3 tcgen05), for the
 * init gates and the parity tests; DC_E_INVAL when that kernel cannot take the
 * shape. */
int dc_bgemm_dev_kind(dc_ctx* ctx, const int8_t* Xq, int ldx, const int8_t* Wt, int ldw, const float* rs,
                      const float* cs, int m, int k, int n, int batch, unsigned flags, void* out, int kind);

/* dc_bgemm_dev without any device allocation (no counterpart in the reference).
 * For callers that cannot let the library call cudaMalloc/cudaFree behind their
 * back: a host that sizes all of HBM up front, a runtime that owns device
 * allocation, or a process whose other streams must not be stalled by the device
 * synchronisation cudaFree implies.  Same arguments, kernels and results as
 * dc_bgemm_dev (k == 0 gives zero accumulators; the SIMT kernel runs when the
 * tcgen05 kernel failed its init gate or cannot take the operands), but the
 * tcgen05 kernel's split-K scratch is a fixed array inside the library
 * (DC_NOALLOC_MAX_OUT int32 + DC_NOALLOC_MAX_TILES counters, about 4.2 MB held
 * on every GPU that loads the library); outputs of more than DC_NOALLOC_MAX_OUT
 * elements (batch*m*n) are refused with DC_E_INVAL.  A call that splits K
 * clears the scratch it uses first; calls that overlap on one GPU race on the
 * shared array.  The first call on a context looks up the array's address with
 * the context's device current: make it before any stream capture. */
#define DC_NOALLOC_MAX_OUT (1 << 20)
#define DC_NOALLOC_MAX_TILES 4096
int dc_bgemm_dev_noalloc(dc_ctx* ctx, const int8_t* Xq, int ldx, const int8_t* Wt, int ldw, const float* rs,
                         const float* cs, int m, int k, int n, int batch, unsigned flags, void* out);

/* Same contraction through the LUT kernel (every product looked up in the mul
 * unit, the reference's WGSL_BG_LUT twin).  Reference-layout device buffers. */
int dc_bgemm_lut_dev(dc_ctx* ctx, const int8_t* Xq, const int8_t* Wq, const float* rs, const float* cs, int m, int k,
                     int n, int batch, unsigned flags, void* out);

/* ---- quantisers (verified_core.js:108-136), device buffers ----------------- */
/* X rows x cols f32 -> q rows x ldq int8 (zero past cols), s[rows] f32. */
int dc_quantize_rows(dc_ctx* ctx, const float* X, int rows, int cols, int8_t* q, int ldq, float* s);
/* W rows x cols f32 (k x n) -> qt cols x ldq int8 = quantised Wᵀ (zero past
 * rows), s[cols] f32.  Asynchronous; a non-finite input is reported by dc_sync. */
int dc_quantize_cols_t(dc_ctx* ctx, const float* W, int rows, int cols, int8_t* qt, int ldq, float* s);

/* ---- resident weights (vgemmBlock's per-call quantizeCols, done once) ------- */
/* W is k x n f32 row-major in HOST memory (the reference's layout after
 * toKN, shard.js:70-76).  Quantised once on the device: bit-identical to the
 * reference re-quantising it on every call (verified_core.js:430). */
int dc_weight_register(dc_ctx* ctx, const float* W, int k, int n, dc_weight** out);
void dc_weight_free(dc_weight* w);
/* Device pointers and leading dimension of a registered weight. */
int dc_weight_info(const dc_weight* w, const int8_t** qt, int* ldw, const float** cs, int* k, int* n);

/* vgemmBlock (verified_core.js:425-449) with a registered weight, device
 * buffers: out (m x n f32) = epilogue(quantizeRows(X) x W).  Asynchronous. */
int dc_vgemm(dc_ctx* ctx, const float* X, int m, const dc_weight* w, unsigned flags, void* out);

/* ---- row operations of the layer forward, device buffers ---------------------
 * The stage kernels' own math, callable on its own (asynchronous; non-finite
 * input is reported by dc_sync).
 * dc_ordered_sum_dev: out[r] = the serial double sum of terms[r*n .. r*n+n) in
 *   index order, each add rounded to nearest even -- the chains of infer.js
 *   rmsnorm (:73-76) and softmax (:100-104), computed by a block in parallel
 *   and bit-identical to the serial loop for every input.
 * dc_rmsnorm_dev: y = infer.js rmsnorm (:70-80) of each of `rows` rows of
 *   `cols` floats with weight w (cols * 12 bytes must fit on chip: cols <=
 *   17066).  The serial sum of squares is first bracketed (any-order sum and
 *   its error bound); exact_sum = 1 always computes the serial-order sum
 *   instead -- both give the same bits. */
int dc_ordered_sum_dev(dc_ctx* ctx, const double* terms, int rows, int n, double* out);
/* dc_exp_dev: y[i] = Math.exp(x[i]) by the fdlibm method (infer.js:59, :192):
 *   sel = 0 its branching form, sel = 1 the branch-free form the softmax and
 *   SiLU kernels evaluate (the same bits for every argument); sel = 2 the
 *   table-driven exp the chunk softmax evaluates first (not fdlibm's bits:
 *   within 2^-51 relative of them for -700 <= x <= 0), sel = 3 the f32
 *   rounding of fdlibm's value as the chunk softmax settles it (as a double);
 *   sel = 4, 5 the SwiGLU value f32(silu(g) * u) (infer.js:59, :212) of
 *   g = f32(x), u = f32(x / 2 + 1/4), as the SwiGLU kernel settles it and by
 *   the exact chain. */
int dc_exp_dev(dc_ctx* ctx, const double* x, int n, double* y, int sel);
int dc_rmsnorm_dev(dc_ctx* ctx, const float* x, int rows, int cols, const float* w, double eps, float* y,
                   int exact_sum);

/* Prefetch [p, p + bytes) of device memory into L2 (16-byte aligned range),
 * asynchronously on the context's stream.  No counterpart in the reference; a
 * host may warm a buffer it is about to use (the stage forward does not call
 * it: issuing the prefetch cost more than it saved on the layer loop). */
int dc_l2_prefetch(dc_ctx* ctx, const void* p, size_t bytes);

/* ---- kernel probe (webgpu.js:998-1060) --------------------------------------
 * Runs the seeded probe GEMM (m=24 k=96 n=24 batch=2, acc) through the live
 * kernels; returns the FNV-1a of the int32 result (before the reference folds in
 * its transcendental hash, which needs V8). */
int dc_kernel_probe(dc_ctx* ctx, uint32_t* hash);

/* FNV-1a (32-bit) of n bytes of host memory: shard.js fnv1a (:195-200), the
 * actHash of an activation frame (wire.js packAct :106-112, over the f32
 * payload's bytes) and the model fingerprint (shard.js:206-213).  Host-only;
 * needs no context. */
uint32_t dc_fnv1a(const void* p, size_t n);

/* ---- pipeline stages (public/infer.js, Llama family) -------------------------
 * A stage owns layers [layer_lo, layer_hi) of one model (shard.js planStages
 * :32-52) with every weight quantised once and resident in HBM, RoPE tables,
 * and a KV cache of max_pos positions per layer; the head stage (head = 1)
 * also owns the embedding, the final norm and lm_head.  Field names follow
 * arch.js fromConfig (:50-71). */
typedef struct dc_spec {
  int hidden, layers, heads, kv_heads, head_dim, inter, vocab;
  double norm_eps, rope_theta;
  int tie; /* lm_head = embᵀ */
} dc_spec;
typedef struct dc_stage dc_stage;

int dc_stage_create(dc_ctx* ctx, const dc_spec* spec, int layer_lo, int layer_hi, int head, int max_rows,
                    int max_pos, dc_stage** out);
void dc_stage_free(dc_stage* stage);
/* Host f32 weights in the reference's k x n (in x out) layout (shard.js toKN :70-76). */
int dc_stage_set_layer(dc_stage* stage, int layer, const float* nrm1, const float* nrm2, const float* Wq,
                       const float* Wk, const float* Wv, const float* Wo, const float* Wgate, const float* Wup,
                       const float* Wdown);
/* emb vocab x hidden, nrmF hidden, lm_kn hidden x vocab or NULL when tied (shard.js:84-94). */
int dc_stage_set_head(dc_stage* stage, const float* emb, const float* nrmF, const float* lm_kn);
/* Synthetic random-init weights generated on the device: counter-based, each
 * element the scaled, centred sum of four splitmix64 draws (norm weights 1). */
int dc_stage_synth(dc_stage* stage, uint64_t model_seed, double factor);
/* embedRows (infer.js:298-310): ids (device int32) -> x (device, T x hidden). */
int dc_stage_embed(dc_stage* stage, const int32_t* ids, int T, float* x);
/* runLayers (use_kv = 0: the full window, positions 0..T-1, infer.js:275-283) or
 * runLayersChunk (use_kv = 1: positions pos0.., keys and values appended to the
 * stage's cache, infer.js:288-296); x (device, T x hidden) is updated in place.
 * Asynchronous: a non-finite activation is reported by dc_sync as DC_E_NONFINITE. */
int dc_stage_forward(dc_stage* stage, float* x, int T, int pos0, int use_kv);
/* runLayersChunk (infer.js:288-296) on nchunks consecutive chunks in one pass
 * over the stage's weights, as generateChunked calls it once per chunk
 * (infer.js:339-367; app.js:877-923 keeps two chunks in flight per ring).
 * rows (host ints) holds the chunks' lengths, summing to T <= max_rows, in
 * position order from pos0 (the cached length); x (device, T x hidden) is
 * updated in place.  The result and the cache are bit-identical to one
 * dc_stage_forward(use_kv = 1) per chunk: each chunk's attention context uses
 * the value channel scales as of its own last row.  Chunks of up to 16 rows,
 * nchunks <= min(DC_MAX_CHUNKS, max_rows) share the weight pass; otherwise the
 * chunks run one by one. */
#define DC_MAX_CHUNKS 32
int dc_stage_forward_chunks(dc_stage* stage, float* x, int T, int pos0, const int* rows, int nchunks);
/* The attention kernel of a pass of several chunks: mode 0 (the default) one
 * CTA per (head, chunk) for the chunk's rows when those CTAs fill half the SMs
 * or more, else one CTA per (head, row) and one per (head, 32 channels);
 * 1 the former whenever it fits, 2 never.  The results are identical. */
int dc_stage_set_pass_attention(dc_stage* stage, int mode);
/* A cached one-row forward (use_kv = 1, T = 1: a decode step of a pipeline
 * stage) runs as a CUDA graph of the stage's layers, captured on first use
 * (the default).  on = 0 launches the kernels one by one instead; the results
 * are identical. */
int dc_stage_set_row_graph(dc_stage* stage, int on);
/* One-row cached forwards (decode steps, and the head's logits in
 * dc_decode_run) run their GEMVs with the neighbouring row operations fused
 * into them (the default): the RMSNorm before the QKV and gate/up projections
 * and before lm_head, the SwiGLU after gate/up, the down projection's row
 * quantisation.  on = 0 runs those as separate kernels; the results are
 * identical (the same arithmetic, infer.js:30-39, 59, 199-219). */
int dc_stage_set_row_fusion(dc_stage* stage, int on);
/* logitsAt (infer.js:324-334) for rows[0..nrows) (host ints, nrows <= 8):
 * logits (device, nrows x vocab) and the greedy pick of each row (device int32,
 * may be NULL), first maximum wins (infer.js:393-395). */
int dc_stage_logits(dc_stage* stage, const float* x, int T, const int32_t* rows, int nrows, float* logits,
                    int32_t* picks);
/* The chunked-decode loop (infer.js:353-365, app.js:907-921) for stages[0..ns)
 * sharing one context (stages[0] the head): n_new laps, each the greedy pick of
 * the previous lap's hidden row, its embedding, and runLayersChunk on every
 * stage.  x_last (device) is the hidden row the first pick reads (the last row
 * of the prefill output); picks (device int32[n_new]) receive the ids, which
 * never leave the device between laps.  use_graph = 1 captures one lap as a
 * CUDA graph (kernel positions live in device memory) and replays it. */
int dc_decode_run(dc_stage** stages, int ns, const float* x_last, int n_new, int32_t* picks, int use_graph);
/* Decode-lap timeline (a measurement aid; no counterpart in the reference).
 * With buf set (device memory, laps x per_lap uint64) on the head stage,
 * dc_decode_run stamps %globaltimer at the start of each lap and after every
 * launch of it, into buf[lap * per_lap + i] (lap = index within the call; the
 * first per_lap launches and the first laps laps only), with a one-thread
 * kernel after each launch, which lengthens a lap by one or two microseconds
 * per launch; per_lap = 0 turns it off.  dc_stage_timeline_info copies out,
 * for stamp i, the kind of the launch it closes (1 one-row GEMV, 3 tcgen05
 * GEMM, 0 other) and that GEMM's algorithmic bytes, and returns the stamps
 * per lap of the last lap enqueued. */
int dc_stage_set_timeline(dc_stage* head, unsigned long long* buf, int per_lap, int laps);
int dc_stage_timeline_info(const dc_stage* head, int* kinds, double* bytes, int cap);
/* The activation hop between pipeline stages (app.js:705-765, the act message
 * of wire.js:106-138): T rows of hidden floats from x_src (device memory of
 * src's GPU) to x_dst (device memory of dst's GPU), ordered after the work
 * already issued for src and before any later work issued for dst (a peer
 * copy over NVLink between devices, a device copy on one).  Asynchronous. */
int dc_stage_handoff(dc_stage* src, dc_stage* dst, const float* x_src, float* x_dst, int T);
/* The chunk path's cache: reset, and the number of cached tokens. */
int dc_stage_kv_reset(dc_stage* stage);
int dc_stage_kv_len(const dc_stage* stage);
/* Copy one layer's cache to host buffers: int8 keys [kv_heads][len][head_dim],
 * key scales [kv_heads][len], f32 values [len][kv_heads*head_dim] (any may be NULL). */
int dc_stage_kv_read(dc_stage* stage, int layer, int8_t* k8, float* ks, float* v);

#ifdef __cplusplus
}
#endif
#endif
