/*
 * snl_b200.h - C ABI of the B200 (sm_100a) decode/prefill path of sensenova-loop.
 *
 * This library replaces the wgpu layer of the reference (src/gpu.rs) and the WGSL
 * kernels it dispatches (src/shaders/{matmul,linear,attention,layers}.wgsl). Two
 * levels are exported:
 *
 *   - Kernel level: one entry point per WGSL entry point, taking the same parameter
 *     structs as the reference's uniforms (byte-identical to the #[repr(C)] structs of
 *     src/engine.rs:24-82) plus device pointers and a cudaStream_t (passed as void*).
 *     A caller such as src/vision.rs, which records Kernels::matmul itself, binds here.
 *   - Engine level: an opaque snl_engine owning all device memory (weights, caches,
 *     activations), with the methods of the reference's Engine (src/engine.rs:229-949).
 *
 * Conventions
 *   - Every function returns 0 (SNL_OK) or a negative SNL_E_* code. The message of the
 *     last failure on the calling thread is returned by snl_last_error().
 *   - Device pointers are CUDA global-memory addresses on the current device; host
 *     pointers are plain process memory. No function keeps a caller pointer after it
 *     returns.
 *   - An snl_engine is not thread-safe: one owner thread drives it (the reference's
 *     Engine is !Sync and lives on the "generation" thread, src/worker.rs:76-106).
 */
#ifndef SNL_B200_H
#define SNL_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The library is built with hidden visibility; everything declared here is exported. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* ---- codes ------------------------------------------------------------------ */

/* Weight dtypes, in the order of weights.rs:25-30 (DType::{F32, Q8_0, Q4_0}). */
enum { SNL_F32 = 0, SNL_Q8_0 = 1, SNL_Q4_0 = 2 };

enum {
  SNL_OK = 0,
  SNL_E_INVALID = -1,     /* bad argument or unsupported request                  */
  SNL_E_RANGE = -2,       /* token id / context / row out of range               */
  SNL_E_CUDA = -3,        /* a CUDA runtime error                                */
  SNL_E_OOM = -4,         /* device allocation failed                            */
  SNL_E_STATE = -5,       /* call not valid in the engine's current state        */
  SNL_E_TIMEOUT = -6,     /* a bounded device-side wait gave up                  */
  SNL_E_UNSUPPORTED = -7, /* model configuration the kernels are not built for   */
  SNL_E_NCCL = -8         /* a tensor-parallel collective failed                 */
};

/* ---- parameter structs (byte-identical to src/engine.rs) ---------------------- */

/* StepU, src/engine.rs:24-32: rows in this step, first cache position, split-K
 * parts of decode attention, and ckpt > 0 = save linear state after token ckpt-1. */
typedef struct snl_step_u {
  uint32_t m, pos0, parts, ckpt;
} snl_step_u;

/* MatP, src/engine.rs:34-45 (matmul.wgsl:18-27). Offsets/strides in floats. */
typedef struct snl_mat_p {
  uint32_t n, k, x_off, x_stride, y_off, y_stride, n_off, m_one;
} snl_mat_p;

/* LayerP, src/engine.rs:47-58 (layers.wgsl:154-163). */
typedef struct snl_layer_p {
  uint32_t h, mode, last_row;
  float eps, weight_one;
  uint32_t iterations, inter, x_stride;
} snl_layer_p;

/* AttnP, src/engine.rs:60-71 (attention.wgsl:17-29). */
typedef struct snl_attn_p {
  uint32_t n_heads, n_kv, rot_dim, proj_stride;
  float rope_theta, eps, scale;
  uint32_t mrope;
} snl_attn_p;

/* LinP, src/engine.rs:73-82 (linear.wgsl:13-22). */
typedef struct snl_lin_p {
  uint32_t conv_dim, proj_stride, n_k, n_v;
  float eps;
  uint32_t pad[3];
} snl_lin_p;

/* ModelConfig, src/config.rs:7-37 (text part). mhc_start < 0 means no mHC.
 * full_attention[i] != 0 marks layer i as a gated full-attention layer. */
#define SNL_MAX_LAYERS 256
typedef struct snl_model_config {
  uint32_t hidden, intermediate, vocab, n_layers;
  uint8_t full_attention[SNL_MAX_LAYERS];
  uint32_t n_heads, n_kv_heads, head_dim, rot_dim;
  float rope_theta;
  uint32_t mrope_section[3];
  uint32_t lin_k_heads, lin_v_heads, lin_k_dim, lin_v_dim, conv_kernel;
  float eps;
  uint32_t loop_start, loop_end, loop_count;
  int32_t mhc_start, mhc_end;
  uint32_t mhc_streams, mhc_iterations;
  uint32_t max_position;
} snl_model_config;

/* ---- errors ------------------------------------------------------------------ */

/* Message of the last failed call on this thread ("" if none). Replaces the
 * anyhow::bail! strings of engine.rs (e.g. "context length exceeded (a > b)"). */
const char* snl_last_error(void);

/* Library version string, and the number of kernel launches the library has issued
 * on the calling process (a launch counter for measurement). */
const char* snl_version(void);
uint64_t snl_launch_count(void);

/* Device error word of the current device: bit 0 = a bounded device-side wait on an
 * asynchronous copy gave up, bit 1 = a tensor-parallel peer did not answer within the
 * wait bound (the kernel returned instead of hanging). Returns the word (>= 0), clearing
 * it when clear != 0, or a negative code. The engine calls (forward_mm, forward_greedy,
 * mtp, generate) read it themselves: a set word makes them fail with SNL_E_TIMEOUT and
 * clears it. */
int snl_device_error(int clear);

/* ModelConfig::validate (src/config.rs:194-240). */
int snl_config_validate(const snl_model_config* cfg);

/* ---- kernel level: matmul.wgsl ------------------------------------------------ */

/* y[m, y_off + m*y_stride + n_off + row] = sum_k x[x_off + m*x_stride + k] * W[row, k]
 * for m < rows_m (m_one > 0 ? m_one : step->m). Replaces the 8 pipelines of
 * Kernels::mat (src/gpu.rs:221-234, :377-382) with the MatKind choice of
 * src/gpu.rs:211-218 made on the host. wq/ws are the reference layout
 * (weights.rs:48-55): Q8_0 int8 [n, k] + f32 scales [n, k/32]; Q4_0 packed u32
 * [n, k/8] + f32 scales [n, k/32]. */
int snl_mat(int dtype, const snl_step_u* step, const snl_mat_p* p, const float* x, const void* wq,
            const float* ws, float* y, void* stream);
/* Weight planes of a Q8_0/Q4_0 matrix for the prefill GEMM: planes [2][n][k] fp16 (4 n k
 * bytes), the hi and lo parts of each dequantized value (x 256). snl_mat_wplanes is
 * snl_mat with them: steps of >= 8 rows then load the weights by TMA instead of
 * dequantizing them; the results are the same. The engine keeps planes for every
 * matrix when device memory allows. */
int snl_weight_planes(int dtype, uint32_t n, uint32_t k, const void* wq, const float* ws, void* planes, void* stream);
int snl_mat_wplanes(int dtype, const snl_step_u* step, const snl_mat_p* p, const float* x, const void* wq,
                    const float* ws, const void* planes, float* y, void* stream);

/* The same product on the tensor cores for 1..4 token rows, with x given as "x planes":
 * [2*rows_m][k] fp16, plane 2t = hi and 2t+1 = lo of x[t]/16 (written by snl_xpack or by
 * the engine's producer kernels). y as snl_mat (y_off, y_stride, n_off); x_off and
 * x_stride of p are unused. */
int snl_xpack(const float* x, uint32_t m, uint32_t k, uint32_t x_stride, void* planes, void* stream);
int snl_mat_xpack(int dtype, const snl_mat_p* p, uint32_t rows_m, const void* planes, const void* wq,
                  const float* ws, float* y, void* stream);

/* Tile layout of a Q8_0/Q4_0 matrix for the decode GEMV: 16-row groups, one 512-byte
 * (Q8) or 256-byte (Q4) tile per 32-element block holding each MMA lane's fragment
 * bytes contiguously, plus grouped block scales. The same values as the file layout in
 * another order (weights.rs:48-55 is the source). snl_tile_sizes gives the buffer sizes
 * in bytes (scales sized for f32). snl_tile_repack converts on the device and waits for
 * it; it keeps the scales as fp16 when every block scale is an fp16 number
 * (*scales_f16 = 1), else as f32 (*scales_f16 = 0). snl_mat_tiles is snl_mat_xpack on
 * the tile layout, given that mode. */
int snl_tile_sizes(int dtype, uint32_t n, uint32_t k, size_t* tile_bytes, size_t* scale_bytes);
int snl_tile_repack(int dtype, uint32_t n, uint32_t k, const void* q, const float* s, void* tiles,
                    void* tile_scales, int* scales_f16, void* stream);
int snl_mat_tiles(int dtype, const snl_mat_p* p, uint32_t rows_m, const void* planes, const void* tiles,
                  const void* tile_scales, int scales_f16, float* y, void* stream);

/* ---- kernel level: layers.wgsl ------------------------------------------------- */

/* branch_norm (layers.wgsl:49-76): n_groups workgroups (step->m, or 1 for the
 * final-row norm). x, coef, w, out as the WGSL bindings. */
int snl_branch_norm(const snl_step_u* step, const snl_layer_p* p, const float* x, const float* coef,
                    const float* w, float* out, uint32_t n_groups, void* stream);
/* mhc_dots (layers.wgsl:78-95): grid (9, step->m); writes raw[m*9 + o]. */
int snl_mhc_dots(const snl_step_u* step, const snl_layer_p* p, const float* x, const float* w,
                 float* raw, void* stream);
/* mhc_finish (layers.wgsl:97-132): coef[m*8 + 0..8] from raw and the router bias. */
int snl_mhc_finish(const snl_step_u* step, const snl_layer_p* p, const float* raw, const float* w,
                   float* coef, void* stream);
/* merge (layers.wgsl:134-164): width = h; modes 0..3. */
int snl_merge(const snl_step_u* step, const snl_layer_p* p, float* x, const float* coef,
              const float* branch, void* stream);
/* swiglu (layers.wgsl:166-175): act[m, i] = silu(gate_up[m, i]) * gate_up[m, I + i]. */
int snl_swiglu(const snl_step_u* step, const snl_layer_p* p, const float* gate_up, float* act,
               void* stream);

/* ---- kernel level: attention.wgsl ---------------------------------------------- */

/* prep (attention.wgsl:59-127): q/k RMSNorm(1+w), partial rotate-half M-RoPE, q to
 * qbuf [m, n_heads*256], k/v as f16 pairs into the caches at position pos0+m.
 * rpos is [m][4] u32 (t, h, w, 0). */
int snl_attn_prep(const snl_step_u* step, const snl_attn_p* p, const float* proj, float* qbuf,
                  uint32_t* kcache, uint32_t* vcache, const float* norms, const uint32_t* rpos,
                  void* stream);
/* attend (attention.wgsl:129-246): causal GQA (4 query heads per KV head) over the f16
 * cache, split into step->parts parts. parts == 1: gated output to out [m, q_dim];
 * otherwise partials [(m*n_heads + h)*parts + part][258] to partial. */
int snl_attend(const snl_step_u* step, const snl_attn_p* p, const float* proj, const float* qbuf,
               const uint32_t* kcache, const uint32_t* vcache, float* out, float* partial,
               void* stream);
/* combine (attention.wgsl:248-269): merge split-K partials and apply the gate. */
int snl_attn_combine(const snl_step_u* step, const snl_attn_p* p, const float* proj,
                     const float* partial, float* out, void* stream);

/* ---- kernel level: linear.wgsl -------------------------------------------------- */

/* conv (linear.wgsl:38-66): causal depthwise conv(4) + SiLU over the qkv channels of
 * proj, carrying conv_state [3, conv_dim]; step->ckpt > 0 also saves the state after
 * token ckpt-1 into conv_ckpt. lw = conv w [conv_dim*4] | A_log | dt_bias | norm. */
int snl_conv(const snl_step_u* step, const snl_lin_p* p, const float* proj, float* conv_out,
             float* conv_state, const float* lw, float* conv_ckpt, void* stream);
/* delta (linear.wgsl:84-140): gated delta rule over the tokens of the step plus the
 * gated RMSNorm; state [n_v, 128, 128] f32 (row i = key dim, column j = value dim). */
int snl_delta(const snl_step_u* step, const snl_lin_p* p, const float* proj, const float* conv_out,
              float* state, const float* lw, float* out, float* state_ckpt, void* stream);
/* conv followed by delta in one kernel, the engine's form: no conv_out buffer; the
 * first value head of each key-head group owns that group's q/k conv state. Same
 * arguments and results as snl_conv then snl_delta. */
int snl_conv_delta(const snl_step_u* step, const snl_lin_p* p, const float* proj, float* conv_state, float* state,
                   const float* lw, float* out, float* conv_ckpt, float* state_ckpt, void* stream);

/* ---- kernel level: sampling ----------------------------------------------------- */

/* Greedy argmax of each of `rows` rows of `n` logits (sampler.rs:169-177: the first
 * maximum wins, -0.0 ties with +0.0, NaN never wins except that a row whose element 0
 * is NaN gives 0, as the reference's scan does); out_idx is a device u32[rows]. */
int snl_argmax(const float* logits, uint32_t rows, uint32_t n, uint32_t* out_idx, void* stream);

/* snl_argmax for callers that must not allocate device memory when they call it (no
 * counterpart in the reference): a host whose device memory is reserved by its own
 * pool allocator, or a serving loop that cannot take the device-wide wait of a free.
 * Same arguments and results as snl_argmax; it calls no cudaMalloc, cudaFree or other
 * allocating routine. Its scratch is a static 16 KB device array per GPU, so rows must
 * be <= 16 (SNL_E_RANGE otherwise). The first call on a device looks up that array's
 * address (cudaGetSymbolAddress) with the device current; make that first call before
 * any stream capture. The address is kept for the life of the process, which assumes
 * one CUDA context per device: do not call it again after cudaDeviceReset. All calls
 * share the array: calls that overlap on the GPU (for example on two streams at once)
 * race and must be serialised by the caller. */
int snl_argmax_noalloc(const float* logits, uint32_t rows, uint32_t n, uint32_t* out_idx, void* stream);

/* SamplingParams (sampler.rs:4-14) without the seed: the host keeps the random number
 * generator and passes its uniform draws. */
typedef struct snl_sample_p {
  float temperature, top_p;
  uint32_t top_k;
  float min_p, presence_penalty, frequency_penalty, repetition_penalty;
  uint32_t pad;
} snl_sample_p;

/* Sampler::sample (draft < 0) or Sampler::verify(draft) (sampler.rs:54-167) on the device,
 * for one row of n logits (device, f32; the penalties modify it in place, as the
 * reference modifies its slice). hist_tok / hist_cnt: device arrays of the n_hist tokens
 * generated so far and their counts (Sampler::counts). u: two host uniform draws in
 * [0, 1) from the caller's generator, used in the reference's order: sample uses u[0] for
 * the draw; verify uses u[0] for the acceptance test when p(draft) > 0 and the next one
 * for the redraw. out: device u32[3] = token, accepted (1/0), draws used (0-2).
 * scratch: snl_sample_scratch_bytes() of device memory. Supported: temperature <= 1e-5
 * (greedy), or top_k in 1..256 (the reference's top_k_small branch, which ranks equal
 * logits by index); top_k 0 or > 256 returns SNL_E_UNSUPPORTED, and n <= 262144. */
int snl_sample(const snl_sample_p* p, float* logits, uint32_t n, const uint32_t* hist_tok, const uint32_t* hist_cnt,
               uint32_t n_hist, const float* u, int64_t draft, uint32_t* out, void* scratch, void* stream);
size_t snl_sample_scratch_bytes(void);
/* ---- seeded synthetic tensors ------------------------------------------------------- */

/* Fill device buffers with tensor `name` of the seeded synthetic model (the benchmark
 * weights; no reference counterpart): quants (Q8_0: rows*cols bytes, Q4_0: rows*cols/2)
 * and f32 scales (rows*cols/32), or f32 values offset + mult * z for segment `sub`. */
int snl_synth_quant(uint64_t seed, const char* name, int dtype, size_t rows, size_t cols, void* q,
                    float* s, void* stream);
int snl_synth_f32(uint64_t seed, const char* name, uint32_t sub, size_t n, float mult, float offset,
                  float* out, void* stream);

/* ---- engine level (src/engine.rs) ----------------------------------------------- */

typedef struct snl_engine snl_engine;

/* Engine::load without the file part (src/engine.rs:230-644): validate cfg, pick the
 * device, record the configuration. Weights are then given tensor by tensor
 * (snl_engine_set_tensor, the upload_q/upload_f of engine.rs:91-113) or generated
 * (snl_engine_fill_synthetic), and snl_engine_finalize allocates caches and
 * activations and builds the op graph. ctx is clamped to cfg->max_position.
 * flags: SNL_ENGINE_MTP = also expect the MTP head tensors ("mtp.*"). */
#define SNL_ENGINE_MTP 1u
#define SNL_ENGINE_F16_SCALES 2u /* store fp16 block scales where every scale is fp16-exact */
int snl_engine_create(const snl_model_config* cfg, size_t ctx, int device, uint32_t flags,
                      snl_engine** out);

/* Tensor parallelism over 2, 4 or 8 GPUs of one node: one process (and one engine) per
 * GPU, all driven through the same call sequence, as the reference's single Engine is.
 * (The reference has no tensor parallelism. A create call taking (tp_rank, tp_size,
 * nccl_id) was the obvious shape; the rendezvous here is CUDA IPC instead of an NCCL id.)
 * The in-projections and the LM head are split by output rows (qkv by head, in_proj by
 * key/value head, gate_up by intermediate slice, lm_head by vocabulary). The
 * out-projections are split by K, and their partial sums are added across GPUs over
 * NVLink inside the projection kernel. Norms, mHC and the embedding are replicated.
 * Steps:
 *   1. snl_engine_create_tp on every rank;
 *   2. snl_engine_tp_handle; all-gather the SNL_TP_HANDLE_BYTES-byte handles in rank
 *      order (e.g. with torch.distributed);
 *   3. snl_engine_tp_connect with the gathered handles;
 *   4. set_tensor / fill_synthetic with the FULL tensors; finalize keeps this rank's
 *      shard.
 * forward_mm returns the full logits row on every rank; forward_greedy returns the same
 * token on every rank. With tp_size == 1 this is snl_engine_create. The MTP layer is
 * replicated (every rank runs it in full) and its head is the vocabulary-split LM head:
 * snl_engine_mtp returns the same draft on every rank, and every rank must make the same
 * mtp calls in the same order as its forward calls.
 * Every cross-GPU wait is bounded: 2 s, or SNL_TP_WAIT_MS milliseconds when that
 * environment variable is set at finalize. When a peer stops taking part, the waiting
 * rank's call returns SNL_E_TIMEOUT after about one bound (later waits of the device give
 * up at once); the engines of every rank must then be destroyed and created again. */
#define SNL_TP_HANDLE_BYTES 64
/* The shard a rank keeps of one named tensor (what finalize applies): kind
 * SNL_TP_FULL (replicated), SNL_TP_ROWS (the listed row ranges of a matrix, in order),
 * SNL_TP_COLS (one column range) or SNL_TP_ELEMS (element ranges of an f32 vector).
 * ranges receives n_ranges (start, count) pairs; cap is its capacity in pairs. */
#define SNL_TP_FULL 0
#define SNL_TP_ROWS 1
#define SNL_TP_COLS 2
#define SNL_TP_ELEMS 3
int snl_tp_plan(const snl_model_config* cfg, int tp_rank, int tp_size, const char* name, int* kind, size_t* ranges,
                size_t cap, size_t* n_ranges);
int snl_engine_create_tp(const snl_model_config* cfg, size_t ctx, int device, uint32_t flags, int tp_rank,
                         int tp_size, snl_engine** out);
int snl_engine_tp_handle(snl_engine* e, void* handle_out);
int snl_engine_tp_connect(snl_engine* e, const void* handles);

/* One tensor of a .snl file (weights.rs:76-104 names and layout): dtype SNL_F32 with
 * rows*cols floats in q (s unused), or Q8_0/Q4_0 with the packed quants in q and the
 * f32 scales in s. Host pointers. */
int snl_engine_set_tensor(snl_engine* e, const char* name, int dtype, size_t rows, size_t cols,
                          const void* q, const void* s);

/* Generate every tensor of the configuration from `seed` on the device (the seeded
 * synthetic model of the benchmarks). quant = SNL_Q8_0 or SNL_Q4_0 for the projections
 * that follow the file quantization (embed, lm_head, in_proj and the MTP head stay
 * Q8_0, as convert.rs:232-234, :286-298, :205-226 lay them out). */
int snl_engine_fill_synthetic(snl_engine* e, uint64_t seed, int quant);

int snl_engine_finalize(snl_engine* e);
void snl_engine_destroy(snl_engine* e);

/* Engine::forward_mm (src/engine.rs:801-936). tokens[n]; pos = NULL (rotary position
 * = cache position) or [n][3] u32; embeds = NULL or n_embeds rows of `hidden` floats
 * replacing the embedding of token embed_idx[i]; logit_rows <= 2; ckpt only with n == 2.
 * With logit_rows > 0, logits_out (host) receives logit_rows * vocab floats. */
int snl_engine_forward_mm(snl_engine* e, const uint32_t* tokens, size_t n, const uint32_t* pos,
                          const uint32_t* embed_idx, const float* embeds, size_t n_embeds,
                          size_t logit_rows, int ckpt, float* logits_out);

/* forward_mm followed by the greedy choice on the device: argmax_out (host) receives
 * logit_rows token ids (sampler.rs:169-177), and only those cross to the host. */
int snl_engine_forward_greedy(snl_engine* e, const uint32_t* tokens, size_t n, const uint32_t* pos,
                              size_t logit_rows, int ckpt, uint32_t* argmax_out);

/* Engine::mtp (src/engine.rs:708-774). With draft != 0, *draft_out = argmax of the
 * MTP head's logits. Returns SNL_E_STATE when the engine has no MTP head. */
int snl_engine_mtp(snl_engine* e, size_t r0, const uint32_t* tokens, size_t n, const uint32_t* pos,
                   size_t slot0, int draft, uint32_t* draft_out);

/* Greedy generation of n tokens after `first_token` entirely on the device: each
 * step's argmax is the next step's input without a host round trip (the loop of
 * main.rs:561-565 / worker.rs:207-213 at temperature 0). out_tokens (host) receives the
 * n generated ids; *device_ms (optional) the CUDA-event time of the n steps. */
int snl_engine_generate(snl_engine* e, uint32_t first_token, size_t n, uint32_t* out_tokens,
                        float* device_ms);

/* Per-op timing of one decode step (the SENSENOVA_PROFILE table of engine.rs:859-886,
 * :939-949): runs forward([token], logits) op by op with CUDA events around each and
 * fills up to `cap` records, aggregated by label. bytes = algorithmic bytes moved. */
typedef struct snl_op_stat {
  char label[32];
  uint32_t calls;
  double ms;
  double bytes;
} snl_op_stat;
int snl_engine_profile(snl_engine* e, uint32_t token, snl_op_stat* out, size_t cap, size_t* n_out);

int snl_engine_reset(snl_engine* e);                             /* engine.rs:652-660 */
int snl_engine_snapshot(snl_engine* e, size_t slot);             /* engine.rs:662-670 */
int snl_engine_restore(snl_engine* e, size_t slot, size_t pos);  /* engine.rs:672-683 */
int snl_engine_rollback(snl_engine* e);                          /* engine.rs:685-697 */
size_t snl_engine_hid_rows(const snl_engine* e);                 /* engine.rs:699-702 */
/* Sampler::sample / Sampler::verify (sampler.rs:54-167) on row `row` of the logits of
 * the last snl_engine_forward_mm, on the device (as snl_sample; out3 on the host:
 * token, accepted, draws used). A forward_mm with logits_out == NULL and logit_rows > 0
 * keeps its logits on the device for this, without the copy to the host. hist_tok /
 * hist_cnt: host arrays of the tokens generated so far and their counts. */
int snl_engine_sample(snl_engine* e, size_t row, const snl_sample_p* p, const uint32_t* hist_tok,
                      const uint32_t* hist_cnt, size_t n_hist, const float* u, int64_t draft, uint32_t* out3);
int snl_engine_has_mtp(const snl_engine* e);                     /* engine.rs:704-706 */
/* Matrices whose decode tile layout keeps fp16 block scales (every scale an fp16
 * number) and those that keep f32 scales. */
int snl_engine_tile_scales(const snl_engine* e, uint32_t* fp16_matrices, uint32_t* f32_matrices);
size_t snl_engine_pos(const snl_engine* e);                      /* pub pos, engine.rs:185 */
size_t snl_engine_ctx(const snl_engine* e);                      /* pub ctx, engine.rs:154 */
/* Bytes of device memory the engine holds (Gpu::allocated, gpu.rs:17-18). */
size_t snl_engine_device_bytes(const snl_engine* e);
/* Copy `rows` rows of the last step's normed hidden states (row 0 = the token before
 * the step) to host memory; for tests of the hidden-row bookkeeping. */
int snl_engine_read_hidden(const snl_engine* e, size_t row0, size_t rows, float* out);
/* Engine::prefill_chunk (engine.rs:187, :599): token rows per forward step. */
size_t snl_engine_prefill_chunk(const snl_engine* e);

/* ---- vision tower (src/vision.rs, src/shaders/vision.wgsl) -------------------------- */

/* VisP (vision.rs:39-50). Rows of one frame are in merge order: each run of 4 rows is
 * a 2x2 block of patches, blocks row-major over a (grid_h/2) x (grid_w/2) grid. */
typedef struct snl_vis_p {
  uint32_t rows, cols, mode, act;
  float eps;
  uint32_t grid_w, heads, pad;
} snl_vis_p;
#define SNL_VIS_HEAD_DIM 72 /* vision.wgsl:22 */
#define SNL_VIS_ACT_GELU_TANH 1
#define SNL_VIS_ACT_GELU_ERF 2

/* The four vision.wgsl entry points (device pointers, f32):
 *   layer_norm (vision.wgsl:42-62): b[r] = LayerNorm(a[r]), w = weight[cols] | bias[cols];
 *   epilogue (:82-98): v = act(a + bias); mode 0: a = v; mode 1: b += v; mode 2: b = v + e;
 *   rope (:102-130): 2D rotary on q and k of qkv rows [rows, 3, heads, 72];
 *   attend (:142-206): bidirectional attention over all rows, out [rows, heads * 72]. */
int snl_vis_layer_norm(const snl_vis_p* p, const float* a, float* b, const float* w, void* stream);
int snl_vis_epilogue(const snl_vis_p* p, float* a, float* b, const float* w, const float* e, void* stream);
int snl_vis_rope(const snl_vis_p* p, float* qkv, void* stream);
int snl_vis_attend(const snl_vis_p* p, const float* qkv, float* out, void* stream);

/* VisionConfig (config.rs:40-70). The kernels need head_dim = hidden / n_heads = 72 and
 * merge = 2, as vision.wgsl hard-codes them. */
typedef struct snl_vision_config {
  uint32_t hidden, intermediate, intermediate_padded, depth, n_heads;
  uint32_t patch, temporal_patch, merge, out_hidden, pos_side;
} snl_vision_config;
typedef struct snl_vision snl_vision;
/* Vision::load without the file part: tensors by name (convert.rs:165-199: v.patch,
 * v.patch_b, v.pos, v{i}.n1/.n2/.qkv/.qkv_b/.proj/.proj_b/.fc1/.fc1_b/.fc2/.fc2_b,
 * vm.norm, vm.fc1, vm.fc1_b, vm.fc2, vm.fc2_b) or the seeded synthetic set, then
 * finalize. Matrices are Q8_0 (q int8 + f32 scales), vectors f32. */
int snl_vision_create(const snl_vision_config* cfg, int device, snl_vision** out);
int snl_vision_set_tensor(snl_vision* v, const char* name, int dtype, size_t rows, size_t cols, const void* q,
                          const void* s);
int snl_vision_fill_synthetic(snl_vision* v, uint64_t seed);
int snl_vision_finalize(snl_vision* v);
/* Vision::encode (vision.rs:176-311): patches (host) = frames * h * w patch vectors of
 * patch_dim floats, in merge order, frame-major; out (host) = frames * h * w / 4 rows of
 * out_hidden floats. Frames are encoded one at a time (attention never crosses frames). */
int snl_vision_encode(snl_vision* v, const float* patches, size_t frames, size_t h, size_t w, float* out);
void snl_vision_destroy(snl_vision* v);

/* ---- generation loop (src/worker.rs) ----------------------------------------------
 *
 * snl_worker is the reference's Worker without its tokenizer, text streaming and media
 * encoding: one request at a time over one engine, reusing cached prefixes across
 * requests (the live cache, and SNL_WORKER_SNAPSHOTS snapshot slots evicted least
 * recently used), with MTP draft-1 / verify-2 speculation, rollback of rejected drafts
 * and the self-pause when drafting does not pay off (worker.rs:118-270, :298-338).
 * Sampling runs on the device (snl_engine_sample); the uniform draws come from a
 * seeded ChaCha12 generator on the host, one draw per use as the reference's Sampler
 * takes them. Stop strings, detokenisation and the vision encoder are outside it: the
 * caller passes the prompt as token ids, prefix keys and M-RoPE positions, with any
 * media rows already encoded.
 *
 * snl_worker_ops is the engine as the worker sees it (the methods of engine.rs that
 * worker.rs calls). snl_worker_create fills it from an snl_engine; snl_worker_create_ops
 * accepts any implementation (a host model in tests). */
#define SNL_WORKER_SNAPSHOTS 4 /* engine.rs:20 */
typedef struct snl_worker snl_worker;
typedef struct snl_worker_ops {
  void* self;
  size_t ctx;           /* Engine::ctx */
  size_t prefill_chunk; /* Engine::prefill_chunk */
  size_t hidden;        /* Config::hidden: floats per encoded media row */
  int has_mtp;          /* Engine::has_mtp */
  /* forward_mm with the logits of the last logit_rows rows kept for `sample` */
  int (*forward)(void* self, const uint32_t* tokens, size_t n, const uint32_t* pos, const uint32_t* embed_idx,
                 const float* embeds, size_t n_embeds, size_t logit_rows, int ckpt);
  /* forward_mm plus the device argmax of each logit row; NULL = forward + sample */
  int (*forward_greedy)(void* self, const uint32_t* tokens, size_t n, const uint32_t* pos, size_t logit_rows,
                        int ckpt, uint32_t* argmax_out);
  /* Sampler::sample (draft < 0) or Sampler::verify (draft >= 0) on a kept logit row;
   * out3 = token, accepted, uniform draws used (as snl_engine_sample) */
  int (*sample)(void* self, size_t row, const snl_sample_p* p, const uint32_t* hist_tok, const uint32_t* hist_cnt,
                size_t n_hist, const float* u, int64_t draft, uint32_t* out3);
  int (*mtp)(void* self, size_t r0, const uint32_t* tokens, size_t n, const uint32_t* pos, size_t slot0, int draft,
             uint32_t* draft_out);
  int (*reset)(void* self);
  int (*snapshot)(void* self, size_t slot);
  int (*restore)(void* self, size_t slot, size_t pos);
  int (*rollback)(void* self);
  size_t (*hid_rows)(void* self);
  size_t (*pos)(void* self);
  double (*now)(void* self); /* seconds; NULL = the host's steady clock */
} snl_worker_ops;

/* GenRequest (worker.rs:17-27) with Prompt (mm.rs:383-392) flattened. */
typedef struct snl_gen_request {
  const uint32_t* tokens; /* [n] */
  const uint64_t* keys;   /* [n] prefix-cache keys; NULL = the token ids (Prompt::text) */
  const uint32_t* pos;    /* [n][3] M-RoPE positions; NULL = [i, i, i] */
  size_t n;
  /* encoded media rows: embeds row i (hidden floats) replaces prompt token embed_idx[i] */
  const uint32_t* embed_idx;
  const float* embeds;
  size_t n_embeds;
  int64_t snapshot_at; /* snapshot the state after this many prompt tokens; < 0 = none */
  snl_sample_p params;
  uint64_t seed; /* SamplingParams::seed */
  int has_seed;  /* 0 = seed from the host's entropy */
  size_t max_tokens;
  const uint32_t* eos; /* end-of-sequence ids (cfg.eos) */
  size_t n_eos;
  /* each generated token as it is produced (EOS excluded); return 0 when the client has
   * gone away. NULL = no streaming. */
  int (*on_token)(void* user, uint32_t token);
  void* user;
} snl_gen_request;

#define SNL_FINISH_STOP 0
#define SNL_FINISH_LENGTH 1
/* Finish (worker.rs:41-55). */
typedef struct snl_finish {
  int reason; /* SNL_FINISH_STOP or SNL_FINISH_LENGTH */
  int cancelled;
  size_t prompt_tokens, completion_tokens, cached_tokens;
  size_t drafted, accepted;
  double prefill_secs, decode_secs;
} snl_finish;

int snl_worker_create(snl_engine* e, snl_worker** out);
int snl_worker_create_ops(const snl_worker_ops* ops, snl_worker** out);
void snl_worker_destroy(snl_worker* w);
/* Worker::run (worker.rs:118-270). out_tokens (optional, out_cap entries) receives the
 * generated ids in order, the EOS id last when reason is SNL_FINISH_STOP. On an error
 * the engine is reset and every cached prefix dropped (worker.rs:93-100). */
int snl_worker_run(snl_worker* w, const snl_gen_request* r, uint32_t* out_tokens, size_t out_cap, snl_finish* fin);
/* The prefix keys of the live cache (slot < 0) or of snapshot slot `slot`, and that
 * slot's last-used clock. *n = 0 and *used = 0 for an empty slot. */
int snl_worker_prefix(const snl_worker* w, int slot, uint64_t* keys, size_t cap, size_t* n, uint64_t* used);
/* Whether the current request drafts, and the requests left in a drafting pause. */
int snl_worker_spec(const snl_worker* w, int* spec, size_t* pause);
/* The first n uniform draws [0, 1) of the worker's generator for `seed`. */
int snl_rng_uniforms(uint64_t seed, size_t n, float* out);
/* The ChaCha block function (Bernstein 2008; RFC 8439 section 2.3) with `rounds`
 * rounds (12 in the worker's generator) on the 16-word input state. */
int snl_chacha_block(const uint32_t in[16], int rounds, uint32_t out[16]);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif
#endif /* SNL_B200_H */
