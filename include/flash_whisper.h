/*
 * flash_whisper_b200 — C ABI of the B200 (sm_100a) kernels for batch-1 Whisper-large-v3-turbo.
 *
 * Every entry point takes raw device pointers, sizes and a CUDA stream, launches asynchronously
 * on that stream, allocates nothing, and returns an int status (FW_OK = 0). On a non-zero status
 * fw_last_error_string() holds a one-line message for the calling thread. No entry point
 * synchronises the host, so all of them can be recorded into a CUDA graph.
 *
 * The first four entry points replace the reference's pybind kernels one for one
 * (custom/kernels/whisper_kernels.cu:278-363, bound by custom/ext.py:13-18); the Python wrapper in
 * flash_whisper_b200/ext.py keeps their argument order and error behaviour. The rest are the fused
 * decode path, the GPU log-mel front end and the tcgen05 encoder that replace the torch / cuBLAS /
 * cuFFT / HF-transformers calls made by custom/model.py.
 *
 * fp16 tensors are passed as `void*` (IEEE binary16), row-major, contiguous.
 */
#ifndef FLASH_WHISPER_H_
#define FLASH_WHISPER_H_

#include <stdbool.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* fw_stream_t; /* a cudaStream_t; NULL means the legacy default stream */

enum {
  FW_OK = 0,
  FW_ERR_NULL = 1,        /* a required pointer is NULL */
  FW_ERR_SHAPE = 2,       /* a size argument is out of range or inconsistent */
  FW_ERR_ALIGN = 3,       /* a pointer or stride is not aligned as the kernel requires */
  FW_ERR_ARG = 4,         /* optional arguments given inconsistently */
  FW_ERR_LAUNCH = 5,      /* the CUDA launch failed */
  FW_ERR_UNSUPPORTED = 6  /* the current device is not an sm_100 part */
};

/* Bits of the device-side error word (fw_device_error). */
#define FW_DEVERR_TIMEOUT 1u    /* a bounded wait inside a kernel gave up */
#define FW_DEVERR_BAD_INDEX 2u  /* a token id / position read from device memory was out of range */

/* Message for the last failing call on this thread ("" if none). */
const char* fw_last_error_string(void);
/* ABI version of this library. */
int fw_version(void);
/* Reads (and optionally clears) the OR of every kernel's device error bits. Synchronises. */
int fw_device_error(unsigned int* bits, int clear);

/* ------------------------------------------------------------------------------------------
 * Reference kernel surface
 * ---------------------------------------------------------------------------------------- */

/* h <- fp16(h + x) when x != NULL, then y = LayerNorm(h) * gamma + beta (fp32 math, two-pass
 * variance). hidden must be 1280.
 * Replaces add_layernorm, custom/kernels/whisper_kernels.cu:341-356 (kernel :217-267). */
int fw_add_layernorm(void* h, const void* x, const void* gamma, const void* beta, void* y, int hidden, float eps,
                     fw_stream_t stream);

/* Single-query split-K attention over k/v [heads, max_len, 64]. Self attention: len_state, k_new
 * and v_new are all given; the attended length is len_state[0] + 1 read on the device, and the row
 * at len_state[0] of k/v is overwritten with k_new/v_new [heads, 64]. Cross attention: all three
 * NULL, length = max_len. part_* are fp32 scratch of at least heads*splits (m, l) and
 * heads*splits*64 (acc) elements, splits = ceil(max_len / 64); their sizes are passed so the call
 * can reject a workspace that is too small. out is fp16 [heads*64].
 * Replaces decode_attention, custom/kernels/whisper_kernels.cu:300-339 (kernels :108-213). */
int fw_decode_attention(const void* q, void* k, void* v, void* out, const int64_t* len_state, const void* k_new,
                        const void* v_new, float* part_m, int64_t part_m_numel, float* part_l, int64_t part_l_numel,
                        float* part_acc, int64_t part_acc_numel, int heads, int max_len, float scale,
                        fw_stream_t stream);

/* fw_decode_attention for callers that cannot allocate device memory. No counterpart in the
 * reference. Some callers cannot call cudaMalloc: a host that is recording a CUDA graph (allocation
 * is not allowed while capture is in progress), a plug-in whose device memory belongs to the host
 * application's allocator or a fixed budget, or a real-time audio thread that must not block on
 * the implicit device synchronisation cudaMalloc / cudaFree can cause. This variant takes no
 * workspace: its split partials live in one fixed device array compiled into the library
 * (528 KB on every GPU that loads it, held until the process exits), so it accepts at most
 * heads * ceil(max_len / 64) <= 2048 head-splits and returns FW_ERR_SHAPE beyond that.
 * Semantics, arguments and results are otherwise those of fw_decode_attention. The first call on
 * each device looks up the array's device address (cudaGetSymbolAddress) with that device current;
 * make that first call before any stream capture. The address is cached per device and context: the
 * first call after a cudaDeviceReset (or in any new context of the device) looks it up again, so that
 * call too must come before any stream capture. All calls share the one array and nothing in it
 * needs to start at zero (every split slot is written before the combine reads it), but calls
 * that overlap on the GPU (e.g. on two streams) race on it and must be serialised. */
int fw_decode_attention_noalloc(const void* q, void* k, void* v, void* out, const int64_t* len_state,
                                const void* k_new, const void* v_new, int heads, int max_len, float scale,
                                fw_stream_t stream);

/* best <- max(best, key of argmax_{r, !suppress[r]} fp16(w[r] . h)) with the packed
 * (score, ~index) u64 key, so ties go to the lower index. best must hold 0 on entry.
 * Replaces lm_head_argmax, custom/kernels/whisper_kernels.cu:278-289 (kernel :30-86). */
int fw_lm_head_argmax(const void* h, const void* w, const bool* suppress, int vocab, int hidden, int64_t* best,
                      fw_stream_t stream);

/* Packs an fp16 LM head w [vocab, hidden] for fw_lm_head_argmax_q: wq int8 [vocab, hidden] (row r =
 * round(w[r] / s_r), s_r = max|w[r]| / 127) and rp float4 [vocab] = {s_r, a_r, c2_r, 0} with
 * a_r >= max_i |w[r,i] - s_r wq[r,i]| + 1e-5 max_i |w[r,i]| and c2_r >= 0.51 s_r sum_i |wq[r,i]|
 * (computed in fp64, rounded up). Run once per weight set. No reference counterpart: the
 * reference streams the fp16 matrix every step (whisper_kernels.cu:30-86). */
int fw_lm_quantize(const void* w, int vocab, int hidden, void* wq, void* rp, fw_stream_t stream);

/* Same contract and result as fw_lm_head_argmax (bit-identical best key) with half the bytes read:
 * streams wq/rp from fw_lm_quantize, bounds every row's fp32 logit, and recomputes exactly (the
 * fw_lm_head_argmax arithmetic) only the rows whose upper bound reaches the best lower bound of
 * their block of rows. w is the fp16 matrix wq was made from. */
int fw_lm_head_argmax_q(const void* h, const void* w, const void* wq, const void* rp, const bool* suppress,
                        int vocab, int hidden, int64_t* best, fw_stream_t stream);

/* Decodes best into a token, appends it to tokens[state[1]] (when state[1] < max_pos and
 * < n_tokens), feeds it back into cur, advances state[0] (capped at max_pos-1) and resets best.
 * Replaces argmax_finalize, custom/kernels/whisper_kernels.cu:291-298 (kernel :90-100). */
int fw_argmax_finalize(int64_t* best, int64_t* tokens, int64_t n_tokens, int64_t* state, int64_t* cur, int max_pos,
                       fw_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * Stand-alone decode ops (the torch calls of custom/model.py:110,120 and the argmax microbench)
 * ---------------------------------------------------------------------------------------- */

/* out[i] = fp16(embed[ids[i]] + pos_embed[positions[i]]), i < n; rows of `hidden` fp16.
 * Replaces the index_select + add of custom/model.py:110. */
int fw_embed_pos(const void* embed, const void* pos_embed, const int64_t* ids, const int64_t* positions, void* out,
                 int n, int vocab, int max_pos, int hidden, fw_stream_t stream);

/* y = fp16(gelu_erf(x)), n elements. Replaces F.gelu of custom/model.py:120. */
int fw_gelu(const void* x, void* y, int64_t n, fw_stream_t stream);

/* out_index[0] = argmax over i < n with !suppress[i] (suppress may be NULL) of fp16 logits,
 * first index on ties (torch.argmax). key is an int64 scratch word that must hold 0 on entry and is
 * left at 0. */
int fw_argmax_f16(const void* logits, int64_t n, const bool* suppress, int64_t* key, int64_t* out_index,
                  fw_stream_t stream);

/* out[r] = epilogue(W[r] . LN(h) + b[r]) for r < n_out, LN over hidden=1280 with gamma/beta/eps.
 * act 0: fp16(acc + b); act 1: fp16(gelu(fp16(acc + b))). b may be NULL.
 * Fuses add_layernorm (custom/model.py:113,116,119) with the F.linear that follows it
 * (custom/model.py:114,117,120). */
int fw_ln_gemv(const void* h, const void* gamma, const void* beta, float eps, const void* w, const void* b,
               void* out, int n_out, int hidden, int act, fw_stream_t stream);

/* h[r] = fp16(h[r] + fp16(W[r] . x + b[r])) for r < n_out; x has k elements (k = 1280 or 5120).
 * Fuses F.linear (custom/model.py:116,119,120) with the residual add of the next add_layernorm. */
int fw_gemv_residual(const void* x, int k, const void* w, const void* b, void* h, int n_out, fw_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * Whole decode step (custom/model.py:107-123) as 17 PDL-chained launches: per layer a self-attention
 * block and a cross-attention block (one thread-block cluster per head: LN, projection, split-K
 * attention, output projection and residual in one launch), fc1 and fc2; then the LM head.
 * ---------------------------------------------------------------------------------------- */
#define FW_MAX_LAYERS 8

typedef struct {
  const void *ln1_g, *ln1_b, *ln2_g, *ln2_b, *ln3_g, *ln3_b; /* [1280] */
  const void *qkv_w, *qkv_b;                                 /* [3840,1280], [3840] (K bias zero) */
  const void *out_w, *out_b;   /* out_proj, HEAD-MAJOR [heads, 1280, 64] = W.view(1280, heads, 64)
                                  .permute(1, 0, 2); [1280] */
  const void *cq_w, *cq_b;     /* cross q_proj [1280,1280], [1280] */
  const void *co_w, *co_b;     /* cross out_proj, head-major like out_w */
  const void *fc1_w, *fc1_b;                                 /* [5120,1280], [5120] */
  const void *fc2_w, *fc2_b;                                 /* [1280,5120], [1280] */
  void *self_k, *self_v;                                     /* [heads, max_pos, 64] */
  const void *cross_k, *cross_v;                             /* [heads, enc_len, 64] */
} fw_decoder_layer_t;

typedef struct {
  int n_layers, heads, max_pos, enc_len, vocab, prompt_len;
  float eps, scale;
  const void *embed, *pos_embed, *lm_head; /* [vocab,1280], [max_pos,1280], [vocab,1280] */
  const void *final_g, *final_b;           /* [1280] */
  const bool *base_mask, *first_mask;      /* [vocab]; first_mask applies to the last prompt step */
  const int64_t* prompt;                   /* [prompt_len] forced input ids (may be NULL if 0) */
  fw_decoder_layer_t layers[FW_MAX_LAYERS];
  void *h, *qkv, *attn, *cq, *ffn;          /* fp16 [1280] residual, -, [1280] attention output of the
                                               last self block (may be NULL), [1280] scratch (the
                                               residual after each self block), [5120] fc1 output;
                                               h and cq 16-byte aligned */
  float *part_m, *part_l, *part_acc;        /* part_acc: fp32 [heads * ws_splits * 64] scratch (per-head
                                               output-projection partials of the self and the cross
                                               block); part_m, part_l unused */
  int64_t ws_splits;                        /* >= 40 (part_acc holds 2 * heads * 1280 floats) */
  unsigned int* counters;                   /* [heads + 1], zero before the first step; left zero */
  int64_t *cur, *state, *tokens, *best;     /* [1], [2] = {position, count}, [n_tokens], [1] (0) */
  int64_t n_tokens;
  const void *lm_q, *lm_rp;                 /* optional (both or neither): fw_lm_quantize output for
                                               lm_head; when set, each step's argmax streams these and
                                               rescores the rows that can still win (same token) */
} fw_decoder_t;

/* Launches `steps` decode steps. Step semantics follow custom/model.py:107-123 and :197-207:
 * while state[0] < prompt_len - 1 the input id is prompt[state[0]] and the prediction is
 * discarded; at state[0] == prompt_len - 1 first_mask applies and the prediction becomes tokens[0];
 * afterwards base_mask applies and each prediction is appended and fed back. */
int fw_decoder_step(const fw_decoder_t* d, int steps, fw_stream_t stream);

/* One launch of the decode step in isolation, as fw_decoder_step issues it (programmatic dependent
 * launch included): block 0 = self-attention block of `layer`, 1 = cross-attention block, 2 = LN3 +
 * fc1 + GELU, 3 = fc2 + residual, 4 = LM head (final LN, argmax, token bookkeeping; `layer` ignored).
 * For per-kernel timing and profiling; a full step is blocks 0-3 of every layer, then block 4. Blocks
 * 0 and 1 end with their output-projection partials in part_acc: block 1 adds block 0's to h (into
 * cq) and block 2 adds block 1's (into h), so only the whole sequence updates h as the step does. No
 * reference counterpart (the reference's step is custom/model.py:107-123 as one sequence). */
int fw_decoder_launch(const fw_decoder_t* d, int layer, int block, fw_stream_t stream);

/* Layout of the fw_decoder_step_trace buffer (fp16 element offsets): per layer l, at
 * l * FW_TRACE_LAYER, the self-attention output, the residual stream after the self-attention block,
 * the cross-attention output, the residual stream after the cross-attention block, the fc1 + GELU
 * output and the residual stream after fc2; then, at n_layers * FW_TRACE_LAYER, the final LayerNorm
 * row the LM head dotted. Total n_layers * FW_TRACE_LAYER + 1280 elements. */
#define FW_TRACE_SELF_ATTN 0
#define FW_TRACE_H_SELF 1280
#define FW_TRACE_CROSS_ATTN 2560
#define FW_TRACE_H_CROSS 3840
#define FW_TRACE_FFN 5120
#define FW_TRACE_H_FFN 10240
#define FW_TRACE_LAYER 11520

/* One decode step of fw_decoder_step (the same kernels, launch configurations and arithmetic) that
 * also records every block's output into `trace` (fp16, 16-byte aligned, FW_TRACE_* layout), for
 * activation-level parity checks of the fused step against a restatement of custom/model.py:107-123.
 * The residual-stream snapshots are device-to-device copies enqueued between the launches, so the
 * step is slower than fw_decoder_step; the results (cache writes, token, state) are identical. */
int fw_decoder_step_trace(const fw_decoder_t* d, void* trace, fw_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * On-device decode loop: one CUDA graph whose WHILE node runs decode steps until a clip is done,
 * with the stop condition evaluated on the GPU. Replaces the host loop of custom/model.py:208-215
 * (replay an 8-step graph, copy the tokens back, check for EOS on the host) with one graph launch.
 * ---------------------------------------------------------------------------------------- */
typedef struct fw_decode_loop fw_decode_loop_t;

/* Builds the loop for decoder `d` (pointers are baked into the graph: d's buffers must stay
 * allocated while the loop exists). ctrl is a device int64[5] that the caller fills before each
 * launch: ctrl[0] = token limit (stop once state[1] reaches it), ctrl[1] = EOS id, ctrl[2] = 1 to stop
 * after the first EOS token (0 to ignore EOS), ctrl[4] = cap on body iterations (a guard; the loop
 * always ends); ctrl[3] receives the number of body iterations run minus one. Each iteration runs
 * `steps_per_iter` decode steps, then re-evaluates the condition (EOS is looked for among the
 * tokens of the whole iteration); the condition is also evaluated once before the first iteration.
 * With steps_per_iter > 1 the last iteration may generate up to steps_per_iter - 1 tokens past the
 * limit or the EOS token, as the reference's 8-step chunks do (custom/model.py:208-215): the caller
 * keeps the first min(state[1], limit) tokens up to the first EOS. Host-side set-up only: it
 * creates (and destroys) a private stream and the graph, and launches nothing. */
int fw_decode_loop_create(const fw_decoder_t* d, int64_t* ctrl, int steps_per_iter, fw_decode_loop_t** out);
/* Launches the loop on `stream` (asynchronous; one graph launch). */
int fw_decode_loop_launch(fw_decode_loop_t* loop, fw_stream_t stream);
/* Frees the graph (NULL is accepted). */
int fw_decode_loop_destroy(fw_decode_loop_t* loop);

/* ------------------------------------------------------------------------------------------
 * Batched decode step: up to FW_MAX_CLIPS independent clips per weight read (no reference
 * counterpart: the reference decodes one clip per step, custom/model.py:107-123). Each clip's
 * arithmetic is exactly the batch-1 step's, so its tokens equal decoding it alone with
 * fw_decoder_step; the weights (216 MB per step without the LM head) are read once for all clips.
 * ---------------------------------------------------------------------------------------- */
#define FW_MAX_CLIPS 8

typedef struct {
  int n_layers, heads, max_pos, enc_len, vocab, prompt_len, clips;
  float eps, scale;
  const void *embed, *pos_embed, *lm_head; /* as fw_decoder_t */
  const void *final_g, *final_b;
  const bool *base_mask, *first_mask;
  const int64_t* prompt;
  fw_decoder_layer_t layers[FW_MAX_LAYERS]; /* weights as fw_decoder_t; self_k/self_v/cross_k/cross_v
                                               point at clip 0's caches of the layer */
  int64_t self_clip_stride;                 /* elements from clip c's self_k/self_v to clip c+1's */
  int64_t cross_clip_stride;                /* elements from clip c's cross_k/cross_v to clip c+1's */
  void *h, *qkv, *attn, *ffn;               /* fp16 [clips,1280], [clips,3840], [clips,1280], [clips,5120] */
  float *part_m, *part_l, *part_acc;        /* fp32 [clips*heads*ws_splits] (m, l), [... * 64] (acc) */
  int64_t ws_splits;                        /* >= ceil(max(max_pos, enc_len) / 64) */
  unsigned int* counters;                   /* [clips*heads + 1], zero before the first step; left zero */
  int64_t *cur, *state, *tokens, *best;     /* [clips], [clips,2], [clips,n_tokens], [clips] (zero) */
  int64_t n_tokens;
  const void *lm_q, *lm_rp;                 /* required: fw_lm_quantize output of lm_head */
} fw_batch_decoder_t;

/* Launches `steps` decode steps of every clip (fw_decoder_step semantics per clip: prompt handling,
 * first_mask on the last prompt step, tokens appended at tokens[c * n_tokens + state[c][1]]). Per step
 * and layer: LN1 + q/k/v, self attention with the cache write, out_proj + residual, LN2 + cross q,
 * cross attention, cross out_proj + residual, LN3 + fc1 + GELU, fc2 + residual; then the pruned LM
 * head of all clips with the final LN, argmax and bookkeeping (33 launches per step). */
int fw_batch_decoder_step(const fw_batch_decoder_t* d, int steps, fw_stream_t stream);

/* One launch of the batched step in isolation, as fw_batch_decoder_step issues it (for per-kernel
 * timing and profiling): block 0 = LN1 + q/k/v of `layer`, 1 = self attention, 2 = out_proj +
 * residual, 3 = LN2 + cross q, 4 = cross attention, 5 = cross out_proj + residual, 6 = LN3 + fc1 +
 * GELU, 7 = fc2 + residual, 8 = LM head of all clips (`layer` ignored). */
int fw_batch_decoder_launch(const fw_batch_decoder_t* d, int layer, int block, fw_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * GPU log-mel front end (custom/model.py:93-98; WhisperFeatureExtractor semantics)
 * ---------------------------------------------------------------------------------------- */

/* wave fp32 [batch, n_samples]; filters fp32 [201, 128] (Slaney mel filterbank, n_fft 400);
 * scratch fp32 [batch, 128, n_frames] and clip_max u32 [batch] are caller-owned scratch;
 * n_frames = n_samples / 160. Output fp16: layout 0 = [batch, 128, n_frames] (as the reference's
 * mel buffer), layout 1 = [batch, n_frames + 2, 128] time-major with one zero row on each side
 * (the encoder's conv1 operand). */
int fw_log_mel(const float* wave, int batch, int n_samples, const float* filters, float* scratch,
               unsigned int* clip_max, void* mel_out, int layout, fw_stream_t stream);

/* ------------------------------------------------------------------------------------------
 * Encoder (HF WhisperEncoder as called by custom/model.py:143-147)
 * ---------------------------------------------------------------------------------------- */

/* Epilogues of fw_gemm_f16 (acc is the fp32 tensor-core accumulator). */
#define FW_EPI_BIAS 0         /* C = fp16(acc + bias) */
#define FW_EPI_BIAS_GELU 1    /* C = fp16(gelu(fp16(acc + bias))) */
#define FW_EPI_BIAS_RESID 2   /* C = fp16(R + fp16(acc + bias)); R may alias C */
#define FW_EPI_GELU_POS 3     /* C = fp16(fp16(gelu(fp16(acc + bias))) + R[row]) (conv2 + positions) */
#define FW_EPI_CROSS_KV 4     /* cross K/V scatter into [layers, 2, heads, M, 64] */
#define FW_EPI_BIAS_SCALE 5   /* C = fp16(fp16(acc + bias) * scale) for columns < scale_cols */
#define FW_EPI_QKV_VT 6       /* as FW_EPI_BIAS_SCALE for columns n < 2N/3 (q | k); the last third (v)
                                 is written transposed instead: R[(n - 2N/3) * ldr + m] */

/* C[M, N] = epilogue(A[M, K] . B[N, K]^T + bias[N]) on tcgen05 tensor cores, fp16 in, fp32
 * accumulate in TMEM. lda/ldb/ldc/ldr are row strides in elements. K % 64 == 0, N % 64 == 0;
 * lda, ldb >= K and multiples of 8; A, B, C, bias, R 16-byte aligned. bias may be NULL.
 * FW_EPI_CROSS_KV writes column n of row m to C[((n / 64) * M + m) * 64 + n % 64], i.e. the
 * [layers, 2, heads, M, 64] cross-attention cache of custom/model.py:146 (ldc ignored).
 * Replaces the torch/cuBLAS GEMMs of the HF encoder and custom/model.py:145. */
int fw_gemm_f16(const void* A, int64_t lda, const void* B, int64_t ldb, const void* bias, void* C, int64_t ldc,
                const void* R, int64_t ldr, int M, int N, int K, int epilogue, float scale, int scale_cols,
                fw_stream_t stream);

/* Conv1d(kernel 3, padding 1, stride 1 or 2) as an implicit GEMM on the same tensor cores.
 * X is the time-major input [rows_padded, C] whose first and last rows are zero padding;
 * W is [N, 3*C] ordered (tap, channel), i.e. torch's [N, C, 3] weight permuted to [N, 3, C].
 * Output row t (t < M) = epilogue(sum_j X[stride*t + j] . W[:, j*C:(j+1)*C]^T + bias).
 * Replaces conv1/conv2 of the HF WhisperEncoder. */
int fw_conv1d_k3_f16(const void* X, int C, int rows_padded, int stride, const void* W, const void* bias, void* Out,
                     int64_t ldc, const void* R, int64_t ldr, int M, int N, int epilogue, fw_stream_t stream);

/* Row-wise LayerNorm: y[r] = LN(x[r]) * g + b, rows x cols fp16 (cols % 256 == 0). */
int fw_layernorm_rows(const void* x, const void* g, const void* b, void* y, int rows, int cols, float eps,
                      fw_stream_t stream);

/* Bidirectional multi-head attention for the encoder (tcgen05, TMEM accumulators). qkv fp16
 * [seq, ld] holding pre-scaled q at column h*64, k at kcol + h*64 and v at vcol + h*64; out fp16
 * [seq, heads*64]. vt_scratch: fp16 [heads*64, round_up(seq, 8)] caller-owned scratch that receives
 * V transposed. Replaces the SDPA attention of the HF WhisperEncoderLayer. */
int fw_encoder_attention(const void* qkv, int64_t ld, int kcol, int vcol, void* out, int seq, int heads,
                         void* vt_scratch, fw_stream_t stream);

#define FW_MAX_ENC_LAYERS 32
typedef struct {
  const void *ln1_g, *ln1_b, *ln2_g, *ln2_b;
  const void *qkv_w, *qkv_b; /* [3840,1280] = q_proj, k_proj, v_proj; bias (k part zero) */
  const void *out_w, *out_b;
  const void *fc1_w, *fc1_b, *fc2_w, *fc2_b;
} fw_encoder_layer_t;

typedef struct {
  int n_layers, n_frames, n_pos, n_dec_layers, heads;
  float eps;
  const void* mel;                 /* fp16 [n_frames + 2, 128] time-major, zero rows at both ends */
  const void *conv1_w, *conv1_b;   /* [1280, 3*128] ordered (tap, channel); [1280] */
  const void *conv2_w, *conv2_b;   /* [1280, 3*1280] ordered (tap, channel); [1280] */
  const void* pos;                 /* [n_pos, 1280] sinusoid table */
  fw_encoder_layer_t layers[FW_MAX_ENC_LAYERS];
  const void *final_g, *final_b;
  const void *cross_w, *cross_b;   /* [n_dec_layers*2*1280, 1280], bias (K parts zero) */
  void* conv1_out;                 /* fp16 [n_frames + 2, 1280], rows 0 and n_frames+1 zero */
  void *x, *y, *qkv, *attn, *ffn;  /* fp16 [n_pos,1280], [n_pos,1280], [n_pos,3840], [n_pos,1280],
                                      [n_pos,5120] */
  void* enc_out;                   /* fp16 [n_pos, 1280] final-LN output */
  void* cross_kv;                  /* fp16 [n_dec_layers, 2, heads, n_pos, 64] */
  void* vt;                        /* fp16 [heads*64, round_up(n_pos, 8)] V^T scratch */
} fw_encoder_t;

/* mel -> encoder states -> cross K/V for every decoder layer (custom/model.py:143-147). */
int fw_encoder_forward(const fw_encoder_t* e, fw_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FLASH_WHISPER_H_ */
