/*
 * tle_forward.h -- C ABI of the device forward pass around attention.
 *
 * Replaces the rest of the reference's per-token forward() (src/forward.h:16,
 * src/forward.cpp:178-265) and the ops it calls (src/ops.h:64-249) with
 * sm_100a kernels, so that a token runs on the GPU end to end: embedding,
 * per layer RMSNorm + q/k/v projections, rope + attention (tle_attn.h),
 * output projection + residual, RMSNorm + SwiGLU feed-forward + residual,
 * final RMSNorm + LM head, greedy sampling.
 *
 * Weights stay in the reference's GGUF block layouts (src/gguf.h:54-135),
 * read in place from device memory: pass the device copy of each tensor's
 * bytes.  Formats: the ggml type numbers TLE_W_*.  All pointers are device
 * pointers unless marked HOST; weight pointers must be 16-byte aligned.
 * Every call is asynchronous on `stream` (a cudaStream_t, NULL = default)
 * and returns TLE_OK or an error code (tle_last_error() has the message).
 * Results match the reference up to fp32 summation order (tolerances in
 * tests/test_forward_gpu.py); there is no CPU fallback.
 */
#ifndef TLE_FORWARD_H
#define TLE_FORWARD_H

#include <stddef.h>
#include <stdint.h>

#include "tle_attn.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ggml_type numbers (reference src/gguf.h:23-33) */
#define TLE_W_F32 0
#define TLE_W_F16 1
#define TLE_W_Q4_0 2
#define TLE_W_Q8_0 8
#define TLE_W_Q6_K 14

/* matmul(out, W, x, rows, cols, type) ops.h:64-66: out[r] = W[r,:] . x.
 * cols at most 16384 and, for the block formats, a multiple of the block
 * (32; 256 for Q6_K). */
int tle_matmul(float* out, const void* W, const float* x, int rows, int cols, int type,
               void* stream);

/* rmsnorm(out, x, weight, size, eps) ops.h:95-96 (out may alias x). */
int tle_rmsnorm(float* out, const float* x, const float* weight, int size, float eps, void* stream);

/* vec_add(out, x, size) ops.h:143: out += x. */
int tle_vec_add(float* out, const float* x, int size, void* stream);

/* ffn_swiglu ops.h:232-235 with the reference's argument list.  The gate
 * and up products and silu(gate) * up are one fused launch writing hb
 * (hb2 is not used: the up rows never leave registers); then the down
 * product writes out.  As in the reference, all three weights are read as
 * `type`. */
int tle_ffn_swiglu(float* out, const float* input, float* hb, float* hb2, const void* W_gate,
                   const void* W_up, const void* W_down, int n_ff, int n_embd, int type,
                   void* stream);

/* sample_argmax ops.h:249: the first index of the largest logit, written to
 * *token (device int32).  NaN logits never win, as with the reference's
 * '>' scan; a NaN at index 0 gives 0. */
int tle_sample_argmax(const float* logits, int n_vocab, int32_t* token, void* stream);

/* sample_temperature ops.h:262 and sample_top_p ops.h:278 with the uniform
 * draw r in [0, 1) passed in (the reference draws it from its own unseeded
 * std::mt19937, ops.cpp:1571; pass dist(rng) from any generator).  As in the
 * reference the logits are scaled by 1/temperature when temperature != 1
 * and > 0 and overwritten with their softmax; the token is written to
 * *token (device int32).  Temperature: the first index whose running
 * probability sum exceeds r (n_vocab - 1 if none).  Top-p: the most probable
 * tokens, sorted by probability (ties by index), up to a cumulative sum
 * >= top_p; r scaled by that sum picks among them in that order.  The
 * reference sorts only its 100 most probable tokens (std::partial_sort)
 * and walks any longer nucleus in an unspecified order; here up to 2048
 * tokens are sorted and a nucleus is cut at 2048.  n_vocab <= 40960. */
int tle_sample_temperature(float* logits, int n_vocab, float temperature, float r, int32_t* token,
                           void* stream);
int tle_sample_top_p(float* logits, int n_vocab, float temperature, float top_p, float r,
                     int32_t* token, void* stream);

/* ---- forward() ---- */

typedef struct {
    int32_t type;     /* TLE_W_* */
    int32_t reserved;
    const void* data; /* device, GGUF layout, [rows][cols] */
} tle_weight_t;

/* The tensors of block l (forward.cpp:184-229 names blk.l.*). */
typedef struct {
    tle_weight_t attn_q, attn_k, attn_v, attn_output, ffn_gate, ffn_up, ffn_down;
    const float* attn_norm; /* [n_embd] fp32 */
    const float* ffn_norm;  /* [n_embd] fp32 */
} tle_layer_t;

/* llama_config_t fields (gguf.h:139-168) plus the global tensors.  The
 * attention kernels need n_head 32, n_head_kv 4, head_dim 64. */
typedef struct {
    int32_t n_layers, n_embd, n_head, n_head_kv, n_ff, n_vocab, n_ctx;
    float rope_freq_base, rms_norm_eps;
    int32_t reserved;
    tle_weight_t token_embd;  /* F16 or F32 [n_vocab][n_embd] */
    tle_weight_t output;      /* LM head; data NULL: token_embd (forward.cpp:253-260) */
    const float* output_norm; /* [n_embd] */
    const tle_layer_t* layers; /* HOST array [n_layers] */
} tle_model_t;

/* RunState (run_state.h:27-182) in device memory.  xb is not needed on the
 * device (the RMSNorms are fused into the products that read them) but is
 * kept so a RunState maps field for field. */
typedef struct {
    float *x, *xb, *xb2, *q, *k, *v, *hb, *hb2, *logits;
    float *key_cache, *value_cache; /* [n_layers][n_ctx][n_head_kv*head_dim] */
    void* workspace;                /* attention scratch, tle_forward_workspace_bytes */
    size_t workspace_bytes;
} tle_state_t;

/* Scratch tle_forward needs (the attention split-K partials). */
size_t tle_forward_workspace_bytes(const tle_model_t* model);

/* 1 when tle_forward(model, state, token, pos) on the current device runs
 * all layers in one persistent launch (every linear weight Q4_0, widths
 * multiples of 256, the pos + 1 cached rows within the launch's attention
 * split, cooperative launch supported), 0 when it launches product by
 * product.  Either way the results agree with forward() (forward.cpp:172). */
int tle_forward_layers_one_launch(const tle_model_t* model, const tle_state_t* state, int pos);

/* forward(model, state, token, pos) forward.h:16 for the token *token
 * (device int32, so a device-side sampler can feed the next step) at
 * position pos: appends row pos of every layer's cache and leaves the
 * logits in state->logits.  Per layer: RMSNorm + q/k/v in one launch,
 * rope + attention (the tle_rope_attention kernels), output projection +
 * residual, RMSNorm + gate/up + SwiGLU, down projection + residual; then
 * RMSNorm + LM head.  A token outside [0, n_vocab) is reported through
 * tle_device_error (0x106) and embeds as zeros. */
int tle_forward(const tle_model_t* model, const tle_state_t* state, const int32_t* token, int pos,
                void* stream);

/* ---- batched prompt ----
 * The reference feeds a prompt one token at a time (generate.cpp:52-59: one
 * forward() per prompt token).  tle_prompt_forward runs those forward()
 * calls for n_tokens tokens at once, layer by layer: every product is one
 * matrix product over all the tokens on the tcgen05 tensor cores (fp16
 * operands, fp32 accumulation), the attention is tle_prefill's.  The
 * products read an fp16 copy of the linear weights made once by
 * tle_prompt_pack_weights. */

/* Bytes of the fp16 weight copy: per layer, in order, q/k/v rows
 * [n_embd + 2*kv_dim][n_embd], output [n_embd][n_embd], gate then up rows
 * [2*n_ff][n_embd], down [n_embd][n_ff].  0 if the model is unsupported
 * (tle_last_error says why): n_head 32, n_head_kv 4, head_dim 64, n_ff a
 * multiple of 128. */
size_t tle_prompt_weights_bytes(const tle_model_t* model);
/* Writes the fp16 copy into dst (device, 16-byte aligned, at least
 * tle_prompt_weights_bytes): each weight dequantised as the reference does
 * (every TLE_W_* format; the feed-forward weights read as ffn_gate's type,
 * forward.cpp:224-227) and rounded to nearest fp16. */
int tle_prompt_pack_weights(const tle_model_t* model, void* dst, size_t dst_bytes, void* stream);
/* Scratch of tle_prompt_forward for n_tokens prompt tokens at pos0. */
size_t tle_prompt_scratch_bytes(const tle_model_t* model, int n_tokens, int pos0);
/* forward() for tokens[0..n_tokens) (device int32) at positions pos0.. in
 * one pass: appends rows pos0 .. pos0+n_tokens-1 of every layer's cache and
 * leaves the last token's logits in state->logits and its final residual
 * in state->x, as the reference's prompt loop does.  scratch: device,
 * 1024-byte aligned, tle_prompt_scratch_bytes.  Tokens outside [0, n_vocab)
 * are reported through tle_device_error (0x106) and embed as zeros.  The
 * products take fp16 operands: an activation whose fp16 rounding overflows
 * (|x| >= 65520) is reported (0x109) rather than passed on silently. */
int tle_prompt_forward(const tle_model_t* model, const void* packed, const tle_state_t* state,
                       const int32_t* tokens, int n_tokens, int pos0, void* scratch,
                       size_t scratch_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TLE_FORWARD_H */
