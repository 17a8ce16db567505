/*
 * fw_model.h -- the model and run-state views that oracle/forward_oracle.c
 * (the C restatement) and oracle/ref_harness.cpp (the reference's own ops)
 * share, so one Python description drives both.  TEST INFRASTRUCTURE ONLY.
 * Fields follow reference src/gguf.h:139-168 (llama_config_t), the tensor
 * names of src/forward.cpp:178-265 and src/run_state.h:27-182 (RunState).
 */
#ifndef TLE_ORACLE_FW_MODEL_H
#define TLE_ORACLE_FW_MODEL_H
#include <stdint.h>

typedef struct {
    int32_t type; /* FW_* */
    int32_t pad;
    const void *data;
} fw_weight_t;

typedef struct {
    fw_weight_t wq, wk, wv, wo, w_gate, w_up, w_down;
    const float *attn_norm; /* [n_embd] */
    const float *ffn_norm;  /* [n_embd] */
} fw_layer_t;

typedef struct {
    int32_t n_layers, n_embd, n_head, n_head_kv, n_ff, n_vocab, n_ctx;
    float rope_freq_base, rms_norm_eps;
    int32_t pad;
    fw_weight_t token_embd; /* F16 or F32 [n_vocab][n_embd] */
    fw_weight_t output;     /* [n_vocab][n_embd]; data NULL = tied to token_embd */
    const float *output_norm;
    const fw_layer_t *layers;
} fw_model_t;

/* RunState (reference src/run_state.h:27-182): the buffers forward() uses. */
typedef struct {
    float *x, *xb, *xb2, *q, *k, *v, *hb, *hb2, *logits;
    float *key_cache, *value_cache; /* [n_layers][n_ctx][n_head_kv*head_dim] */
    float *att;                     /* [n_ctx] */
} fw_state_t;

#endif
