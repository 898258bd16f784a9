/*
 * sf_oracle.h -- CPU restatement of StrataFlow's per-token MoE decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA path in
 * strataflow_b200/: only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference leg may load it.  The product never links it
 * and never falls back to it.
 *
 * What it restates (reference = Coaade-Inc/strataflow, paths relative to the
 * reference project root):
 *   - the op order of engine::Engine::forward, src/model/engine/engine.cpp:2498-3025
 *     (embedding :2708-2723, router segment :1854-1947, KV attention
 *     :1633-1762, expert segment :1956-1989, final norm + lm_head :2958-3006)
 *   - greedy argmax, strict '>' first-max-wins, engine.cpp:3111-3121
 *   - the ggml b11379 CPU arithmetic those call sites reach (ggml is an
 *     un-vendored submodule, .gitmodules:1-3; it is restated here from ggml's
 *     published reference kernels, see sf_oracle.c for each function):
 *       quantized mul_mat / mul_mat_id quantize the activation row to the
 *       weight type's dot type (Q8_K for Q4_K/Q6_K, Q8_0 for Q8_0) and take
 *       integer sub-block dot products scaled in fp32; rms_norm sums squares in
 *       double; soft_max subtracts the max and sums in double; silu = x/(1+e^-x).
 *
 * Block formats (ggml; sizes pinned by gguf-py 0.19.0 constants.py:4239-4246):
 *   Q8_0 : 32 weights, 34 B  = f16 d, int8 qs[32]
 *   Q4_K : 256 weights, 144 B = f16 d, f16 dmin, u8 scales[12], u8 qs[128]
 *   Q6_K : 256 weights, 210 B = u8 ql[128], u8 qh[64], i8 scales[16], f16 d
 *   Q8_K : 256 values, 292 B  = f32 d, i8 qs[256], i16 bsums[16]  (activations)
 *
 * Parity pin: the dequantizers and the Q8_0 quantizer are checked against
 * gguf-py 0.19.0 (a numpy restatement of ggml's reference kernels) through the
 * committed fixtures in tests/golden/.  The engine-level numerics (activation
 * quantization, dot order) have no reference output in this container
 * (ggml is absent), so those are "parity unpinned" beyond the block level.
 */
#ifndef SF_ORACLE_H
#define SF_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml_type ids (ggml.h enum values; also gguf-py GGMLQuantizationType). */
enum { SFO_F32 = 0, SFO_F16 = 1, SFO_Q8_0 = 8, SFO_Q4_K = 12, SFO_Q6_K = 14, SFO_Q8_K = 15 };

/* ---- scalar helpers ---------------------------------------------------- */
uint16_t sfo_fp32_to_fp16(float f);
float    sfo_fp16_to_fp32(uint16_t h);

/* bytes of one row of `n` elements of ggml type `type` (GGUF layout). */
size_t sfo_row_bytes(int type, int64_t n);

/* ---- block-level quant / dequant ---------------------------------------- */
int  sfo_dequantize(int type, const void *src, float *dst, int64_t n);
int  sfo_quantize_q8_0(const float *x, void *dst, int64_t n);   /* ggml ref */
int  sfo_quantize_q8_K(const float *x, void *dst, int64_t n);   /* ggml ref */
/* the build's own weight quantizers (structure of ggml's ref, simplified scale
 * search; used only to make fixtures) */
int  sfo_quantize_weights(int type, const float *x, void *dst, int64_t nrows, int64_t ncols);

/* ---- deterministic synthetic weights ------------------------------------ */
/* Irwin-Hall(12) approximation of N(0,1) built from splitmix64 counters, so the
 * CUDA generator reproduces it bit for bit.  value = std * z. */
void sfo_synth_f32(uint64_t seed, int64_t offset, int64_t n, float std_, float *dst);

/* ---- ops ---------------------------------------------------------------- */
/* exp(x) shared bit-for-bit with the CUDA kernels (Cody-Waite + Taylor) */
float sfo_expf(float x);
/* y[r] = dot(W[r,:], x) for a quantized or F32 weight matrix [nrows x ncols],
 * activation quantized to the weight's dot type first (ggml-exact mode, the
 * kernels' fp32 accumulation order), weights dequantized and dotted in
 * f32/double (fp32_mode 1, diagnostic) or ggml's generic per-block fp32
 * order (fp32_mode 2, for comparison). */
int  sfo_mul_mat(int type, const void *w, int64_t nrows, int64_t ncols,
                 const float *x, float *y, int fp32_mode);
/* Token sampling of the generate loop (greedy when temperature <= 0; see
 * sf_oracle.c for the definition shared with the device sampler). */
int32_t sfo_sample(const float *logits, int64_t V, float temperature, int32_t top_k, float top_p, uint64_t seed,
                   int32_t step);
void sfo_rms_norm(const float *x, const float *w, int64_t n, float eps, float *y);
void sfo_rope_normal(float *x, int n_head, int head_dim, int pos, float freq_base);
void sfo_soft_max(const float *x, float *y, int64_t n, float scale);
void sfo_top_k_desc(const float *x, int64_t n, int k, int32_t *ids);

/* Fused routed-expert FFN for b tokens (mul_mat_id gate/up, swiglu, down,
 * routing-weight multiply, sum over k, residual): engine.cpp:1956-1989.
 *   x    [b, d]     ffn-normed expert input
 *   res  [b, d]     residual branch (ffn_inp); may be NULL for no residual
 *   ids  [b, k]     routed expert ids
 *   wts  [b, k]     routing weights
 *   gate/up         [E, F, d] stacked, type `type`;  down [E, d, F]
 *   out  [b, d]
 * gu_out (optional) receives the swiglu activation [b, k, F]. */
int  sfo_moe_ffn(int type_gu, int type_down, const void *gate, const void *up, const void *down,
                 int n_expert, int d, int F, int b, int k,
                 const float *x, const float *res, const int32_t *ids, const float *wts,
                 float *out, float *gu_out, int fp32_mode);

/* Router: probs = soft_max(W_r x); ids = top-k; weights = probs[ids] /
 * max(sum, 6.103515625e-5): engine.cpp:1913-1924. W_r is F32 [E, d]. */
void sfo_router(const float *w_r, int n_expert, int d, const float *x, int k,
                int32_t *ids, float *weights, float *probs_out);

/* GQA decode attention of one query token over n_kv cached positions, ggml
 * op order of engine.cpp:1751-1761.  q [Hq*hd]; k,v [n_kv][Hkv][hd] (f32);
 * out [Hq*hd]. */
void sfo_attn_decode(const float *q, const float *k, const float *v, int n_kv,
                     int n_head, int n_head_kv, int head_dim, float *out);

/* ---- whole model -------------------------------------------------------- */
typedef struct sfo_hparams {
    int32_t n_embd, n_head, n_head_kv, n_layer, n_ff, n_expert, n_expert_used, n_vocab, n_ctx;
    float   rms_eps, freq_base;
    int32_t type_embd, type_attn, type_ffn_gu, type_ffn_down, type_output;
    int32_t kv_f16;       /* round stored K/V through f16 (the paged-f16 KV mode) */
    int32_t fp32_mode;    /* diagnostic: dequantize weights, f32 activations */
    int32_t head_dim;     /* 0: n_embd / n_head (engine.cpp:1161); else the stated head width */
    /* Expert parallelism's fp32 order (the B200 engine over ep_size GPUs; the
     * reference has no such mode): each rank's expert outputs are summed
     * over its own experts [r E/N, (r+1) E/N) in slot order, rank 0 adds the
     * residual, and the ranks' partials are added in rank order; with
     * ep_head_par the output projection is the same: each rank's dot over its
     * heads' column slice, residual on rank 0, partials in rank order.
     * 0 or 1: one GPU. */
    int32_t ep_size;
    int32_t ep_head_par;
} sfo_hparams;

/* tensor ids shared with the CUDA engine's C ABI (include/sfk.h) */
enum {
    SFO_T_TOK_EMBD = 0, SFO_T_OUTPUT_NORM = 1, SFO_T_OUTPUT = 2,
    SFO_T_ATTN_NORM = 3, SFO_T_ATTN_Q = 4, SFO_T_ATTN_K = 5, SFO_T_ATTN_V = 6, SFO_T_ATTN_OUT = 7,
    SFO_T_FFN_NORM = 8, SFO_T_FFN_GATE_INP = 9, SFO_T_FFN_GATE_EXPS = 10, SFO_T_FFN_UP_EXPS = 11,
    SFO_T_FFN_DOWN_EXPS = 12, SFO_T_COUNT = 13
};

typedef struct sfo_model sfo_model;
typedef struct sfo_seq   sfo_seq;

sfo_model *sfo_model_create(const sfo_hparams *hp);
void       sfo_model_free(sfo_model *m);
/* fp32 accumulation order of the quantized mul_mats of later forwards: 0 the
 * decode kernels' unit order, 2 ggml's generic per-block order (the order of
 * the tensor-core prefill GEMMs), 1 the dequantize-and-dot diagnostic. */
void       sfo_set_fp32_mode(sfo_model *m, int mode);
/* shape/type/size of tensor (tid, layer) in GGUF bytes; returns bytes or 0 */
size_t     sfo_tensor_bytes(const sfo_model *m, int tid, int layer, int *type, int64_t ne[3]);
void      *sfo_tensor_data(sfo_model *m, int tid, int layer);
/* fill every tensor from the seeded synthetic generator (norms = 1) */
int        sfo_model_synth(sfo_model *m, uint64_t seed);
sfo_seq   *sfo_seq_create(const sfo_model *m);
void       sfo_seq_free(sfo_seq *s);
void       sfo_seq_reset(sfo_seq *s);
/* one token at `pos` (causal over 0..pos); logits [n_vocab]; returns argmax or <0 */
int32_t    sfo_forward(const sfo_model *m, sfo_seq *s, int32_t token, int32_t pos, float *logits);
/* timing support: positions 0..n_pos-1 of the KV cache filled with seeded
 * values in [-1, 1) (a stand-in for a fed prompt); returns 0 or -1 */
int        sfo_seq_fill_kv(sfo_seq *s, int n_pos, uint64_t seed);
/* per-layer hooks for tests: hidden state after layer `il` of the last forward */
const float *sfo_seq_hidden(const sfo_seq *s, int il);
const int32_t *sfo_seq_ids(const sfo_seq *s, int il);
/* intermediates of layer `il` in the last forward: which = 0 attention output
 * [Hq*hd], 1 ffn_inp [d], 2 ffn-normed expert input [d], 3 routing weights [k],
 * 4 q after RoPE [Hq*hd]; returns NULL for an unknown buffer */
const float *sfo_seq_debug(const sfo_seq *s, int il, int which);
int32_t    sfo_argmax(const float *v, int n);
/* wall seconds spent in the layer loop and in embedding + head, summed over
 * every sfo_forward of this sequence (for the timed CPU baseline) */
void       sfo_seq_timing(const sfo_seq *s, double *layers_s, double *head_s);

/* seed of tensor (tid, layer) under model seed (shared with the CUDA synth) */
uint64_t   sfo_tensor_seed(uint64_t seed, int tid, int layer);
void       sfo_set_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
