/*
 * sfk.h -- C ABI of the B200 (sm_100a) decode path for StrataFlow.
 *
 * This is the drop-in boundary for the per-token MoE decode hot path of
 * Coaade-Inc/strataflow (reference paths below are relative to that project).
 * The reference runs the path as ggml graphs built by engine::Engine
 * (src/model/engine/engine.h:102-308, engine.cpp:2498-3025).  A StrataFlow
 * build links libsfk.so and calls these entry points from its own C++ host
 * code: Engine::load -> sfk_engine_create + sfk_weights_put (the HBM tier),
 * Engine::forward -> sfk_forward, Engine::reset_kv -> sfk_kv_reset.  The
 * .strata format, the public include/strataflow API and the planner /
 * predictor contracts are unchanged.
 *
 * Conventions
 *   - Plain C types only; no exceptions cross this boundary.
 *   - Status codes are the reference's sf_status values
 *     (include/strataflow/strataflow.h:46-55).
 *   - Tensor ids and ggml type ids follow GGUF naming (token_embd.weight, ...)
 *     and ggml.h's ggml_type enum.
 *   - An engine is used by one host thread at a time (engine.h:101: forward()
 *     is not thread-safe).  All device work is ordered on the engine's stream.
 *   - Pointers documented as "device" are CUDA device pointers; "host"
 *     pointers are ordinary (pageable or pinned) host memory.
 */
#ifndef SFK_H
#define SFK_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SFK_API __attribute__((visibility("default")))
#else
#define SFK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status (== sf_status, strataflow.h:46-55) ------------------------- */
typedef int32_t sfk_status;
#define SFK_OK 0
#define SFK_ERR_INVALID_ARGUMENT 1
#define SFK_ERR_UNSUPPORTED 3
#define SFK_ERR_OUT_OF_MEMORY 4
#define SFK_ERR_RUNTIME 7

/* ggml_type ids (ggml.h) accepted by this library */
#define SFK_TYPE_F32 0
#define SFK_TYPE_F16 1
#define SFK_TYPE_Q8_0 8
#define SFK_TYPE_Q4_K 12
#define SFK_TYPE_Q6_K 14
#define SFK_TYPE_Q8_K 15

/* tensor ids (GGUF names used by engine.cpp:1854-1989,2712,2994) */
#define SFK_T_TOK_EMBD 0       /* token_embd.weight          [d, V]        */
#define SFK_T_OUTPUT_NORM 1    /* output_norm.weight         [d]   F32     */
#define SFK_T_OUTPUT 2         /* output.weight              [d, V]        */
#define SFK_T_ATTN_NORM 3      /* blk.L.attn_norm.weight     [d]   F32     */
#define SFK_T_ATTN_Q 4         /* blk.L.attn_q.weight        [d, Hq*hd]    */
#define SFK_T_ATTN_K 5         /* blk.L.attn_k.weight        [d, Hkv*hd]   */
#define SFK_T_ATTN_V 6         /* blk.L.attn_v.weight        [d, Hkv*hd]   */
#define SFK_T_ATTN_OUT 7       /* blk.L.attn_output.weight   [Hq*hd, d]    */
#define SFK_T_FFN_NORM 8       /* blk.L.ffn_norm.weight      [d]   F32     */
#define SFK_T_FFN_GATE_INP 9   /* blk.L.ffn_gate_inp.weight  [d, E] F32    */
#define SFK_T_FFN_GATE_EXPS 10 /* blk.L.ffn_gate_exps.weight [d, F, E]     */
#define SFK_T_FFN_UP_EXPS 11   /* blk.L.ffn_up_exps.weight   [d, F, E]     */
#define SFK_T_FFN_DOWN_EXPS 12 /* blk.L.ffn_down_exps.weight [F, d, E]     */

#define SFK_KV_F32 0
#define SFK_KV_F16 1

/* Model shape and engine options.  The first block mirrors
 * engine::EngineHParams (engine.h:41-55); types name the quantization of each
 * weight class; kv_type selects the KV cache element type (the reference keeps
 * F32 K/V, engine.cpp:1253-1286; F16 pages halve the attention bytes);
 * max_batch bounds the sequences decoded per step (sfk_forward_batch). */
typedef struct sfk_hparams {
    int32_t n_embd, n_head, n_head_kv, n_layer, n_ff, n_expert, n_expert_used, n_vocab, n_ctx;
    float rms_eps, freq_base;
    int32_t type_embd, type_attn, type_ffn_gu, type_ffn_down, type_output;
    int32_t kv_type;
    int32_t max_batch;
    /* Expert parallelism (experts sharded across the GPUs of one box).
     * ep_size ranks, one engine per GPU; rank ep_rank holds
     * experts [ep_rank * E / ep_size, (ep_rank + 1) * E / ep_size) of every
     * layer.  When both head counts divide by ep_size and a rank's query
     * columns are whole 256-column blocks, the rank also holds only its share
     * of the attention heads (their Q/K/V rows, output-projection columns and
     * KV pages; the environment variable SFK_HEAD_PARALLEL=0 keeps them
     * replicated); everything else is a full copy.  0 or 1: no sharding. */
    int32_t ep_size, ep_rank;
    /* Attention head width; 0 = n_embd / n_head (the reference's rule,
     * engine.cpp:1161).  Set it when n_head * head_dim != n_embd. */
    int32_t head_dim;
    /* HBM slots for routed expert bundles (the reference's expert_slots,
     * Engine::load engine.h:153, engine.cpp:1386-1422).  0 or >= n_layer *
     * n_expert: every expert resident.  Otherwise the bundles live in pinned
     * host memory and a bounded pool of this many HBM slots holds the working
     * set: a layer-stratified LRU (SlotPool, src/tws/weight_store.h:69-266;
     * SFK_POOL_GLOBAL_LRU=1 selects the single global LRU), refilled by one
     * host-to-device copy per missing bundle on a copy stream, with the next
     * layer's predicted experts prefetched (ExpertPredictor,
     * src/predict/predictor.h) into free slots (SFK_PREFETCH=2: evicting
     * within that layer; SFK_PREFETCH=0: off).  The expert
     * kernels read the slots in place, so a pool must hold one step's routed
     * experts of a layer: at least min(n_expert, max_batch * n_expert_used).
     * Single-GPU engines only (ep_size <= 1). */
    int32_t expert_slots;
    /* Resident KV window in tokens (the reference's kv_window, KvStore
     * src/kv/kv_store.h:30-95; engine.cpp:1633-1762).  0 or >= n_ctx: the
     * whole context's KV stays in HBM.  Otherwise each sequence keeps its most
     * recent ceil(kv_window / 16) 16-token pages in HBM, written as a ring;
     * the page a new position would overwrite is first copied to a pinned
     * host cold store, and every layer's attention reads the cold pages
     * staged back into one layer's worth of HBM -- lossless: the same keys
     * and values in the same order as the resident cache.  Positions of a
     * sequence move forward (a position whose page has gone cold is refused);
     * at least two pages; single-GPU engines only. */
    int32_t kv_window;
} sfk_hparams;

typedef struct sfk_engine sfk_engine;

/* Message of the most recent failure on this thread (never NULL). */
SFK_API const char *sfk_last_error(void);
SFK_API const char *sfk_status_str(sfk_status s);

/* ---- engine lifecycle: replaces engine::Engine::load (engine.h:153-157,
 *      engine.cpp:983) for the HBM-resident case --------------------------
 * Allocates the HBM weight tier (every expert resident: the reference's
 * expert_slots = 0 "auto" working set, engine.cpp:1389-1394), the paged KV
 * cache (16-token pages, one page table per sequence) and the step buffers on
 * CUDA device `device`.  Weights are uninitialised until sfk_weights_put or
 * sfk_weights_synth. */
SFK_API sfk_status sfk_engine_create(int device, const sfk_hparams *hp, sfk_engine **out);
SFK_API void sfk_engine_free(sfk_engine *eng);
/* The engine's cudaStream_t: every call on this engine is ordered on it, so a
 * caller can record events or order its own work against the decode steps. */
SFK_API void *sfk_engine_stream(sfk_engine *eng);

/* Upload one tensor's verbatim GGUF bytes (host) into the HBM tier; the bytes
 * are what StrataReader::read_bundle / read_trunk_tensor return
 * (src/tws/strata_file.cpp:368,462) and what a GGUF stores.  Quantized
 * matrices are re-laid out on the device for coalesced streaming; the byte
 * count streamed per token is unchanged.  `ne` is the ggml shape. */
SFK_API sfk_status sfk_weights_put(sfk_engine *eng, int tensor, int layer, int ggml_type, const int64_t ne[3],
                           const void *host_bytes, size_t n_bytes);
/* One routed expert bundle gate|up|down as the .strata stores it
 * (src/tws/strata_format.h:122-130: gate_rel = 0, up_rel = gate_len,
 * down_rel = gate_len + up_len) -- the SlotPool::acquire load path
 * (src/tws/weight_store.h:174) with HBM as the tier. */
SFK_API sfk_status sfk_expert_put(sfk_engine *eng, int layer, int expert, const void *bundle, size_t n_bytes);
/* Read a tensor back as GGUF bytes (host). */
SFK_API sfk_status sfk_weights_get(sfk_engine *eng, int tensor, int layer, void *host_out, size_t n_bytes);
/* Fill every tensor with the seeded synthetic generator on the device (norms
 * = 1, other tensors N(0, 0.02) as Irwin-Hall(12) then quantized).  Produces
 * the same bytes as the CPU fixture generator for the same seed. */
SFK_API sfk_status sfk_weights_synth(sfk_engine *eng, uint64_t seed);
/* Bytes of a tensor in GGUF layout (0 for an unknown tensor). */
SFK_API size_t sfk_tensor_bytes(const sfk_engine *eng, int tensor, int layer);

/* ---- .strata files (src/tws/strata_format.h:77-177): the reader and the
 *      HBM loader.  Host-only except sfk_strata_load. ---------------------- */
typedef struct sfk_strata sfk_strata;
/* StrataReader::open (src/tws/strata_file.cpp:30-230): superblock v1/v2/v3
 * (header CRC32 checked), embedded GGUF metadata, expert index, optional trunk
 * index (checked against the GGUF-order trunk walk).  Files whose expert blobs
 * are LZ-compressed (v3 flag bit 3) are rejected with SFK_ERR_UNSUPPORTED. */
SFK_API sfk_status sfk_strata_open(const char *path, sfk_strata **out);
SFK_API void sfk_strata_close(sfk_strata *s);
/* The model-shape fields of *hp from the GGUF keys and tensor shapes, as
 * Engine::load reads them (src/model/engine/engine.cpp:1078-1087,1131-1137);
 * kv_type, max_batch, ep_size, ep_rank are left as the caller set them, and
 * n_ctx too unless it is <= 0 (then llama.context_length). */
SFK_API sfk_status sfk_strata_hparams(const sfk_strata *s, sfk_hparams *hp);
/* The GGUF tensor table: name, ggml type, ne, ggml_nbytes, and whether the
 * tensor lives in the expert bundles rather than the trunk block. */
SFK_API int64_t sfk_strata_n_tensors(const sfk_strata *s);
SFK_API sfk_status sfk_strata_tensor_info(const sfk_strata *s, int64_t i, char *name, size_t name_cap, int32_t *type,
                                          int64_t ne[4], uint64_t *n_bytes, int32_t *is_expert);
/* One trunk tensor's verbatim bytes (StrataReader::read_at over the trunk
 * block, engine.cpp:786-830: trunk tensors packed in GGUF order). */
SFK_API sfk_status sfk_strata_read_trunk(const sfk_strata *s, const char *name, void *host_out, size_t n_bytes);
/* StrataReader::read_bundle (src/tws/strata_file.cpp:368-444): the bundle
 * gate|up|down of (layer, expert), each slice read at its *_rel offset. */
SFK_API size_t sfk_strata_bundle_bytes(const sfk_strata *s, int32_t layer);
SFK_API sfk_status sfk_strata_read_bundle(const sfk_strata *s, int32_t layer, int32_t expert, void *host_out,
                                          size_t n_bytes);
/* Engine::load_strata_weights (engine.cpp:556-830) for the HBM tier: every
 * trunk tensor through sfk_weights_put, every bundle through sfk_expert_put.
 * An expert-parallel engine reads only its own experts' bundles and, when its
 * attention heads are split over the ranks, uploads its heads' rows of Q, K,
 * V and its heads' columns of the output projection.  The engine must have
 * been created with sfk_strata_hparams' shape. */
SFK_API sfk_status sfk_strata_load(const sfk_strata *s, sfk_engine *eng);
/* Pack a GGUF checkpoint into a .strata file: the reference's
 * pack_gguf_to_strata (src/tws/strata_pack.h:16-46, strata_pack.cpp:251-1108)
 * without its optional LZ compression.  Weight bytes are copied verbatim;
 * stacked (blk.N.ffn_*_exps) and per-expert (blk.N.ffn_*.E) expert tensors
 * become one gate|up|down bundle per (layer, expert); a file mixing the two,
 * one whose metadata declares experts none of which are found, and fused
 * gate_up expert tensors are refused.  Tensor types: F32, F16, Q8_0, Q4_K,
 * Q6_K.  Host-only; a failed pack removes its partial output. */
SFK_API sfk_status sfk_strata_pack(const char *gguf_path, const char *strata_path);

/* ---- decode: replaces Engine::forward / reset_kv (engine.h:241,245) ----- */
/* Clear every sequence's KV so the next step starts at position 0. */
SFK_API sfk_status sfk_kv_reset(sfk_engine *eng);
/* One token of sequence 0 at `pos` (0 <= pos < n_ctx), attending over
 * positions 0..pos.  logits_host (optional, n_vocab floats) receives the
 * logits; argmax_out (optional) the greedy token (first max wins,
 * engine.cpp:3111-3121). */
SFK_API sfk_status sfk_forward(sfk_engine *eng, int32_t token, int32_t pos, float *logits_host, int32_t *argmax_out);
/* One step of n_seq <= max_batch independent sequences: sequence s takes
 * tokens[s] at positions[s].  logits_host: [n_seq][n_vocab] or NULL. */
SFK_API sfk_status sfk_forward_batch(sfk_engine *eng, int32_t n_seq, const int32_t *tokens, const int32_t *positions,
                             float *logits_host, int32_t *argmax_out);
/* Greedy decode of n_steps tokens for the first n_seq sequences, continuing
 * from the last sfk_forward/_batch step (its argmax is the first input).
 * The loop runs on the device as one captured CUDA graph per step, with no
 * host round trip; tokens_out: [n_steps][n_seq] (host). */
SFK_API sfk_status sfk_decode_greedy(sfk_engine *eng, int32_t n_seq, int32_t n_steps, int32_t *tokens_out);
/* Batched prompt prefill: tokens[0..n) of sequence `seq` at positions
 * pos0 .. pos0 + n - 1 (pos0 + n <= n_ctx), every layer run over a chunk of
 * up to 512 prompt tokens at once (tensor-core GEMMs; routed pairs grouped by
 * expert; each token attends over its own prefix).  It replaces feeding the
 * prompt one position per Engine::forward call (tests/test_engine_oracle.cpp:
 * 182-187): the KV cache, the next position and the argmax key end as they
 * would after the last prompt token's forward, so sfk_decode_greedy
 * continues from it.  logits_host (optional, n_vocab floats) and argmax_out
 * (optional) receive the last prompt token's logits and greedy token.  The
 * GEMMs add the 256-column blocks of a row in order, so values differ from
 * token-by-token decode in fp32 rounding only.  One GPU (no expert
 * parallelism). */
SFK_API sfk_status sfk_prefill(sfk_engine *eng, int32_t seq, const int32_t *tokens, int32_t n, int32_t pos0,
                               float *logits_host, int32_t *argmax_out);

/* Sampling of the generate loop: the reference's sf_sampling_params
 * (include/strataflow/strataflow.h:193-199) plus the end-of-sequence token
 * (the reference asks its model; -1: none).  temperature <= 0 is greedy (the
 * argmax, first maximum wins); otherwise p_i = exp((l_i - max l) / T), the
 * top_k largest kept (<= 0: all; ties by the lower index), then the shortest
 * prefix in (p descending, index ascending) order whose mass reaches top_p
 * of the kept mass (>= 1: all), drawn by inverse CDF in index order with
 * u = splitmix64(seed + (step + 1) * 0x9E3779B97F4A7C15) / 2^64 (53 bits),
 * step = the generated token's index.  On the device. */
typedef struct sfk_sampling {
  float temperature;
  float top_p;
  int32_t top_k;
  uint64_t seed;
  int32_t max_tokens; /* <= 0: 256, the reference's default cap */
  int32_t eos_token;
} sfk_sampling;
/* The reference's defaults (strataflow_api.cpp:89-97): greedy, top_p 1,
 * top_k 0, seed 0, 256 tokens; eos_token -1. */
SFK_API sfk_sampling sfk_sampling_defaults(void);
/* Called with each generated token; a nonzero return stops the loop. */
typedef int (*sfk_token_cb)(int32_t token, void *user);
/* The reference's sf_generate drive (strataflow_api.cpp:308-335) on sequence
 * 0, with its prompt defect fixed: EVERY prompt token is fed at its position
 * (batched, sfk_prefill) continuing from the sequence's next position, not
 * only the last one.  Then up to max_tokens tokens (and at most cap_out, and
 * n_ctx) are generated one decode step at a time; the loop stops before
 * emitting eos_token, or after the callback (optional) returns nonzero.
 * tokens_out (optional) receives the generated tokens, *n_out their count. */
SFK_API sfk_status sfk_generate(sfk_engine *eng, const int32_t *prompt, int32_t n_prompt, const sfk_sampling *sampling,
                                int32_t *tokens_out, int32_t cap_out, int32_t *n_out, sfk_token_cb cb, void *user);

/* The generate loop's sampler as an operator: one token from n_vocab device
 * logits (f32) under `sampling` (temperature > 0) at generated-token index
 * `step`; *token_out (host) receives it. */
SFK_API sfk_status sfk_sample_logits(const float *dev_logits, int32_t n_vocab, const sfk_sampling *sampling,
                                     int32_t step, int32_t *token_out, void *stream);

/* ---- per-layer entry points: the reference's segment structure ---------
 * For a host engine that keeps its own layer loop (engine.cpp:2498-3025 runs
 * an attention segment and an expert segment per layer, engine.cpp:
 * 1854-1989).  n_tok sequences 0 .. n_tok-1 of the engine, one token each;
 * `hidden` is a DEVICE buffer [n_tok][n_embd] f32 read and written in place;
 * `positions` are host [n_tok].  Each call runs on the engine's stream and
 * returns after its kernels finished (their device status checked).  The
 * chain embed -> L x (attn, moe) -> lm_head computes exactly what
 * sfk_forward_batch computes.  Single-GPU engines (ep_size <= 1). */
/* token_embd rows of `tokens` (host [n_tok]) into hidden (engine.cpp:2708-2723) */
SFK_API sfk_status sfk_embed(sfk_engine *eng, const int32_t *tokens, const int32_t *positions, int32_t n_tok,
                             float *dev_hidden);
/* attn_norm -> Q/K/V -> RoPE -> KV append at `positions` -> GQA attention ->
 * O-projection + residual (engine.cpp:1878-1906) */
SFK_API sfk_status sfk_decode_layer_attn(sfk_engine *eng, int32_t layer, const int32_t *positions, int32_t n_tok,
                                         float *dev_hidden);
/* ffn_norm -> router softmax / top-k -> routed gate/up + SwiGLU -> routed down
 * -> weighted combine + residual (engine.cpp:1909-1986).  dev_ids_out /
 * dev_w_out (optional, DEVICE [n_tok][n_expert_used]) receive the routing. */
SFK_API sfk_status sfk_decode_layer_moe(sfk_engine *eng, int32_t layer, int32_t n_tok, float *dev_hidden,
                                        int32_t *dev_ids_out, float *dev_w_out);
/* output_norm -> lm_head -> argmax (engine.cpp:2988-3006): dev_logits_out
 * (optional, DEVICE [n_tok][n_vocab]) and argmax_out (optional, host
 * [n_tok]). */
SFK_API sfk_status sfk_lm_head(sfk_engine *eng, const float *dev_hidden, int32_t n_tok, float *dev_logits_out,
                               int32_t *argmax_out);

/* Routing of the last layer of the last step: ids [n_seq][k] and weights
 * [n_seq][k] (host) -- the router segment's read-back (engine.cpp:2823-2833). */
SFK_API sfk_status sfk_route_get(sfk_engine *eng, int32_t *ids_out, float *w_out, size_t n);

/* Step buffers of the last layer of the last step, for inspection:
 * which = 0 attention output [n_seq][Hq*hd], 1 ffn_inp [n_seq][d],
 * 2 q after RoPE [n_seq][Hq*hd], 3 SwiGLU activation [n_seq*k][n_ff]. */
SFK_API sfk_status sfk_debug_get(sfk_engine *eng, int32_t which, float *host_out, size_t n_floats);

/* Hidden state after the last step, [n_seq][n_embd] (host). */
SFK_API sfk_status sfk_hidden_get(sfk_engine *eng, float *host_out, size_t n_floats);

/* Average device time (ms) of each kernel of one decode step, launched
 * `iters` times back to back on the engine's stream, layer = i % n_layer so
 * consecutive launches stream different weights.  ms_out[8]: embed, qkv,
 * attention, o_proj, router, gate_up, down, lm_head.  Needs one prior step
 * (routing and KV state are reused); afterwards the step state is undefined,
 * so call sfk_kv_reset before decoding again. */
SFK_API sfk_status sfk_time_kernels(sfk_engine *eng, int32_t n_seq, int32_t iters, float *ms_out, int32_t n_out);

typedef struct sfk_stats {
    uint64_t weight_bytes_hbm;   /* resident weight bytes (HBM tier) */
    uint64_t kv_bytes_hbm;       /* reserved KV cache bytes */
    uint64_t scratch_bytes_hbm;  /* step buffers */
    uint64_t steps;              /* decode steps run */
    uint64_t kernels_per_step;   /* kernel launches per decode step */
    uint64_t active_bytes_per_token; /* weight bytes one b=1 token streams */
    /* bounded expert tier (zero when every expert is resident): the
     * reference's CacheStats (weight_store.h) and prefetch counters
     * (engine.cpp:187-201) */
    uint64_t pool_slots;         /* HBM expert slots */
    uint64_t pool_hits;          /* acquires that found the bundle resident */
    uint64_t pool_misses;        /* acquires that copied the bundle in */
    uint64_t pool_evictions;     /* bundles displaced from a slot */
    uint64_t h2d_expert_bytes;   /* bundle bytes copied host -> HBM */
    uint64_t prefetch_warmed;    /* bundles copied in ahead of their layer */
    uint64_t prefetch_used;      /* of those, routed when their layer ran */
    /* KV window (zero without one) */
    uint64_t kv_window_pages;    /* HBM pages per sequence */
    uint64_t kv_pages_evicted;   /* pages moved to the cold store */
    uint64_t kv_staged_bytes;    /* cold K/V bytes staged back for attention */
} sfk_stats;
SFK_API sfk_status sfk_get_stats(const sfk_engine *eng, sfk_stats *out);

/* ---- the bounded expert tier's host logic (no GPU needed) ---------------
 * The slot pool and the predictor the engine drives when expert_slots bounds
 * the HBM tier, exposed for the host-side tests.  sfk_pool restates
 * SlotPool (src/tws/weight_store.h:69-266, weight_store.cpp): n_layer == 0
 * gives the global-LRU pool (the two-argument constructor), otherwise the
 * layer-stratified one.  Pins (an addition: slots still read by queued
 * kernels) keep a slot from being chosen as a victim. */
typedef struct sfk_pool sfk_pool;
SFK_API sfk_status sfk_pool_create(uint32_t n_slots, uint32_t n_layer, uint32_t n_expert, uint32_t n_expert_used,
                                   sfk_pool **out);
SFK_API void sfk_pool_free(sfk_pool *pool);
/* SlotPool::acquire: the slot of (layer, expert), loading it on a miss
 * (*miss_out = 1); -1 when there is no slot (n_slots 0, or all victims
 * pinned). */
SFK_API int64_t sfk_pool_acquire(sfk_pool *pool, uint32_t layer, uint32_t expert, int32_t *miss_out);
SFK_API int32_t sfk_pool_resident(const sfk_pool *pool, uint32_t layer, uint32_t expert);
SFK_API int32_t sfk_pool_stratified(const sfk_pool *pool);
SFK_API uint32_t sfk_pool_layer_capacity(const sfk_pool *pool, uint32_t layer);
SFK_API int32_t sfk_pool_has_free_slot_in_layer(const sfk_pool *pool, uint32_t layer);
SFK_API sfk_status sfk_pool_set_layer_weights(sfk_pool *pool, const uint64_t *weights, uint32_t n_layer);
SFK_API sfk_status sfk_pool_pin(sfk_pool *pool, uint32_t slot);
SFK_API sfk_status sfk_pool_unpin_all(sfk_pool *pool);
/* hits, misses, evictions */
SFK_API sfk_status sfk_pool_stats(const sfk_pool *pool, uint64_t out[3]);
/* ExpertPredictor (src/predict/predictor.h:15-43): per-layer activation
 * counts; predict() returns up to k experts, most frequent first (equal
 * counts by the lower id) and the count written. */
typedef struct sfk_predictor sfk_predictor;
SFK_API sfk_status sfk_predictor_create(uint32_t n_layer, uint32_t n_expert, sfk_predictor **out);
SFK_API void sfk_predictor_free(sfk_predictor *pred);
SFK_API sfk_status sfk_predictor_observe(sfk_predictor *pred, uint32_t layer, uint32_t expert);
SFK_API uint32_t sfk_predictor_predict(sfk_predictor *pred, uint32_t layer, uint32_t k, uint32_t *out);
SFK_API double sfk_predictor_accuracy(const sfk_predictor *pred);
SFK_API sfk_status sfk_predictor_layer_activity(const sfk_predictor *pred, uint64_t *out, uint32_t n_layer);

/* ---- operator-level entry points (device pointers, caller's stream) -----
 * `stream` is a cudaStream_t (NULL = legacy default stream). */

/* Bytes of one row of K columns of `ggml_type` in the device layout. */
SFK_API int64_t sfk_dev_row_bytes(int ggml_type, int64_t K);
/* GGUF rows -> device layout and back (nrows rows of K columns). */
SFK_API sfk_status sfk_repack(int ggml_type, const void *dev_gguf, void *dev_out, int64_t nrows, int64_t K, void *stream);
SFK_API sfk_status sfk_unpack(int ggml_type, const void *dev_in, void *dev_gguf, int64_t nrows, int64_t K, void *stream);

/* ggml dequantize_row_* (bit-exact) of n elements of GGUF-layout data. */
SFK_API sfk_status sfk_dequantize(int ggml_type, const void *dev_src, float *dev_dst, int64_t n, void *stream);

/* Quantize b activation rows [b][K] (f32) to Q8_K or Q8_0 blocks in GGUF
 * block layout (ggml quantize_row_q8_K_ref / quantize_row_q8_0_ref). */
SFK_API sfk_status sfk_quantize_act(int act_type, const float *dev_x, int32_t b, int64_t K, void *dev_out, void *stream);

/* ggml_mul_mat: y[t][r] = W[r,:] . x[t] for a [rows x K] weight in device
 * layout, b <= 16 activation rows; activations quantized the ggml way. */
SFK_API sfk_status sfk_mul_mat(int ggml_type, const void *dev_w, int64_t rows, int64_t K, const float *dev_x, int32_t b,
                       float *dev_y, void *stream);

/* The same product for many activation rows at once on the tensor cores
 * (tcgen05 kind::i8): y[t][r] = W[r,:] . x[t], t < n (any n >= 1), the
 * activations quantized the ggml way and the sub-block integer dots exact; the
 * fp32 sum over 256-column blocks is taken in block order.  For prefill and
 * large batches (the reference feeds a prompt one position per call,
 * tests/test_engine_oracle.cpp:182-187; this is the batched form of
 * ggml_mul_mat, engine.cpp:1882-1889). */
SFK_API sfk_status sfk_mul_mat_tc(int ggml_type, const void *dev_w, int64_t rows, int64_t K, const float *dev_x,
                                  int32_t n, float *dev_y, void *stream);

/* ggml_mul_mat_id for the routed experts (engine.cpp:1967-1970):
 * w: stacked [E][rows][K] (device layout), x: [b][K] (one row per token,
 * broadcast over its k experts) or [b][k][K] when x_per_pair,
 * ids: [b][k] int32, y: [b][k][rows]. */
SFK_API sfk_status sfk_mul_mat_id(int ggml_type, const void *dev_w, int32_t n_expert, int64_t rows, int64_t K,
                          const float *dev_x, int32_t x_per_pair, const int32_t *dev_ids, int32_t b, int32_t k,
                          float *dev_y, void *stream);

/* sfk_mul_mat_id on the tensor cores, for batches whose routed pairs give
 * the experts many activation rows (b * k in the tens and up): the pairs are
 * grouped by expert into 64-row tiles, each tile is a tcgen05 kind::i8 GEMM
 * against its expert's matrix (sfk_mul_mat_tc's arithmetic: exact sub-block
 * integer dots, fp32 sum over 256-column blocks in block order), and the rows
 * are put back in pair order.  Same arguments and layout as sfk_mul_mat_id,
 * any b >= 1 with b * k <= 2^20, n_expert <= 1024; an id outside
 * [0, n_expert) returns SFK_ERR_RUNTIME.  Synchronizes the stream. */
SFK_API sfk_status sfk_mul_mat_id_tc(int ggml_type, const void *dev_w, int32_t n_expert, int64_t rows, int64_t K,
                                     const float *dev_x, int32_t x_per_pair, const int32_t *dev_ids, int32_t b,
                                     int32_t k, float *dev_y, void *stream);

/* The fused routed-expert FFN of build_expert_segment (engine.cpp:1956-1989):
 * out[t] = res[t] + sum_j w[t][j] * Down_e( silu(Gate_e x[t]) * Up_e x[t] ),
 * e = ids[t][j].  gate/up: [E][F][d], down: [E][d][F] (device layout);
 * x, res, out: [b][d]; res may be NULL. */
SFK_API sfk_status sfk_moe_ffn(int type_gu, int type_down, const void *dev_gate, const void *dev_up, const void *dev_down,
                       int32_t n_expert, int64_t d, int64_t F, const float *dev_x, const float *dev_res,
                       const int32_t *dev_ids, const float *dev_w, int32_t b, int32_t k, float *dev_out,
                       void *stream);

/* sfk_moe_ffn computed without allocating device memory.  No counterpart in
 * the reference: it exists for callers that cannot let a library call
 * cudaMalloc -- an engine whose planner already handed all of HBM to its own
 * pools, a process whose device memory belongs to another framework's
 * allocator, or a latency-critical loop where cudaMalloc/cudaFree would
 * synchronize the device.  Same arguments and result as sfk_moe_ffn.  Its
 * scratch lives in one fixed array of SFK_NOALLOC_SCRATCH_BYTES compiled into
 * the library (every GPU that loads the library holds it until exit); a shape
 * whose scratch does not fit (roughly b*k*F*4 + b*k*F*1.2 + b*d*1.2 bytes) is
 * rejected with SFK_ERR_INVALID_ARGUMENT before any work is queued.  The first
 * call on a device looks up the array's device address (cudaGetSymbolAddress)
 * and keeps it for the later calls on that device.  All calls
 * share the array and it keeps the last call's contents (the call clears what
 * must start at zero): calls whose work overlaps on the GPU (other streams,
 * other threads on the same device) race on it.  The call returns only after
 * its work is done: it copies the device status word back into a host
 * variable and synchronizes `stream` before returning. */
#define SFK_NOALLOC_SCRATCH_BYTES (4u << 20)
SFK_API sfk_status sfk_moe_ffn_noalloc(int type_gu, int type_down, const void *dev_gate, const void *dev_up,
                                       const void *dev_down, int32_t n_expert, int64_t d, int64_t F,
                                       const float *dev_x, const float *dev_res, const int32_t *dev_ids,
                                       const float *dev_w, int32_t b, int32_t k, float *dev_out, void *stream);

/* ---- expert parallelism (no counterpart in the reference, which runs one
 *      device; the north star shards the experts over the GPUs of a box) ----
 * Every rank's engine exposes one exchange buffer (partial MoE outputs and
 * flag words).  Each rank passes sfk_ep_handle's bytes (SFK_EP_HANDLE_BYTES,
 * a CUDA IPC handle) to every other rank by its own means (e.g. a
 * torch.distributed all-gather); sfk_ep_connect then opens every rank's
 * buffer.  Connect before the first decode step.  All ranks must run the
 * same steps (same tokens, positions and batch) in the same order: after
 * every layer's expert FFN the ranks exchange partial outputs through peer
 * memory and add them in rank order, so every rank holds the same hidden
 * state and produces the same logits.  Waits for a peer are bounded (about a
 * second) and end the step with SFK_ERR_RUNTIME. */
#define SFK_EP_HANDLE_BYTES 64
SFK_API sfk_status sfk_ep_handle(sfk_engine *eng, void *handle_out, size_t n_bytes);
SFK_API sfk_status sfk_ep_connect(sfk_engine *eng, const void *handles, int32_t n_ranks);

/* GQA decode attention over a paged KV cache (engine.cpp:1751-1761 math):
 * q [b][Hq][hd] f32; k_pages/v_pages [n_pages][Hkv][16][hd] (f16 or f32 per
 * kv_type); page_table [b][max_pages] of ids in [0, n_pages); positions [b]:
 * sequence t attends over 0..positions[t]; out [b][Hq*hd].  A page id outside
 * the pool is never dereferenced: the call returns SFK_ERR_RUNTIME. */
SFK_API sfk_status sfk_attn_decode_paged(const float *dev_q, const void *dev_k_pages, const void *dev_v_pages, int32_t kv_type,
                                 int32_t n_pages, const int32_t *dev_page_table, int32_t max_pages, const int32_t *dev_positions,
                                 int32_t b, int32_t n_head, int32_t n_head_kv, int32_t head_dim, float *dev_out,
                                 void *stream);

#ifdef __cplusplus
}
#endif
#endif /* SFK_H */
