// sfk_kernels.cuh -- kernel parameter blocks and launch entry points shared by
// sfk_kernels.cu (device code) and sfk_api.cu (host orchestration).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

struct sfk_engine;  // include/sfk.h

namespace sfk {

constexpr int MAXP = 128;  // max (token, expert) pairs per step  (b * k)
constexpr int MAXB = 16;   // max tokens per step
constexpr int NW = 8;      // consumer warps of the producer/consumer streaming kernel
constexpr int RING_BYTES = 96 * 1024;
constexpr int MAXR = 8;    // max expert-parallel ranks

// Routing of one MoE step, written by the router kernel (device memory).
// Pair p = t * k + j is token t's j-th routed expert.  Slots are the distinct
// experts in use; each slot lists its pairs in ascending pair order.
struct Route {
  int n_slots;
  int k;
  int b;
  int pad;
  int slot_expert[MAXP];
  int slot_off[MAXP + 1];
  int slot_pairs[MAXP];
  int ids[MAXP];
  float w[MAXP];
  int pad2[3];  // size a multiple of 16 bytes: one bulk copy moves it
};
static_assert(sizeof(Route) % 16 == 0, "Route is moved by 1-D bulk copies");

enum Prologue : int {
  PRO_QUANT = 0,  // x f32 [b][K] (+ optional RMSNorm * w) -> quantize to act type
  PRO_LOAD = 1,   // copy precomputed qact vectors from global
  PRO_ROUTE = 2,  // gate/up: ffn_norm + quantize + router + top-k in the prologue
};
enum Epilogue : int {
  EPI_STORE = 0,    // y[pair][row] = dot            (mul_mat / mul_mat_id)
  EPI_QKV = 1,      // RoPE, q -> qbuf, k/v -> paged KV cache
  EPI_RESID = 2,    // y[t][row] = dot + res[t][row]
  EPI_GATEUP = 3,   // h = silu(gate)*up -> h f32, Q8_K/Q8_0 quant per 256-row group
  EPI_DOWN = 4,     // y[t][row] = sum_j w_tj * dot_tj + res[t][row]
  EPI_LMHEAD = 5,   // logits (optional) + per-token argmax (atomicMax)
};

struct KvView {
  void* k;               // [n_pages][Hkv][16][hd]  (f16 or f32)
  void* v;
  const int* page_table; // [b][max_pages]
  int max_pages;
  int n_pages;           // pages in the pool (page ids are checked against it)
  int n_head_kv;
  int head_dim;
  int f16;
  // KV window: ids from n_hot up name the cold pages staged for this layer
  // at k2 / v2 (page id - n_hot); n_hot = 0: every id addresses k / v.
  // Only pages below n_hot are written.
  void* k2;
  void* v2;
  int n_hot;
};

// Address of page `pg` of K (v = 0) or V (v = 1), `page_bytes` apart.
__host__ __device__ __forceinline__ const uint8_t* kv_page(const KvView& kv, int v, int pg, int64_t page_bytes) {
  const bool cold = kv.n_hot > 0 && pg >= kv.n_hot;
  const void* base = cold ? (v ? kv.v2 : kv.k2) : (v ? kv.v : kv.k);
  return static_cast<const uint8_t*>(base) + (int64_t)(cold ? pg - kv.n_hot : pg) * page_bytes;
}
// A page id that may be written: inside the pool and not a staged cold page.
__host__ __device__ __forceinline__ bool kv_page_writable(const KvView& kv, int pg) {
  return pg >= 0 && (kv.n_pages <= 0 || pg < kv.n_pages) && (kv.n_hot <= 0 || pg < kv.n_hot);
}

// Shared-memory plan of the warp-tile streaming kernel (computed on the host
// at launch; the kernel reads it from its parameters)
struct Plan2 {
  int nws;  // consumer warps (the block is nws * 32 threads)
  int occ;  // CTAs per SM the plan is sized for (1, or 2 so the next kernel's CTAs can start beside this one's)
  int stages, R, G, tile_bytes;
  int ring_off, xq_off, acc_off, red_off, route_off, xn_off, seg_off, probs_off, total;
  int xq_smem, xq_vec_bytes;
};

struct StreamParams {
  // weights (device layout)
  const uint8_t* w0;
  const uint8_t* w1;       // second matrix (up) when nmat == 2
  int64_t rowstride;
  int64_t expert_stride;   // bytes between experts of a stacked tensor
  int rows;                // rows per matrix
  int K;
  int wtype;
  int nmat;
  int act_type;            // T_Q8_K or T_Q8_0
  int row_align;           // CTA row ranges are multiples of this
  int rows_per_cta;        // ceil(rows / grid), aligned
  // tokens / routing
  int b;
  int k;                   // experts per token (1 for dense)
  int n_pairs;             // accumulator pairs: b (dense) or b*k (routed)
  int n_vec;               // activation vectors: b, or b*k when xq_by_pair
  const Route* route;      // null: dense (one slot, pairs = tokens)
  // prologue
  int pro;
  const float* x;          // PRO_QUANT input [b][K]
  const float* norm_w;     // RMSNorm weight or null (no norm)
  float eps;
  const uint8_t* qact;     // PRO_LOAD source
  int64_t qact_stride;     // bytes between qact vectors
  int xq_by_pair;          // PRO_LOAD: vector index = pair (1) or token (0)
  int xq_resident;         // all groups of all vectors fit in smem
  const float* w_r;        // PRO_ROUTE: F32 router [n_expert][K]; the routing is written to `route`
  int n_expert;
  float* logits;           // PRO_ROUTE: [b][n_expert] router logits, exchanged between the CTAs
  int* rsync;              // PRO_ROUTE: [2] arrival / departure counters, zero between launches
  // epilogue
  int epi;
  float* y;                // EPI_STORE / EPI_RESID / EPI_DOWN output; EPI_QKV q out
  const float* res;        // residual [b][rows]
  int64_t y_stride;        // floats between rows of y per vector (== rows)
  // EPI_QKV
  KvView kv;
  int n_head;
  const float* rope;       // [n_ctx][head_dim/2] (cos, sin) pairs, built on the host
  const int* pos;          // [b] positions
  // EPI_GATEUP
  float* h;                // [pairs][rows] f32
  uint8_t* hq;             // [pairs] qact of h (K = rows)
  int* grp_counter;        // [rows/256] counters, self-resetting
  int h_act_type;          // act type of the down projection
  // EPI_LMHEAD
  unsigned long long* argmax_key;  // [b]
  int store_logits;
  unsigned long long* clear_keys;  // zeroed by CTA 0 once the previous kernel finished (or null)
  int clear_n;
  int* status;
  // warp-tile kernel ring: tile target bytes and stages per warp (0: defaults)
  int s2_tile;
  int s2_stages;
  int s2_occ;  // 2: size the kernel for two CTAs per SM (half the shared memory and registers)
  // expert parallelism: this rank holds experts [ep_e0, ep_e0 + ep_eloc)
  // (ep_eloc = 0: all experts are local); routed tiles and the weighted
  // combine skip the others
  int ep_e0, ep_eloc;
  // EPI_LMHEAD: index of row 0 in the argmax keys (a rank's vocabulary slice)
  int argmax_base;
  // unrouted matrices: issue the first ring fill before waiting on the
  // previous kernel (the weights do not depend on it)
  int early_fill;
  // bounded expert tier: routed expert e is read from slot slot_map[e] of the
  // pool (w0 / w1 = the pool's matrices, expert_stride = the slot size);
  // null: experts are addressed directly
  const int* slot_map;
  int n_map_slots;
  Plan2 pl;  // filled by the launcher
};

struct AttnParams {
  const float* q;          // [b][Hq][hd]
  KvView kv;
  const int* pos;          // [b]; attends over 0..pos
  int b, n_head;
  int cluster;             // CTAs per (token, kv head): one thread-block cluster
  int max_chunk;           // positions per CTA at the longest context: ceil(max_pages / cluster) * 16
  float* out;              // [b][Hq*hd]
  int* status;
};

struct RouterParams {
  const float* x;          // [b][d] ffn_inp
  const float* norm_w;     // ffn_norm weight
  const float* w_r;        // [E][d] f32 router
  int b, d, E, k;
  float eps;
  int act_type;            // act quant type for gate/up weights
  uint8_t* xq;             // [b] qact of ffn_norm(x)
  float* xn;               // [b][d] ffn_norm(x) f32 (optional, may be null)
  Route* route;
  float* logits;           // [b][E] scratch
  int* counter;            // self-resetting
  int ep_e0, ep_eloc;      // local experts (ep_eloc = 0: all)
  int* status;
};

struct EmbedParams {
  const uint8_t* tok_embd; // GGUF layout rows [V][d], type `type`
  int type, d, V, b;
  const int* tok_in;       // host-supplied tokens [b]
  unsigned long long* argmax_key;  // [b]; greedy mode reads and resets it
  int greedy;
  int* tok_hist;           // [b] token consumed this step (out)
  const int* pos_in;       // [b] host-supplied positions (or null: use pos_state)
  int* pos_state;          // [b] persistent position counters (greedy loop)
  int* pos_cur;            // [b] position of this step (out)
  float* x;                // [b][d]
  unsigned* ep_step;       // expert parallelism: step counter the combine epochs derive from (or null)
  int* status;
};

// Combine of one layer stage across the ranks: every rank wrote its partial
// (stage 1: its local experts' weighted sum; stage 0: its heads' share of the
// output projection; plus the residual on rank 0) into slot
// parts[rank] + ((layer & 1) * 2 + stage) * half; x = sum of the ranks'
// partials in rank order, identical on every rank.  Peers signal through each
// other's flag words over peer memory (epoch = ep_epoch(step, n_layer, layer,
// stage)).
struct EpParams {
  const float* parts[MAXR];  // every rank's partial buffer (peer pointers; own buffer at [rank])
  unsigned* flags;           // this rank's flag words [MAXR] (peers write them)
  unsigned* peer_flags[MAXR];  // every rank's flag words
  int n_ranks, rank;
  int layer, n_layer;
  int stage;                 // 0: attention output projection, 1: expert FFN
  const unsigned* ep_step;
  int half;                  // floats in one partial slot ([layer parity][stage] slots)
  int n;                     // floats to combine (b * d)
  float* x;
  int* status;
};

// Combine epochs are 32-bit unsigned and wrap (after about 2^32 / (2 * n_layer)
// steps: ~35 M at 61 layers).  A flag has reached an epoch when the wrapped
// difference is non-negative, which stays correct across the wrap because
// ranks are never more than one stage apart (far less than 2^31 epochs).
__host__ __device__ inline unsigned ep_epoch(unsigned step, int n_layer, int layer, int stage) {
  return (step * (unsigned)n_layer + (unsigned)layer) * 2u + (unsigned)stage + 1u;
}
__host__ __device__ inline bool ep_reached(unsigned flag, unsigned epoch) { return (int)(flag - epoch) >= 0; }

// Grid, rows per CTA, activation residency and ring plan of one streaming
// launch (sfk_api.cu): the same plan for the engine, the operator calls and
// the no-allocation entry point.  Returns an sfk_status (0 = SFK_OK).
int plan_stream(StreamParams& p, int sm_count, int* grid_out);

// launch helpers (implemented in sfk_kernels.cu)
int stream_smem_bytes(const StreamParams& p, int* n_stages, int* stage_bytes, int* rows_per_warp);
int stream2_smem_bytes(const StreamParams& p);  // the warp-tile kernel's shared memory
int stream2_occupancy(const StreamParams& p);   // CTAs per SM its plan allows (0: the kernel cannot run it)
cudaError_t launch_stream(const StreamParams& p, int grid, cudaStream_t st, bool pdl);
cudaError_t launch_attn(const AttnParams& p, cudaStream_t st, bool pdl);
cudaError_t launch_ep_combine(const EpParams& p, cudaStream_t st, bool pdl);

// The lm_head's argmax across ranks when each rank scored a slice of the
// vocabulary: every rank publishes its b keys ((ordered value, ~index) as the
// lm_head epilogue writes them), raises its flag on every rank (epoch = the
// step counter), waits for all flags, and takes the maximum key per token --
// the first maximum of the whole vocabulary on every rank.
struct EpHeadParams {
  unsigned long long* key;                     // [b]: this rank's keys in, the global keys out
  unsigned long long* own_keys;                // this rank's published keys [b] (peers read them)
  const unsigned long long* peer_keys[MAXR];   // every rank's published keys
  unsigned* flags;                             // this rank's head flag words [MAXR]
  unsigned* peer_flags[MAXR];                  // every rank's head flag words
  int n_ranks, rank, b;
  const unsigned* ep_step;
  int* status;
};
cudaError_t launch_ep_argmax(const EpHeadParams& p, cudaStream_t st, bool pdl);
// clusters of `cluster` attention CTAs that fit on the device at once (0 if
// that cluster size cannot be launched)
int attn_active_clusters(int head_dim, int f16, int gqa, int cluster, int max_chunk);
size_t attn_smem_bytes(int hd, int gqa, int f16, int max_chunk);
cudaError_t launch_router(const RouterParams& p, cudaStream_t st, bool pdl);
cudaError_t launch_embed(const EmbedParams& p, cudaStream_t st, bool pdl);
cudaError_t launch_repack(int type, const uint8_t* src, uint8_t* dst, int64_t nrows, int K, cudaStream_t st);
cudaError_t launch_unpack(int type, const uint8_t* src, uint8_t* dst, int64_t nrows, int K, cudaStream_t st);
cudaError_t launch_dequant(int type, const uint8_t* src, float* dst, int64_t n, cudaStream_t st);
cudaError_t launch_synth(int type, uint64_t seed, float std_, uint8_t* dst_gguf, int64_t nrows, int K,
                         cudaStream_t st, int64_t row0 = 0, int64_t col0 = 0, int64_t kfull = 0);
cudaError_t launch_synth_f32(uint64_t seed, float std_, float* dst, int64_t n, cudaStream_t st);
cudaError_t launch_quant_act(int act_type, const float* x, int b, int K, uint8_t* dst, cudaStream_t st);
cudaError_t launch_fill_f32(float* dst, float v, int64_t n, cudaStream_t st);
cudaError_t launch_route_build(const int* ids, const float* w, int b, int k, int n_expert, Route* r, int* status,
                               cudaStream_t st);
// sets the message sfk_last_error() returns on the calling thread
void set_last_error(const char* msg);

// An engine's share of a sharded model (see engine_shard in sfk_api.cu).
struct EngineShard {
  int head_split, q0, hq_loc, kv0, hkv_loc, hd, e0, e_loc;
};
void engine_shard(const ::sfk_engine* e, EngineShard* out);
cudaError_t launch_quant_act_gguf(int act_type, const float* x, int b, int K, uint8_t* dst, cudaStream_t st);

}  // namespace sfk
