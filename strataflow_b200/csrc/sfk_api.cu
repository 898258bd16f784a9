// sfk_api.cu -- host side of the C ABI (include/sfk.h): the HBM weight tier,
// the paged KV cache, the per-step launch sequence and its CUDA graphs.
//
// One decode step (b sequences) is this launch chain on the engine's stream,
// each kernel launched with programmatic dependent launch so the next GEMV's
// weights stream while the previous kernel finishes:
//   embed -> L x [ qkv(norm+quant, RoPE, KV append) -> attention(split-K)
//               -> o_proj(+residual) -> router(norm, softmax, top-k)
//               -> gate_up(SwiGLU, requant) -> down(weighted combine + residual) ]
//   -> lm_head(norm, argmax)
// which is engine::Engine::forward (src/model/engine/engine.cpp:2498-3025) with
// every host round trip between its 2L+2 ggml segments removed.  The chain is
// captured once per (batch, token source) into a CUDA graph and replayed.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstddef>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <new>
#include <set>
#include <string>
#include <vector>

#include "../../include/sfk.h"
#include "sfk_dequant.cuh"
#include "sfk_device.cuh"
#include "sfk_kernels.cuh"
#include "sfk_mega.cuh"
#include "sfk_prefill.cuh"
#include "sfk_sample.cuh"
#include "sfk_tc.cuh"
#include "sfk_tier.h"

using namespace sfk;

namespace {

thread_local std::string g_err = "no error";

}  // namespace

namespace sfk {
void set_last_error(const char* msg) { g_err = msg; }
}  // namespace sfk

namespace {

sfk_status fail(sfk_status st, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return st;
}

#define CK(call)                                                                              \
  do {                                                                                        \
    cudaError_t e_ = (call);                                                                  \
    if (e_ != cudaSuccess)                                                                    \
      return fail(e_ == cudaErrorMemoryAllocation ? SFK_ERR_OUT_OF_MEMORY : SFK_ERR_RUNTIME,  \
                  "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__); \
  } while (0)

int act_for(int wtype) { return wtype == T_Q8_0 ? T_Q8_0 : T_Q8_K; }
bool quant_ok(int t) { return t == T_Q4_K || t == T_Q6_K || t == T_Q8_0; }

int sm_count_of(int dev) {
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

constexpr int XQ_RESIDENT_BUDGET = 48 * 1024;
constexpr int SMEM_LIMIT = 227 * 1024;

// fill in grid / rows_per_cta / xq_resident and check shared memory
// Ring shape of the warp-tile kernel: tile target bytes and stages per warp.
// 0 keeps the kernel's defaults; SFK_STREAM_TILE_BYTES / SFK_STREAM_STAGES
// override them (read once, for tuning on new parts).
struct StreamTuning {
  int tile = 0, stages = 0, occ = 0;
};
const StreamTuning& stream_tuning() {
  static const StreamTuning t = [] {
    StreamTuning r;
    if (const char* v = getenv("SFK_STREAM_TILE_BYTES")) r.tile = atoi(v);
    if (const char* v = getenv("SFK_STREAM_STAGES")) r.stages = atoi(v);
    if (const char* v = getenv("SFK_STREAM_OCC")) r.occ = atoi(v);
    return r;
  }();
  return t;
}

}  // namespace

namespace sfk {
// declared in sfk_kernels.cuh: also plans the no-allocation entry point's launches
sfk_status plan_stream(StreamParams& p, int sm_count, int* grid_out) {
  if (!p.s2_tile) p.s2_tile = stream_tuning().tile;
  if (!p.s2_stages) p.s2_stages = stream_tuning().stages;
  if (stream_tuning().occ == 2 && p.s2_occ == 0) {
    // two CTAs per SM: the next kernel's CTAs start beside this kernel's last ones
    StreamParams q = p;
    q.s2_occ = 2;
    int g2 = std::min(2 * sm_count, std::max(1, (q.rows + 7) / 8));
    int r2 = (q.rows + g2 - 1) / g2;
    r2 = (r2 + q.row_align - 1) / q.row_align * q.row_align;
    g2 = (q.rows + r2 - 1) / r2;
    q.rows_per_cta = r2;
    q.xq_resident = (int64_t)q.n_vec * qact_bytes(q.K) <= XQ_RESIDENT_BUDGET ? 1 : 0;
    if (q.pro == PRO_QUANT) q.xq_resident = 1;
    if (stream2_occupancy(q) == 2) {
      p = q;
      *grid_out = g2;
      return SFK_OK;
    }
  }
  p.s2_occ = 0;
  int grid = std::min(sm_count, std::max(1, (p.rows + 15) / 16));
  int rpc = (p.rows + grid - 1) / grid;
  rpc = (rpc + p.row_align - 1) / p.row_align * p.row_align;
  grid = (p.rows + rpc - 1) / rpc;
  p.rows_per_cta = rpc;
  p.xq_resident = (int64_t)p.n_vec * qact_bytes(p.K) <= XQ_RESIDENT_BUDGET ? 1 : 0;
  if (p.pro == PRO_QUANT) p.xq_resident = 1;
  const int smem = stream_smem_bytes(p, nullptr, nullptr, nullptr);
  if (smem > SMEM_LIMIT)
    return fail(SFK_ERR_UNSUPPORTED, "stream kernel needs %d B shared memory (rows %d, K %d, vectors %d)", smem,
                p.rows, p.K, p.n_vec);
  *grid_out = grid;
  return SFK_OK;
}
}  // namespace sfk

namespace {

// CTAs per (token, kv head) in the attention cluster: 8 (portable) unless a
// CTA would own more than 2048 positions at the longest context
int attn_cluster_for(int max_ctx) { return (max_ctx + 7) / 8 > 2048 ? 16 : 8; }

// cached scratch for operator-level calls, per device
struct OpScratch {
  void* buf = nullptr;
  size_t bytes = 0;
  Route* route = nullptr;
  int* status = nullptr;
  int* counters = nullptr;  // zeroed, self-resetting
  size_t n_counters = 0;
};
std::mutex g_op_mu;
std::map<int, OpScratch> g_op;

sfk_status op_scratch(size_t need, size_t n_counters, OpScratch** out) {
  int dev = 0;
  CK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_op_mu);
  OpScratch& s = g_op[dev];
  if (!s.route) {
    CK(cudaMalloc(&s.route, sizeof(Route)));
    CK(cudaMalloc(&s.status, sizeof(int)));
    CK(cudaMemset(s.status, 0, sizeof(int)));
  }
  if (s.bytes < need) {
    if (s.buf) cudaFree(s.buf);
    s.buf = nullptr;
    s.bytes = 0;
    CK(cudaMalloc(&s.buf, need));
    s.bytes = need;
  }
  if (s.n_counters < n_counters) {
    if (s.counters) cudaFree(s.counters);
    s.counters = nullptr;
    CK(cudaMalloc(&s.counters, n_counters * sizeof(int)));
    CK(cudaMemset(s.counters, 0, n_counters * sizeof(int)));
    s.n_counters = n_counters;
  }
  *out = &s;
  return SFK_OK;
}

// The host's answer to a status word already read back as h: OK, or the
// error it records (the device word is cleared for the next call).
sfk_status status_result(int* dev_status, int h) {
  if (h != ERR_NONE) {
    int z = 0;
    cudaMemcpy(dev_status, &z, sizeof(int), cudaMemcpyHostToDevice);
    return fail(SFK_ERR_RUNTIME, "device reported error %d (%s)", h,
                h == ERR_TIMEOUT    ? "bounded wait expired"
                : h == ERR_BAD_ID   ? "id out of range"
                : h == ERR_BAD_PAGE ? "page id outside the KV pool"
                                    : "bad position");
  }
  return SFK_OK;
}

sfk_status check_status_word(int* dev_status, cudaStream_t st) {
  int h = 0;
  CK(cudaMemcpyAsync(&h, dev_status, sizeof(int), cudaMemcpyDeviceToHost, st));
  CK(cudaStreamSynchronize(st));
  return status_result(dev_status, h);
}

}  // namespace

// ---------------------------------------------------------------------------
// engine
// ---------------------------------------------------------------------------
struct LayerW {
  uint8_t* qkv = nullptr;   // [Hq*hd + 2*Hkv*hd] rows of K = d (device layout)
  uint8_t* wo = nullptr;    // [d] rows of K = Hq*hd
  float* attn_norm = nullptr;
  float* ffn_norm = nullptr;
  float* router = nullptr;  // [E][d]
  uint8_t* gate = nullptr;  // [E][F] rows of K = d
  uint8_t* up = nullptr;
  uint8_t* down = nullptr;  // [E][d] rows of K = F
};

struct sfk_engine {
  int device = 0;
  sfk_hparams hp{};
  int hd = 0, nq = 0, nk = 0, nqkv = 0;
  cudaStream_t stream = nullptr;
  int sm_count = 148;
  std::vector<void*> allocs;
  // weights
  uint8_t* tok_embd = nullptr;  // GGUF layout
  float* out_norm = nullptr;
  uint8_t* output = nullptr;
  std::vector<LayerW> L;
  uint64_t weight_bytes = 0, kv_bytes = 0, scratch_bytes = 0;
  // KV
  void* k_pool = nullptr;
  void* v_pool = nullptr;
  int64_t kv_layer_elems = 0;
  int* page_table = nullptr;  // [max_batch][max_pages]
  int max_pages = 0;
  int n_pages = 0;  // HBM pages per layer
  // KV window (hp.kv_window): each sequence's last `pages` pages form a ring
  // of HBM pages; older pages live in a pinned host cold store and are staged
  // back into one layer's worth of HBM for each layer's attention
  struct Window {
    bool on = false;
    int pages = 0;                              // ring pages per sequence
    int64_t page_bytes = 0;                     // one page of K (or V) of one layer
    void *k_stage[2] = {}, *v_stage[2] = {};     // [max_batch][max_pages] pages; layer l uses l & 1
    cudaStream_t copy = nullptr;                 // decode steps stage cold pages here, a layer ahead
    cudaEvent_t start = nullptr, staged[2] = {}, used[2] = {};
    uint8_t *k_cold = nullptr, *v_cold = nullptr; // pinned [n_layer][max_batch][max_pages] pages
    std::vector<int> cold;                      // per sequence: logical pages 0 .. cold-1 are cold
    std::vector<int> ring;                      // [max_batch][pages] HBM page of each ring slot
    uint64_t evicted = 0, staged_bytes = 0;
  } win;
  std::vector<int> step_pos;  // host: the position of each sequence in the step being launched
  std::vector<int> pt0;       // the page table after a reset
  // step buffers
  float *x = nullptr, *ffn_inp = nullptr, *q = nullptr, *attn_out = nullptr, *h = nullptr, *logits = nullptr;
  float *router_logits = nullptr;
  float* rope = nullptr;  // [n_ctx][hd/2] (cos, sin)
  uint8_t *xq_ffn = nullptr, *hq = nullptr;
  Route* route = nullptr;
  int *router_counter = nullptr, *grp_counter = nullptr;
  unsigned long long* argmax_key = nullptr;  // [B] keys, then the status word: one read-back
  int *tok_in = nullptr, *pos_in = nullptr, *pos_state = nullptr, *pos_cur = nullptr, *tok_hist = nullptr;
  int* status = nullptr;  // right after argmax_key[B]
  // the gate/up kernel can route in its prologue (no router kernel); steps of
  // at most fused_route_max_b tokens do, larger steps run the router kernel
  bool fused_route = false;
  int fused_route_max_b = 0;
  // expert parallelism: this rank holds experts [e0, e0 + e_loc)
  int ep_size = 1, ep_rank = 0, e_loc = 0, e0 = 0;
  // head parallelism (with expert parallelism when the heads divide): this
  // rank computes query heads [q0, q0 + hq_loc) and kv heads [kv0, kv0 + hkv_loc)
  bool head_par = false;
  int hq_loc = 0, hkv_loc = 0, q0 = 0, kv0 = 0;
  float* ep_buf = nullptr;      // [2][B][d] partial outputs (layer parity) | flags [MAXR] ints
  unsigned* ep_flags = nullptr;
  unsigned* ep_step = nullptr;
  const float* ep_parts[MAXR] = {};
  unsigned* ep_peer_flags[MAXR] = {};
  // vocabulary-sharded lm_head (expert parallelism, steps that return no
  // logits): this rank scores rows [v0, v0 + v_loc) and the argmax keys are
  // exchanged (ep_argmax_kernel) through the tail of ep_buf
  bool head_shard = false;  // the engine may shard the head
  bool shard_now = false;   // the step being captured / launched does
  int v0 = 0, v_loc = 0;
  unsigned* ep_head_flags = nullptr;
  unsigned long long* ep_keys = nullptr;
  unsigned* ep_peer_head_flags[MAXR] = {};
  const unsigned long long* ep_peer_keys[MAXR] = {};
  std::vector<void*> ep_opened;  // peer buffers opened through IPC
  bool ep_connected = false;
  int attn_cluster = 8;
  int attn_max_chunk = 0;
  // pinned staging: tokens and positions side by side (tok_in / pos_in are
  // side by side on the device too: one upload), keys then status (one
  // read-back), the logits of a host-buffer step
  int* h_tok = nullptr;
  int* h_pos = nullptr;  // h_tok + B
  int* h_hist = nullptr;
  unsigned long long* h_keys = nullptr;
  int* h_status = nullptr;  // right after h_keys[B]
  float* h_logits = nullptr;
  // persistent step kernel (sfk_mega.cu): one cooperative launch per step
  // when the shape fits its plan; otherwise the launch chain below
  bool mega = false;
  MegaLayer* d_layers = nullptr;  // per-layer weight pointers on the device
  float *att_y = nullptr, *att_cmax = nullptr, *att_stat = nullptr;
  double* att_opart = nullptr;
  int* att_cnt = nullptr;
  unsigned* att_ready = nullptr;
  unsigned* gbar = nullptr;
  int att_nc = 0;
  bool last_step_mega = false;
  // graphs: key = b * 2 + greedy
  std::map<int, cudaGraphExec_t> graphs;
  uint64_t steps = 0;
  int kernels_per_step = 0;
  int last_b = 0;
  std::vector<int> seq_pos;  // host mirror of the next position per sequence
  // batched prompt prefill (sfk_prefill): buffers for a chunk of `cap` prompt
  // tokens, allocated at the first prefill
  struct Prefill {
    int cap = 0;  // prompt tokens per chunk
    int mt = 0;   // 64-row tiles of the routed pairs (expert-grouped, padded)
    int *tok = nullptr, *pos = nullptr, *pt = nullptr;
    float *x = nullptr, *ffn = nullptr, *xn = nullptr, *qkv = nullptr, *q = nullptr, *att = nullptr;
    float *h = nullptr, *yd = nullptr, *w = nullptr;
    float* score = nullptr;     // attention score rows (pf_attn scratch)
    size_t score_bytes = 0;
    uint8_t *act = nullptr, *xqd = nullptr;
    uint8_t* act_dn = nullptr;  // bounded tier only: the down GEMM's activation slabs
    int *ids = nullptr, *pos_of_pair = nullptr, *rows_tok = nullptr, *rows_self = nullptr, *tile_expert = nullptr;
  } pf;
  // generate loop: the sampler's probabilities [V] and its token
  float* sample_p = nullptr;
  int* sample_tok = nullptr;
  // bounded expert tier (hp.expert_slots): every bundle gate|up|down in the
  // device row layout in pinned host memory, a pool of HBM slots holding the
  // working set, and per layer the slot of each routed expert
  struct Tier {
    bool on = false;
    uint32_t n_slots = 0;
    int64_t slot_bytes = 0, off_up = 0, off_down = 0;  // one slot: gate at 0, up, down
    uint8_t* pool = nullptr;   // [n_slots][slot_bytes] HBM
    uint8_t* host = nullptr;   // [n_layer][n_expert][slot_bytes] pinned
    int* d_map = nullptr;      // [n_layer][n_expert] slot of each routed expert (device)
    int* h_map = nullptr;      // pinned mirror
    Route* h_route = nullptr;  // pinned read-back of one layer's routing
    int* d_tile = nullptr;     // prefill: the slot of each expert tile of a pass (-1: not in it)
    int* h_tile = nullptr;     // pinned: tile experts read back, then the pass's tile slots
    int* h_ids = nullptr;      // pinned: a prefill chunk's routed ids
    cudaStream_t copy = nullptr;
    cudaEvent_t copied = nullptr;
    std::unique_ptr<SlotPool> sp;
    std::unique_ptr<ExpertPredictor> pred;
    int prefetch = 1;  // 0 off; 1 only into free slots; 2 may evict within the predicted layer
    uint64_t h2d = 0, warmed = 0, used = 0, tokens = 0;
    std::set<uint64_t> warmed_now;  // (layer, expert) prefetched during this step
  } tier;

  template <typename T>
  sfk_status alloc(T** p, size_t bytes, uint64_t* acct) {
    void* v = nullptr;
    cudaError_t e = cudaMalloc(&v, bytes);
    if (e != cudaSuccess)
      return fail(SFK_ERR_OUT_OF_MEMORY, "cudaMalloc(%zu) failed: %s", bytes, cudaGetErrorString(e));
    allocs.push_back(v);
    *p = reinterpret_cast<T*>(v);
    if (acct) *acct += bytes;
    return SFK_OK;
  }
};

namespace {

int64_t tensor_rows(const sfk_engine* e, int tid) {
  const sfk_hparams& hp = e->hp;
  switch (tid) {
    case SFK_T_TOK_EMBD: case SFK_T_OUTPUT: return hp.n_vocab;
    case SFK_T_ATTN_Q: return e->nq;
    case SFK_T_ATTN_K: case SFK_T_ATTN_V: return e->nk;
    case SFK_T_ATTN_OUT: return hp.n_embd;
    case SFK_T_FFN_GATE_INP: return hp.n_expert;
    case SFK_T_FFN_GATE_EXPS: case SFK_T_FFN_UP_EXPS: return (int64_t)e->e_loc * hp.n_ff;  // local experts
    case SFK_T_FFN_DOWN_EXPS: return (int64_t)e->e_loc * hp.n_embd;
    default: return 1;
  }
}
int64_t tensor_cols(const sfk_engine* e, int tid) {
  const sfk_hparams& hp = e->hp;
  switch (tid) {
    case SFK_T_ATTN_OUT: return e->nq;
    case SFK_T_FFN_DOWN_EXPS: return hp.n_ff;
    default: return hp.n_embd;
  }
}
int tensor_type(const sfk_engine* e, int tid) {
  const sfk_hparams& hp = e->hp;
  switch (tid) {
    case SFK_T_TOK_EMBD: return hp.type_embd;
    case SFK_T_OUTPUT: return hp.type_output;
    case SFK_T_ATTN_Q: case SFK_T_ATTN_K: case SFK_T_ATTN_V: case SFK_T_ATTN_OUT: return hp.type_attn;
    case SFK_T_FFN_GATE_EXPS: case SFK_T_FFN_UP_EXPS: return hp.type_ffn_gu;
    case SFK_T_FFN_DOWN_EXPS: return hp.type_ffn_down;
    default: return T_F32;
  }
}
bool layered(int tid) { return tid >= SFK_T_ATTN_NORM && tid <= SFK_T_FFN_DOWN_EXPS; }

// device destination of a tensor: base pointer (device layout) for matrices,
// plain pointer for F32 / GGUF-layout tensors
uint8_t* tensor_dst(sfk_engine* e, int tid, int layer) {
  const int64_t rs = dev_row_bytes(e->hp.type_attn, e->hp.n_embd);
  switch (tid) {
    case SFK_T_TOK_EMBD: return e->tok_embd;
    case SFK_T_OUTPUT_NORM: return reinterpret_cast<uint8_t*>(e->out_norm);
    case SFK_T_OUTPUT: return e->output;
    case SFK_T_ATTN_NORM: return reinterpret_cast<uint8_t*>(e->L[layer].attn_norm);
    case SFK_T_ATTN_Q: return e->L[layer].qkv;
    case SFK_T_ATTN_K: return e->L[layer].qkv + (int64_t)e->nq * rs;
    case SFK_T_ATTN_V: return e->L[layer].qkv + (int64_t)(e->nq + e->nk) * rs;
    case SFK_T_ATTN_OUT: return e->L[layer].wo;
    case SFK_T_FFN_NORM: return reinterpret_cast<uint8_t*>(e->L[layer].ffn_norm);
    case SFK_T_FFN_GATE_INP: return reinterpret_cast<uint8_t*>(e->L[layer].router);
    case SFK_T_FFN_GATE_EXPS: return e->L[layer].gate;
    case SFK_T_FFN_UP_EXPS: return e->L[layer].up;
    case SFK_T_FFN_DOWN_EXPS: return e->L[layer].down;
    default: return nullptr;
  }
}
// stored in the interleaved device layout (vs verbatim)
bool relaid(int tid) {
  return tid == SFK_T_OUTPUT || tid == SFK_T_ATTN_Q || tid == SFK_T_ATTN_K || tid == SFK_T_ATTN_V ||
         tid == SFK_T_ATTN_OUT || tid == SFK_T_FFN_GATE_EXPS || tid == SFK_T_FFN_UP_EXPS ||
         tid == SFK_T_FFN_DOWN_EXPS;
}

uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}
// per-tensor seed (same function as the CPU fixture generator)
uint64_t tensor_seed(uint64_t seed, int tid, int layer) {
  return splitmix64(seed * 0x100000001B3ull + (uint64_t)(tid + 1) * 0x9E3779B1ull + (uint64_t)(layer + 1) * 0x85EBCA77ull);
}

// ---- the step launch chain -------------------------------------------------
enum KernelClass { K_EMBED = 0, K_QKV, K_ATTN, K_OPROJ, K_ROUTER, K_GATEUP, K_DOWN, K_LMHEAD, K_NCLASS };

// The device status word after a step; on a device error the counters that
// CTAs hand between launches (routing arrivals, SwiGLU group counters) may be
// left mid-count, so they are cleared before the engine is used again.
void reset_counters(sfk_engine* e) {
  cudaMemset(e->router_counter, 0, 2 * sizeof(int));
  cudaMemset(e->grp_counter, 0, sizeof(int) * (e->hp.n_ff / 256));
  if (e->mega) {  // a failed persistent step may leave its barrier and attention words mid-count
    cudaMemset(e->gbar, 0, 2 * sizeof(unsigned));
    cudaMemset(e->att_cnt, 0, sizeof(int) * 2 * e->hp.max_batch * e->hkv_loc);
    cudaMemset(e->att_ready, 0, sizeof(unsigned) * e->hp.max_batch * e->hkv_loc);
  }
}

sfk_status engine_check(sfk_engine* e) {
  sfk_status s = check_status_word(e->status, e->stream);
  if (s != SFK_OK) reset_counters(e);
  return s;
}

KvView kv_view(const sfk_engine* e, int l) {
  const sfk_hparams& hp = e->hp;
  KvView kv{};
  kv.page_table = e->page_table;
  kv.max_pages = e->max_pages;
  kv.n_pages = e->n_pages;
  kv.n_head_kv = e->hkv_loc;
  kv.head_dim = e->hd;
  kv.f16 = hp.kv_type == SFK_KV_F16 ? 1 : 0;
  const size_t kv_elem = kv.f16 ? 2 : 4;
  kv.k = static_cast<uint8_t*>(e->k_pool) + (int64_t)l * e->kv_layer_elems * kv_elem;
  kv.v = static_cast<uint8_t*>(e->v_pool) + (int64_t)l * e->kv_layer_elems * kv_elem;
  if (e->win.on) {  // ids from n_pages up: the staged cold pages (page_table: n_pages + seq * max_pages + page)
    kv.n_hot = e->n_pages;
    kv.n_pages = e->n_pages + hp.max_batch * e->max_pages;
    kv.k2 = e->win.k_stage[l & 1];
    kv.v2 = e->win.v_stage[l & 1];
  }
  return kv;
}

// Whether a step of b tokens routes inside its gate/up kernel.  The fused
// prologue routes the step's tokens one after another in every CTA: cheapest
// for one or two tokens, while from four tokens on the router kernel, which
// routes them in parallel, and a plain gate/up prologue are faster (Mixtral
// shape, b = 8: 637 vs 605 tok/s; b = 16: 637 vs 495).
bool route_fused(const sfk_engine* e, int b) { return e->fused_route && b <= e->fused_route_max_b; }

StreamParams gateup_params(const sfk_engine* e, int l, int b) {
  const sfk_hparams& hp = e->hp;
  const int d = hp.n_embd, F = hp.n_ff, k = hp.n_expert_used;
  const LayerW& W = e->L[l];
  StreamParams p{};
  p.w0 = W.gate;
  p.w1 = W.up;
  p.rowstride = dev_row_bytes(hp.type_ffn_gu, d);
  p.expert_stride = (int64_t)F * p.rowstride;
  p.rows = F;
  p.K = d;
  p.wtype = hp.type_ffn_gu;
  p.nmat = 2;
  p.act_type = act_for(hp.type_ffn_gu);
  p.row_align = 1;
  p.b = b; p.k = k; p.n_pairs = b * k; p.n_vec = b;
  p.route = e->route;
  if (e->ep_size > 1) {
    p.ep_e0 = e->e0;
    p.ep_eloc = e->e_loc;
  }
  if (e->tier.on) {  // the routed experts' slots of the bounded pool
    p.w0 = e->tier.pool;
    p.w1 = e->tier.pool + e->tier.off_up;
    p.expert_stride = e->tier.slot_bytes;
    p.slot_map = e->tier.d_map + (size_t)l * hp.n_expert;
    p.n_map_slots = (int)e->tier.n_slots;
  }
  if (route_fused(e, b)) {
    p.pro = PRO_ROUTE;  // ffn_norm + quantize + router + top-k in the prologue
    p.x = e->ffn_inp;
    p.norm_w = W.ffn_norm;
    p.eps = hp.rms_eps;
    p.w_r = W.router;
    p.n_expert = hp.n_expert;
    p.logits = e->router_logits;
    p.rsync = e->router_counter;
  } else {
    p.pro = PRO_LOAD;
    p.qact = e->xq_ffn;
    p.qact_stride = qact_bytes(d);
  }
  p.xq_by_pair = 0;
  p.epi = EPI_GATEUP;
  p.h = e->h;
  p.hq = e->hq;
  p.grp_counter = e->grp_counter;
  p.h_act_type = act_for(hp.type_ffn_down);
  p.status = e->status;
  return p;
}

// Kernels whose first weight fill goes out before their wait on the previous
// kernel (bit 0: output projection, 1: QKV, 2: lm_head); SFK_EARLY_FILL
// overrides the default.
int early_fill_mask() {
  static const int m = [] {
    const char* v = getenv("SFK_EARLY_FILL");
    return v ? atoi(v) : 3;
  }();
  return m;
}

// Launch one kernel of the step: class `c` of layer `l` for b sequences.
sfk_status launch_one(sfk_engine* e, int c, int l, int b, bool greedy, bool pdl) {
  const sfk_hparams& hp = e->hp;
  cudaStream_t st = e->stream;
  const int d = hp.n_embd, F = hp.n_ff, k = hp.n_expert_used;
  int grid = 0;
  sfk_status s = SFK_OK;
  switch (c) {
    case K_EMBED: {  // ggml_get_rows(token_embd) (engine.cpp:2708-2723)
      EmbedParams ep{};
      ep.tok_embd = e->tok_embd;
      ep.type = hp.type_embd;
      ep.d = d;
      ep.V = hp.n_vocab;
      ep.b = b;
      ep.tok_in = e->tok_in;
      ep.argmax_key = e->argmax_key;
      ep.greedy = greedy ? 1 : 0;
      ep.tok_hist = e->tok_hist;
      ep.pos_in = greedy ? nullptr : e->pos_in;
      ep.pos_state = e->pos_state;
      ep.pos_cur = e->pos_cur;
      ep.x = e->x;
      ep.ep_step = e->ep_step;
      ep.status = e->status;
      CK(launch_embed(ep, st, pdl));
      return SFK_OK;
    }
    case K_QKV: {  // attn_norm + Q/K/V + RoPE + KV append (engine.cpp:1878-1897,1646-1656)
      const LayerW& W = e->L[l];
      StreamParams p{};
      p.w0 = W.qkv;
      p.rowstride = dev_row_bytes(hp.type_attn, d);
      p.rows = e->nqkv;
      p.K = d;
      p.wtype = hp.type_attn;
      p.nmat = 1;
      p.act_type = act_for(hp.type_attn);
      p.row_align = 2;
      p.b = b; p.k = 1; p.n_pairs = b; p.n_vec = b;
      p.pro = PRO_QUANT;
      p.x = e->x;
      p.norm_w = W.attn_norm;
      p.eps = hp.rms_eps;
      p.epi = EPI_QKV;
      p.early_fill = (early_fill_mask() >> 1) & 1;
      p.y = e->q;
      p.kv = kv_view(e, l);
      p.n_head = e->hq_loc;
      p.rope = e->rope;
      p.pos = e->pos_cur;
      if (l == 0) {  // the embedding kernel has read the argmax keys by now
        p.clear_keys = e->argmax_key;
        p.clear_n = b;
      }
      p.status = e->status;
      if ((s = plan_stream(p, e->sm_count, &grid))) return s;
      CK(launch_stream(p, grid, st, pdl));
      return SFK_OK;
    }
    case K_ATTN: {  // attention over the paged KV (engine.cpp:1751-1761)
      AttnParams a{};
      a.q = e->q;
      a.kv = kv_view(e, l);
      a.pos = e->pos_cur;
      a.b = b;
      a.n_head = e->hq_loc;
      a.cluster = e->attn_cluster;
      a.max_chunk = e->attn_max_chunk;
      a.out = e->attn_out;
      a.status = e->status;
      CK(launch_attn(a, st, pdl));
      return SFK_OK;
    }
    case K_OPROJ: {  // O projection + residual (engine.cpp:1905-1906)
      StreamParams p{};
      p.w0 = e->L[l].wo;
      p.rowstride = dev_row_bytes(hp.type_attn, e->nq);
      p.rows = d;
      p.K = e->nq;
      p.wtype = hp.type_attn;
      p.nmat = 1;
      p.act_type = act_for(hp.type_attn);
      p.row_align = 1;
      p.b = b; p.k = 1; p.n_pairs = b; p.n_vec = b;
      p.pro = PRO_QUANT;
      p.x = e->attn_out;
      p.epi = EPI_RESID;
      p.early_fill = early_fill_mask() & 1;
      p.y = e->ffn_inp;
      p.res = e->x;
      p.y_stride = d;
      if (e->head_par) {
        // this rank's heads' share of the projection (its columns) into the
        // exchange slot; the residual is added once, by rank 0
        p.y = e->ep_buf + (size_t)((l & 1) * 2 + 0) * e->hp.max_batch * d;
        p.res = e->ep_rank == 0 ? e->x : nullptr;
      }
      p.status = e->status;
      if ((s = plan_stream(p, e->sm_count, &grid))) return s;
      CK(launch_stream(p, grid, st, pdl));
      return SFK_OK;
    }
    case K_ROUTER: {  // ffn_norm + router + top-k (engine.cpp:1909-1924)
      if (route_fused(e, b)) return SFK_OK;  // done inside the gate/up kernel
      const LayerW& W = e->L[l];
      RouterParams r{};
      r.x = e->ffn_inp;
      r.norm_w = W.ffn_norm;
      r.w_r = W.router;
      r.b = b; r.d = d; r.E = hp.n_expert; r.k = k;
      r.eps = hp.rms_eps;
      r.act_type = act_for(hp.type_ffn_gu);
      r.xq = e->xq_ffn;
      r.route = e->route;
      r.logits = e->router_logits;
      r.counter = e->router_counter;
      if (e->ep_size > 1) {
        r.ep_e0 = e->e0;
        r.ep_eloc = e->e_loc;
      }
      r.status = e->status;
      CK(launch_router(r, st, pdl));
      return SFK_OK;
    }
    case K_GATEUP: {  // (routing +) routed gate/up + SwiGLU (engine.cpp:1909-1924,1967-1969)
      StreamParams p = gateup_params(e, l, b);
      if ((s = plan_stream(p, e->sm_count, &grid))) return s;
      CK(launch_stream(p, grid, st, pdl));
      return SFK_OK;
    }
    case K_DOWN: {  // routed down + weighted combine + residual (engine.cpp:1970-1986)
      StreamParams p{};
      p.w0 = e->L[l].down;
      p.rowstride = dev_row_bytes(hp.type_ffn_down, F);
      p.expert_stride = (int64_t)d * p.rowstride;
      p.rows = d;
      p.K = F;
      p.wtype = hp.type_ffn_down;
      p.nmat = 1;
      p.act_type = act_for(hp.type_ffn_down);
      p.row_align = 1;
      p.b = b; p.k = k; p.n_pairs = b * k; p.n_vec = b * k;
      p.route = e->route;
      p.pro = PRO_LOAD;
      p.qact = e->hq;
      p.qact_stride = qact_bytes(F);
      p.xq_by_pair = 1;
      p.epi = EPI_DOWN;
      p.y = e->x;
      p.res = e->ffn_inp;
      if (e->ep_size > 1) {
        // this rank's experts into its exchange buffer (layer parity); the
        // residual is added once, by rank 0; the combine writes x
        p.ep_e0 = e->e0;
        p.ep_eloc = e->e_loc;
        p.y = e->ep_buf + (size_t)((l & 1) * 2 + 1) * e->hp.max_batch * d;
        p.res = e->ep_rank == 0 ? e->ffn_inp : nullptr;
      }
      p.y_stride = d;
      if (e->tier.on) {
        p.w0 = e->tier.pool + e->tier.off_down;
        p.expert_stride = e->tier.slot_bytes;
        p.slot_map = e->tier.d_map + (size_t)l * hp.n_expert;
        p.n_map_slots = (int)e->tier.n_slots;
      }
      p.status = e->status;
      if ((s = plan_stream(p, e->sm_count, &grid))) return s;
      CK(launch_stream(p, grid, st, pdl));
      return SFK_OK;
    }
    case K_LMHEAD: {  // output_norm + lm_head + argmax (engine.cpp:2988-3006, ggml_model.cpp:284-292)
      StreamParams p{};
      p.w0 = e->output;
      p.rowstride = dev_row_bytes(hp.type_output, d);
      p.rows = hp.n_vocab;
      p.K = d;
      p.wtype = hp.type_output;
      p.nmat = 1;
      p.act_type = act_for(hp.type_output);
      p.row_align = 1;
      p.b = b; p.k = 1; p.n_pairs = b; p.n_vec = b;
      p.pro = PRO_QUANT;
      p.x = e->x;
      p.norm_w = e->out_norm;
      p.eps = hp.rms_eps;
      p.epi = EPI_LMHEAD;
      p.early_fill = (early_fill_mask() >> 2) & 1;
      p.y = e->logits;
      p.y_stride = hp.n_vocab;
      p.argmax_key = e->argmax_key;
      p.store_logits = 1;
      if (e->shard_now) {  // this rank's vocabulary slice; the keys carry global row ids
        p.w0 = e->output + (int64_t)e->v0 * p.rowstride;
        p.rows = e->v_loc;
        p.y = e->logits + e->v0;
        p.argmax_base = e->v0;
      }
      p.status = e->status;
      if ((s = plan_stream(p, e->sm_count, &grid))) return s;
      CK(launch_stream(p, grid, st, pdl));
      if (e->shard_now) {  // the first maximum over every rank's slice
        EpHeadParams h{};
        h.key = e->argmax_key;
        h.own_keys = e->ep_keys;
        for (int r = 0; r < e->ep_size; ++r) {
          h.peer_keys[r] = e->ep_peer_keys[r];
          h.peer_flags[r] = e->ep_peer_head_flags[r];
        }
        h.flags = e->ep_head_flags;
        h.n_ranks = e->ep_size;
        h.rank = e->ep_rank;
        h.b = b;
        h.ep_step = e->ep_step;
        h.status = e->status;
        CK(launch_ep_argmax(h, st, true));
      }
      return SFK_OK;
    }
    default: return fail(SFK_ERR_INVALID_ARGUMENT, "kernel class %d", c);
  }
}

// Combine of a layer stage across the expert-parallel ranks (peer memory).
sfk_status launch_combine(sfk_engine* e, int l, int stage, int b, float* dst) {
  EpParams q{};
  for (int r = 0; r < e->ep_size; ++r) {
    q.parts[r] = e->ep_parts[r];
    q.peer_flags[r] = e->ep_peer_flags[r];
  }
  q.flags = e->ep_flags;
  q.n_ranks = e->ep_size;
  q.rank = e->ep_rank;
  q.layer = l;
  q.n_layer = e->hp.n_layer;
  q.stage = stage;
  q.ep_step = e->ep_step;
  q.half = e->hp.max_batch * e->hp.n_embd;
  q.n = b * e->hp.n_embd;
  q.x = dst;
  q.status = e->status;
  CK(launch_ep_combine(q, e->stream, true));
  return SFK_OK;
}

// Plan of the persistent step kernel for b sequences: rows per CTA, ring
// slot size, tile rows per phase, shared-memory layout.  False when the shape
// does not fit it (the step then runs as the launch chain).
constexpr int MEGA_CH = 64;  // attention positions per work item

bool mega_params(const sfk_engine* e, int b, bool greedy, MegaParams* out, int* grid_out) {
  if (!e->mega || b < 1 || b > e->hp.max_batch) return false;
  const sfk_hparams& hp = e->hp;
  const int d = hp.n_embd, F = hp.n_ff, E = hp.n_expert, k = hp.n_expert_used, V = hp.n_vocab;
  const int hd = e->hd, gqa = hp.n_head / hp.n_head_kv;
  if (b * k > 32) return false;
  const int grid = e->sm_count;
  MegaParams p{};
  p.layers = e->d_layers;
  p.n_layer = hp.n_layer;
  p.d = d; p.nq = e->nq; p.nk = e->nk; p.nqkv = e->nqkv; p.hd = hd; p.n_head = hp.n_head; p.n_head_kv = hp.n_head_kv;
  p.gqa = gqa; p.F = F; p.E = E; p.k = k; p.V = V; p.b = b; p.n_ctx = hp.n_ctx;
  p.eps = hp.rms_eps;
  p.att_scale = 1.0f / sqrtf((float)hd);
  p.t_embd = hp.type_embd; p.t_attn = hp.type_attn; p.t_gu = hp.type_ffn_gu; p.t_down = hp.type_ffn_down;
  p.t_out = hp.type_output;
  p.a_attn = act_for(hp.type_attn); p.a_gu = act_for(hp.type_ffn_gu); p.a_down = act_for(hp.type_ffn_down);
  p.a_out = act_for(hp.type_output);
  p.rs_attn = dev_row_bytes(hp.type_attn, d);
  p.rs_o = dev_row_bytes(hp.type_attn, e->nq);
  p.rs_gu = dev_row_bytes(hp.type_ffn_gu, d);
  p.rs_down = dev_row_bytes(hp.type_ffn_down, F);
  p.rs_out = dev_row_bytes(hp.type_output, d);
  auto rpc = [&](int rows, int align) {
    int r = (rows + grid - 1) / grid;
    return (r + align - 1) / align * align;
  };
  p.rpc_qkv = rpc(e->nqkv, 2);
  p.rpc_o = rpc(d, 1);
  p.rpc_gu = rpc(F, 1);
  p.rpc_down = rpc(d, 1);
  p.rpc_out = rpc(V, 1);
  // router rows: pieces of d / parts columns (a multiple of 128); the pieces
  // are dealt to the warps like row blocks, one piece per ring slot.  At
  // least one piece per warp when the columns allow it; pieces are cut
  // further below until one fits a slot (checked once the slot is known).
  int parts = 1;
  while (E * parts < MEGA_NC && d % (parts * 2 * 128) == 0) parts *= 2;
  if (d % (parts * 128)) return false;
  // shared memory
  auto al = [](int64_t v, int a) { return (v + a - 1) / a * a; };
  const int kvb = hp.kv_type == SFK_KV_F16 ? 2 : 4;
  const int64_t qd = qact_bytes(d), qq = qact_bytes(e->nq), qf = qact_bytes(F);
  int64_t xq = std::max<int64_t>(b * qd, b * qq);
  xq = std::max<int64_t>(xq, (int64_t)b * k * qf);
  xq = std::max<int64_t>(xq, al(b * qd, 16) + (int64_t)b * d * 4 + (int64_t)b * E * 4);
  xq = std::max<int64_t>(xq, 2ll * MEGA_CH * hd * kvb);
  xq = al(xq, 128);
  int64_t acc = std::max<int64_t>((int64_t)p.rpc_qkv * b, (int64_t)p.rpc_o * b);
  acc = std::max<int64_t>(acc, (int64_t)p.rpc_gu * b * k * 2);
  acc = std::max<int64_t>(acc, (int64_t)p.rpc_down * b * k);
  acc = std::max<int64_t>(acc, (int64_t)p.rpc_out * b);
  acc = al(acc * 4, 16);
  const int64_t route = al(2 * sizeof(Route), 16);  // double-buffered by layer parity
  const int64_t red = MEGA_RED * 8;
  const int64_t probs = al((int64_t)b * E * (d / 128) * 8, 16);  // partial logits, any piece count
  const int64_t att = al((int64_t)gqa * hd * 4 + 2ll * gqa * MEGA_CH * 4 + gqa * 8, 16);
  const int64_t misc = al((2 * MAXB + 4) * 4, 16);  // tokens | positions | routed layer | flag | phase limit
  const int64_t bars = al(2 * MEGA_NWS * MEGA_MAXS * 8 + 3 * 8, 128);  // full | empty slot barriers, prologue barriers
  const int64_t layers = al((int64_t)hp.n_layer * sizeof(MegaLayer), 16);
  const int64_t fixed = bars + xq + acc + route + red + probs + att + misc + layers;
  // ring slots per warp, a power of two (SFK_MEGA_STAGES / SFK_MEGA_SLOT
  // override the ring shape)
  int S = 1;
  if (const char* v = getenv("SFK_MEGA_STAGES")) S = atoi(v);
  if (S != 1 && S != 2 && S != 4) return false;
  p.S_log2 = S == 1 ? 0 : (S == 2 ? 1 : 2);
  p.lookahead = 1 << 20;  // unlimited: rings run ahead across every phase boundary
  if (const char* v = getenv("SFK_MEGA_LOOKAHEAD")) p.lookahead = atoi(v);
  int64_t slot = (SMEM_LIMIT - fixed) / (MEGA_NC * S);
  slot = std::min<int64_t>(slot, 32 * 1024) / 128 * 128;
  if (const char* v = getenv("SFK_MEGA_SLOT")) slot = std::min<int64_t>(slot, atoi(v) / 128 * 128);
  if (slot <= 0) return false;
  while ((int64_t)(d / parts) * 4 > slot && d % (parts * 2 * 128) == 0) parts *= 2;
  if ((int64_t)(d / parts) * 4 > slot) return false;
  p.rt_parts = parts;
  // Tiles per weight phase: R whole rows (at most four (row, matrix) unit dots
  // of a one-group row, or eight (row, matrix, group) values), or, for a row
  // longer than a slot (one matrix only), column-group ranges of one row
  auto plan_tiles = [&](int k, int64_t rs, int nmat, int wt, int K) {
    const int G = n_groups(K);
    // (row, matrix) values per tile: up to four for one-group rows, two for
    // longer rows, and at most eight (row, matrix, group) values
    const int rmax = G == 1 ? 4 / nmat : std::min(2 / nmat, 8 / (nmat * G));
    p.R[k] = (int)std::min<int64_t>(std::max(rmax, 1), slot / (nmat * rs));
    p.H[k] = 1;
    p.gpp[k] = 8;
    if (p.R[k] >= 1 && rmax >= 1) return true;
    if (nmat != 1) return false;
    const int64_t gb = group_bytes(wt, GROUP_UNITS);  // a full group; the last may be shorter
    const int gpp = (int)std::min<int64_t>(8, slot / gb);
    if (gpp < 1) return false;
    p.R[k] = 1;
    p.gpp[k] = gpp;
    p.H[k] = (G + gpp - 1) / gpp;
    return true;
  };
  if (!plan_tiles(MEGA_PK_QKV, p.rs_attn, 1, hp.type_attn, d) || !plan_tiles(MEGA_PK_O, p.rs_o, 1, hp.type_attn, e->nq) ||
      !plan_tiles(MEGA_PK_GU, p.rs_gu, 2, hp.type_ffn_gu, d) ||
      !plan_tiles(MEGA_PK_DN, p.rs_down, 1, hp.type_ffn_down, F) ||
      !plan_tiles(MEGA_PK_OUT, p.rs_out, 1, hp.type_output, d))
    return false;
  p.S = S;
  p.slot = (int)slot;
  p.att_ch = MEGA_CH;
  p.att_nc = e->att_nc;
  p.off_ring = (int)bars;
  p.off_xq = p.off_ring + (int)(MEGA_NC * S * slot);
  p.off_acc = p.off_xq + (int)xq;
  p.off_route = p.off_acc + (int)acc;
  p.off_red = p.off_route + (int)route;
  p.off_probs = p.off_red + (int)red;
  p.off_att = p.off_probs + (int)probs;
  p.off_misc = p.off_att + (int)att;
  p.off_layers = p.off_misc + (int)misc;
  p.smem = p.off_layers + (int)layers;
  p.xq_bytes = (int)xq;
  if (p.smem > SMEM_LIMIT) return false;
  p.tok_embd = e->tok_embd;
  p.out_norm = e->out_norm;
  p.output = e->output;
  p.tok_in = e->tok_in;
  p.pos_in = greedy ? nullptr : e->pos_in;
  p.greedy = greedy ? 1 : 0;
  p.pos_state = e->pos_state;
  p.pos_cur = e->pos_cur;
  p.tok_hist = e->tok_hist;
  p.argmax_key = e->argmax_key;
  p.k_pool = e->k_pool;
  p.v_pool = e->v_pool;
  p.kv_layer_bytes = e->kv_layer_elems * kvb;
  p.page_table = e->page_table;
  p.max_pages = e->max_pages;
  p.n_pages = e->n_pages;
  p.kv_f16 = hp.kv_type == SFK_KV_F16 ? 1 : 0;
  p.rope = e->rope;
  p.x = e->x;
  p.ffn_inp = e->ffn_inp;
  p.q = e->q;
  p.attn_out = e->attn_out;
  p.h = e->h;
  p.hq = e->hq;
  p.logits = e->logits;
  p.grp_counter = e->grp_counter;
  p.route_out = e->route;
  p.att_y = e->att_y;
  p.att_cmax = e->att_cmax;
  p.att_stat = e->att_stat;
  p.att_opart = e->att_opart;
  p.att_cnt = e->att_cnt;
  p.att_ready = e->att_ready;
  p.gbar = e->gbar;
  p.status = e->status;
  p.store_logits = 1;
  *out = p;
  *grid_out = grid;
  return true;
}

sfk_status enqueue_step(sfk_engine* e, int b, bool greedy) {
  MegaParams mp;
  int mgrid = 0;
  if (mega_params(e, b, greedy, &mp, &mgrid)) {
    CK(launch_mega(mp, mgrid, e->stream));
    e->kernels_per_step = 1;
    return SFK_OK;
  }
  int nk = 0;
  sfk_status s = launch_one(e, K_EMBED, 0, b, greedy, true);
  if (s) return s;
  ++nk;
  for (int l = 0; l < e->hp.n_layer; ++l) {
    for (int c = K_QKV; c <= K_DOWN; ++c) {
      if (c == K_ROUTER && route_fused(e, b)) continue;
      if ((s = launch_one(e, c, l, b, greedy, true))) return s;
      ++nk;
      if (c == K_OPROJ && e->head_par) {  // add the ranks' attention projections
        if ((s = launch_combine(e, l, 0, b, e->ffn_inp))) return s;
        ++nk;
      }
    }
    if (e->ep_size > 1) {  // add the ranks' expert outputs (peer memory)
      if ((s = launch_combine(e, l, 1, b, e->x))) return s;
      ++nk;
    }
  }
  if ((s = launch_one(e, K_LMHEAD, 0, b, greedy, true))) return s;
  nk += e->shard_now ? 2 : 1;  // (+ the argmax exchange)
  e->kernels_per_step = nk;
  return SFK_OK;
}

sfk_status get_graph(sfk_engine* e, int b, bool greedy, cudaGraphExec_t* out) {
  if (e->ep_size > 1 && !e->ep_connected)
    return fail(SFK_ERR_INVALID_ARGUMENT, "expert-parallel engine: call sfk_ep_connect before decoding");
  const int key = (b * 2 + (greedy ? 1 : 0)) * 2 + (e->shard_now ? 1 : 0);
  auto it = e->graphs.find(key);
  if (it != e->graphs.end()) {
    *out = it->second;
    return SFK_OK;
  }
  cudaGraph_t g = nullptr;
  CK(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
  sfk_status s = enqueue_step(e, b, greedy);
  cudaError_t ce = cudaStreamEndCapture(e->stream, &g);
  if (s != SFK_OK) {
    if (g) cudaGraphDestroy(g);
    return s;
  }
  if (ce != cudaSuccess) return fail(SFK_ERR_RUNTIME, "graph capture failed: %s", cudaGetErrorString(ce));
  cudaGraphExec_t ex = nullptr;
  ce = cudaGraphInstantiate(&ex, g, 0);
  cudaGraphDestroy(g);
  if (ce != cudaSuccess) return fail(SFK_ERR_RUNTIME, "graph instantiate failed: %s", cudaGetErrorString(ce));
  e->graphs[key] = ex;
  *out = ex;
  return SFK_OK;
}

// ---- the bounded expert tier ----------------------------------------------
// The reference keeps every expert bundle in its .strata file and a bounded
// SlotPool of host slots that it copies into staging tensors for the expert
// segment (engine.cpp:2004-2133); its prefetch warms the next layer's
// predicted experts (engine.cpp:2900-2923).  Here the bundles sit in pinned
// host memory in the device row layout, the slots are HBM, the expert kernels
// read the slots in place through a per-layer slot table, and every missing
// bundle is one host-to-device copy on a copy stream that the expert kernels
// wait for.  A layer's routing is read back before its experts run (the
// reference reads its ids back at the same point, engine.cpp:2840-2880).

int64_t round256(int64_t x) { return (x + 255) / 256 * 256; }

sfk_status tier_create(sfk_engine* e) {
  sfk_engine::Tier& T = e->tier;
  const sfk_hparams& hp = e->hp;
  const int d = hp.n_embd, F = hp.n_ff, E = hp.n_expert, k = hp.n_expert_used;
  const int64_t gu = (int64_t)F * dev_row_bytes(hp.type_ffn_gu, d);
  T.off_up = round256(gu);
  T.off_down = T.off_up + round256(gu);
  T.slot_bytes = round256(T.off_down + (int64_t)d * dev_row_bytes(hp.type_ffn_down, F));
  T.n_slots = (uint32_t)hp.expert_slots;
  sfk_status s = e->alloc(&T.pool, (size_t)T.n_slots * T.slot_bytes, &e->weight_bytes);
  if (!s) s = e->alloc(&T.d_map, sizeof(int) * (size_t)hp.n_layer * E, &e->scratch_bytes);
  if (s) return s;
  // the expert tiles of a prefill chunk (prefill_alloc's bound)
  const int C = std::min(512, hp.n_ctx), np = C * k;
  const int mt = (np + TC_TT - 1) / TC_TT + std::min(E, np);
  if ((s = e->alloc(&T.d_tile, sizeof(int) * mt, &e->scratch_bytes))) return s;
  CK(cudaMemset(T.d_map, 0xFF, sizeof(int) * (size_t)hp.n_layer * E));
  CK(cudaHostAlloc(&T.host, (size_t)hp.n_layer * E * T.slot_bytes, cudaHostAllocDefault));
  CK(cudaHostAlloc(&T.h_map, sizeof(int) * (size_t)hp.n_layer * E, cudaHostAllocDefault));
  CK(cudaHostAlloc(&T.h_route, sizeof(Route), cudaHostAllocDefault));
  CK(cudaHostAlloc(&T.h_tile, sizeof(int) * mt, cudaHostAllocDefault));
  CK(cudaHostAlloc(&T.h_ids, sizeof(int) * np, cudaHostAllocDefault));
  std::fill(T.h_map, T.h_map + (size_t)hp.n_layer * E, -1);
  CK(cudaStreamCreateWithFlags(&T.copy, cudaStreamNonBlocking));
  CK(cudaEventCreateWithFlags(&T.copied, cudaEventDisableTiming));
  // layer-stratified unless SFK_POOL_GLOBAL_LRU=1 (the reference's
  // STRATAFLOW_ENGINE_GLOBAL_LRU, engine.cpp:1404-1420)
  const char* g = getenv("SFK_POOL_GLOBAL_LRU");
  if (g && g[0] == '1')
    T.sp.reset(new (std::nothrow) SlotPool(T.n_slots));
  else
    T.sp.reset(new (std::nothrow) SlotPool(T.n_slots, hp.n_layer, E, k));
  T.pred.reset(new (std::nothrow) ExpertPredictor(hp.n_layer, E));
  if (!T.sp || !T.pred) return fail(SFK_ERR_OUT_OF_MEMORY, "host alloc");
  // prefetch policy (SFK_PREFETCH): 1 (default) installs a predicted bundle
  // only where that evicts nothing -- the reference's asynchronous install
  // rule (has_free_slot_in_layer, weight_store.h:94-123); 2 warms like its
  // synchronous warm_expert (engine.cpp:2135-2196), evicting within the
  // predicted layer; 0 turns prefetch off
  const char* pf = getenv("SFK_PREFETCH");
  T.prefetch = pf && (pf[0] == '0' || pf[0] == '2') ? pf[0] - '0' : 1;
  return SFK_OK;
}

// Bundle bytes of (layer l, expert x) in the pinned store.
uint8_t* tier_bundle(sfk_engine* e, int l, int x) {
  return e->tier.host + ((int64_t)l * e->hp.n_expert + x) * e->tier.slot_bytes;
}

// The host store changed: no slot holds a current copy any more.
sfk_status tier_invalidate(sfk_engine* e) {
  CK(cudaStreamSynchronize(e->tier.copy));
  CK(cudaStreamSynchronize(e->stream));
  e->tier.sp->clear();
  std::fill(e->tier.h_map, e->tier.h_map + (size_t)e->hp.n_layer * e->hp.n_expert, -1);
  return SFK_OK;
}

// SlotPool::acquire of (l, x); a miss copies the bundle into its slot on the
// copy stream.  *slot is SlotPool::NONE when every candidate slot is pinned.
sfk_status tier_acquire(sfk_engine* e, int l, int x, bool pin, uint32_t* slot) {
  sfk_engine::Tier& T = e->tier;
  bool miss = false;
  *slot = T.sp->acquire((uint32_t)l, (uint32_t)x, &miss);
  if (*slot == SlotPool::NONE) return SFK_OK;
  if (pin) T.sp->pin(*slot);
  if (miss) {
    CK(cudaMemcpyAsync(T.pool + (int64_t)*slot * T.slot_bytes, tier_bundle(e, l, x), T.slot_bytes,
                       cudaMemcpyHostToDevice, T.copy));
    T.h2d += T.slot_bytes;
  }
  return SFK_OK;
}

// The engine's stream waits for every bundle copy issued so far.
sfk_status tier_fence(sfk_engine* e) {
  CK(cudaEventRecord(e->tier.copied, e->tier.copy));
  CK(cudaStreamWaitEvent(e->stream, e->tier.copied, 0));
  return SFK_OK;
}

// Layer l's routing (already queued on the stream) read back; its experts
// acquired in the reference's order (each token's top-k in rank order, a
// token's duplicates skipped: engine.cpp:2036-2047) after the predictor
// observed them (engine.cpp:2863-2880); the layer's slot table uploaded.
sfk_status tier_route_layer(sfk_engine* e, int l, int b) {
  sfk_engine::Tier& T = e->tier;
  const int E = e->hp.n_expert, k = e->hp.n_expert_used;
  CK(cudaMemcpyAsync(T.h_route, e->route, sizeof(Route), cudaMemcpyDeviceToHost, e->stream));
  CK(cudaStreamSynchronize(e->stream));
  // every kernel queued before the read-back has finished: no slot is read
  T.sp->unpin_all();
  const Route& r = *T.h_route;
  if (r.b != b || r.k != k) return fail(SFK_ERR_RUNTIME, "layer %d: routing read back for %d x %d", l, r.b, r.k);
  for (int i = 0; i < b * k; ++i)
    if (r.ids[i] < 0 || r.ids[i] >= E) return fail(SFK_ERR_RUNTIME, "layer %d: routed expert %d", l, r.ids[i]);
  for (int i = 0; i < b * k; ++i) {
    const uint64_t key = (uint64_t)l << 32 | (uint32_t)r.ids[i];
    if (T.warmed_now.count(key)) ++T.used;
    T.pred->observe((uint32_t)l, (uint32_t)r.ids[i]);
  }
  int* row = T.h_map + (size_t)l * E;
  for (int t = 0; t < b; ++t)
    for (int j = 0; j < k; ++j) {
      const int x = r.ids[t * k + j];
      bool dup = false;
      for (int q = 0; q < j; ++q) dup = dup || r.ids[t * k + q] == x;
      if (dup) continue;
      uint32_t slot = 0;
      sfk_status s = tier_acquire(e, l, x, true, &slot);
      if (s) return s;
      if (slot == SlotPool::NONE)
        return fail(SFK_ERR_RUNTIME, "layer %d: no unpinned slot for expert %d", l, x);
      row[x] = (int)slot;
    }
  CK(cudaMemcpyAsync(T.d_map + (size_t)l * E, row, sizeof(int) * E, cudaMemcpyHostToDevice, e->stream));
  return tier_fence(e);
}

// Warm layer l's predicted experts (engine.cpp:2900-2923): no pin, so a
// later acquire may take the slot back; the copies overlap the kernels
// already queued.  By default only into free capacity: a warm that evicts
// trades a likely hit of the layer's resident set for a guess.
sfk_status tier_prefetch(sfk_engine* e, int l) {
  sfk_engine::Tier& T = e->tier;
  if (!T.prefetch || l >= e->hp.n_layer) return SFK_OK;
  for (uint32_t x : T.pred->predict((uint32_t)l, (uint32_t)e->hp.n_expert_used)) {
    if (T.sp->resident((uint32_t)l, x)) continue;
    if (T.prefetch == 1 && !T.sp->has_free_slot_in_layer((uint32_t)l)) break;
    uint32_t slot = 0;
    sfk_status s = tier_acquire(e, l, (int)x, false, &slot);
    if (s) return s;
    if (slot == SlotPool::NONE) continue;
    T.warmed_now.insert((uint64_t)l << 32 | x);
    ++T.warmed;
  }
  return SFK_OK;
}

// ---- the KV window ----------------------------------------------------------
// KvStore (src/kv/kv_store.h:30-95) with 16-token pages: sequence t's logical
// page j lives in ring slot j % pages of its HBM pages; before a position
// whose slot still holds a live older page is written, that page (every
// layer, K and V) goes to the pinned cold store and its page-table entry to
// its staged copy (KvStore::evicts, kv_store.h:84: the evicted column is saved
// before the ring write).  Each layer's attention then reads the cold pages
// from one layer's worth of staging HBM, refilled before the layer (the
// reference assembles cold + ring columns per layer, engine.cpp:1660-1749).

// The page table after a reset: every logical page in its first ring slot
// (or the permuted pool without a window); no page cold.
sfk_status window_table(sfk_engine* e) {
  CK(cudaMemcpyAsync(e->page_table, e->pt0.data(), sizeof(int) * e->pt0.size(), cudaMemcpyHostToDevice, e->stream));
  CK(cudaStreamSynchronize(e->stream));
  std::fill(e->win.cold.begin(), e->win.cold.end(), 0);
  return SFK_OK;
}

// Make position `pos` of sequence t writable: its page must not have gone
// cold, and every older page still in the slot it lands in is evicted.
sfk_status window_advance(sfk_engine* e, int t, int pos) {
  sfk_engine::Window& w = e->win;
  const int j = pos / 16, MP = e->max_pages, L = e->hp.n_layer;
  if (j < w.cold[t])
    return fail(SFK_ERR_INVALID_ARGUMENT, "sequence %d: position %d lies in a page that has left the KV window", t,
                pos);
  const size_t kv_elem = e->hp.kv_type == SFK_KV_F16 ? 2 : 4;
  const size_t layer_bytes = (size_t)e->kv_layer_elems * kv_elem;          // HBM pool, one layer
  const size_t cold_layer = (size_t)e->hp.max_batch * MP * w.page_bytes;    // cold store, one layer
  while (w.cold[t] + w.pages <= j) {
    const int q = w.cold[t];
    const int h = w.ring[(size_t)t * w.pages + q % w.pages];
    for (int v = 0; v < 2; ++v) {
      const uint8_t* src = static_cast<const uint8_t*>(v ? e->v_pool : e->k_pool) + (int64_t)h * w.page_bytes;
      uint8_t* dst = (v ? w.v_cold : w.k_cold) + ((size_t)t * MP + q) * w.page_bytes;
      if (layer_bytes < (1ull << 31) && cold_layer < (1ull << 31)) {
        CK(cudaMemcpy2DAsync(dst, cold_layer, src, layer_bytes, w.page_bytes, L, cudaMemcpyDeviceToHost, e->stream));
      } else {
        for (int l = 0; l < L; ++l)
          CK(cudaMemcpyAsync(dst + l * cold_layer, src + l * layer_bytes, w.page_bytes, cudaMemcpyDeviceToHost,
                             e->stream));
      }
    }
    CK(launch_pt_set(e->page_table, t * MP + q, e->n_pages + t * MP + q, e->stream));
    w.cold[t] = q + 1;
    ++w.evicted;
  }
  return SFK_OK;
}

// Layer l's cold pages of sequences [t0, t1) into staging buffer l & 1 (ids
// n_pages + t * max_pages + j), on stream `st`; *copied tells whether any were.
sfk_status window_stage(sfk_engine* e, int l, int t0, int t1, cudaStream_t st, bool* copied) {
  sfk_engine::Window& w = e->win;
  *copied = false;
  const int B = e->hp.max_batch, MP = e->max_pages;
  for (int t = t0; t < t1; ++t) {
    const int c = w.cold[t];
    if (c == 0) continue;
    for (int v = 0; v < 2; ++v) {
      const uint8_t* src = (v ? w.v_cold : w.k_cold) + ((size_t)l * B + t) * MP * w.page_bytes;
      uint8_t* dst = static_cast<uint8_t*>(v ? w.v_stage[l & 1] : w.k_stage[l & 1]) + (size_t)t * MP * w.page_bytes;
      CK(cudaMemcpyAsync(dst, src, (size_t)c * w.page_bytes, cudaMemcpyHostToDevice, st));
    }
    w.staged_bytes += 2ull * c * w.page_bytes;
    *copied = true;
  }
  return SFK_OK;
}

// Decode steps stage on the window's copy stream, a layer ahead: layer l's
// copies go into buffer l & 1 once layer l - 2's attention has read it, and
// layer l's attention waits for them.  The first two layers' copies wait
// for everything queued before the step (evictions included).
sfk_status window_stage_async(sfk_engine* e, int l, int b, bool* copied) {
  sfk_engine::Window& w = e->win;
  CK(cudaStreamWaitEvent(w.copy, l < 2 ? w.start : w.used[l & 1], 0));
  sfk_status s = window_stage(e, l, 0, b, w.copy, copied);
  if (s) return s;
  if (*copied) CK(cudaEventRecord(w.staged[l & 1], w.copy));
  return SFK_OK;
}

// A decode step as a direct launch chain, for engines whose steps need the
// host between launches: a bounded expert tier reads each layer's routing
// back before its experts run; a KV window evicts pages before the step and
// stages each layer's cold pages before its QKV kernel.
sfk_status run_step_direct(sfk_engine* e, int b, bool greedy) {
  sfk_engine::Tier& T = e->tier;
  sfk_status s = SFK_OK;
  if (e->win.on)
    for (int t = 0; t < b && !s; ++t) s = window_advance(e, t, e->step_pos[t]);
  if (s) return s;
  if (T.on) {
    // spare slots follow the observed per-layer activity, every 4 tokens
    // (engine.cpp:2511-2523)
    if (T.sp->stratified() && T.tokens % 4 == 0) T.sp->set_layer_weights(T.pred->layer_activity());
    T.warmed_now.clear();
  }
  const int L = e->hp.n_layer;
  bool staged[2] = {false, false};
  if (e->win.on) {
    if (!s) s = cudaEventRecord(e->win.start, e->stream) == cudaSuccess ? SFK_OK : fail(SFK_ERR_RUNTIME, "event");
    for (int l = 0; l < std::min(2, L) && !s; ++l) s = window_stage_async(e, l, b, &staged[l]);
  }
  if (!s) s = launch_one(e, K_EMBED, 0, b, greedy, false);
  int nk = 1;
  for (int l = 0; l < L && !s; ++l) {
    s = launch_one(e, K_QKV, l, b, greedy, true);
    const bool wait = e->win.on && staged[l & 1];
    if (!s && wait && cudaStreamWaitEvent(e->stream, e->win.staged[l & 1], 0) != cudaSuccess)
      s = fail(SFK_ERR_RUNTIME, "stream wait");
    // (a kernel that follows an event wait is a plain launch)
    if (!s) s = launch_one(e, K_ATTN, l, b, greedy, !wait);
    if (!s && e->win.on && l + 2 < L) {
      if (cudaEventRecord(e->win.used[l & 1], e->stream) != cudaSuccess) s = fail(SFK_ERR_RUNTIME, "event");
      if (!s) s = window_stage_async(e, l + 2, b, &staged[l & 1]);
    }
    if (!s) s = launch_one(e, K_OPROJ, l, b, greedy, true);
    nk += 3;
    if (!route_fused(e, b)) {
      if (!s) s = launch_one(e, K_ROUTER, l, b, greedy, true);
      ++nk;
    }
    if (!s && T.on) s = tier_route_layer(e, l, b);
    if (!s) s = launch_one(e, K_GATEUP, l, b, greedy, !T.on);
    if (!s) s = launch_one(e, K_DOWN, l, b, greedy, true);
    nk += 2;
    if (!s && T.on) s = tier_prefetch(e, l + 1);
  }
  if (!s) s = launch_one(e, K_LMHEAD, 0, b, greedy, true);
  if (s) {
    cudaStreamSynchronize(e->stream);
    if (e->win.on) cudaStreamSynchronize(e->win.copy);
    if (T.on) {
      cudaStreamSynchronize(T.copy);
      T.sp->unpin_all();
    }
    return s;
  }
  e->kernels_per_step = nk + 1;
  if (T.on) T.tokens += 1;
  return SFK_OK;
}

sfk_status validate_hp(const sfk_hparams* hp) {
  if (!hp) return fail(SFK_ERR_INVALID_ARGUMENT, "null hparams");
  if (hp->n_embd <= 0 || hp->n_head <= 0 || hp->n_head_kv <= 0 || hp->n_layer <= 0 || hp->n_ff <= 0 ||
      hp->n_expert <= 0 || hp->n_expert_used <= 0 || hp->n_vocab <= 0 || hp->n_ctx <= 0)
    return fail(SFK_ERR_INVALID_ARGUMENT, "hparams must be positive");
  if (hp->expert_slots < 0) return fail(SFK_ERR_INVALID_ARGUMENT, "expert_slots %d", hp->expert_slots);
  if (hp->n_head % hp->n_head_kv || (hp->head_dim <= 0 && hp->n_embd % hp->n_head))
    return fail(SFK_ERR_INVALID_ARGUMENT, "n_head must divide by n_head_kv and n_embd by n_head");
  const int hd = hp->head_dim > 0 ? hp->head_dim : hp->n_embd / hp->n_head;
  if (hd != 32 && hd != 64 && hd != 128 && hd != 256)
    return fail(SFK_ERR_UNSUPPORTED, "head_dim %d not in {32,64,128,256}", hd);
  if (hp->n_embd % 256 || hp->n_ff % 256)
    return fail(SFK_ERR_UNSUPPORTED, "n_embd and n_ff must be multiples of 256");
  if (hp->n_expert_used > hp->n_expert || hp->n_expert_used > 16 || hp->n_expert > 512)
    return fail(SFK_ERR_UNSUPPORTED, "need n_expert_used <= min(16, n_expert) and n_expert <= 512");
  if (hp->max_batch < 1 || hp->max_batch > MAXB || hp->max_batch * hp->n_expert_used > MAXP)
    return fail(SFK_ERR_UNSUPPORTED, "max_batch must be in [1,%d] with max_batch*n_expert_used <= %d", MAXB, MAXP);
  const int types[] = {hp->type_attn, hp->type_ffn_gu, hp->type_ffn_down, hp->type_output};
  for (int t : types)
    if (!quant_ok(t)) return fail(SFK_ERR_UNSUPPORTED, "weight type %d not supported (Q4_K, Q6_K, Q8_0)", t);
  if (!quant_ok(hp->type_embd) && hp->type_embd != T_F32 && hp->type_embd != T_F16)
    return fail(SFK_ERR_UNSUPPORTED, "embedding type %d not supported", hp->type_embd);
  if (hp->kv_type != SFK_KV_F32 && hp->kv_type != SFK_KV_F16)
    return fail(SFK_ERR_INVALID_ARGUMENT, "kv_type must be SFK_KV_F32 or SFK_KV_F16");
  if (hp->ep_size > 1) {
    if (hp->ep_size > MAXR || hp->n_expert % hp->ep_size || hp->ep_rank < 0 || hp->ep_rank >= hp->ep_size)
      return fail(SFK_ERR_INVALID_ARGUMENT, "ep_size must be in [2,%d] and divide n_expert; 0 <= ep_rank < ep_size",
                  MAXR);
  }
  return SFK_OK;
}

}  // namespace

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" {

const char* sfk_last_error(void) { return g_err.c_str(); }

const char* sfk_status_str(sfk_status s) {
  switch (s) {
    case SFK_OK: return "ok";
    case SFK_ERR_INVALID_ARGUMENT: return "invalid argument";
    case SFK_ERR_UNSUPPORTED: return "unsupported";
    case SFK_ERR_OUT_OF_MEMORY: return "out of memory";
    case SFK_ERR_RUNTIME: return "runtime error";
    default: return "unknown status";
  }
}

void sfk_engine_free(sfk_engine* e) {
  if (!e) return;
  cudaSetDevice(e->device);
  if (e->stream) cudaStreamSynchronize(e->stream);
  for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
  for (void* p : e->ep_opened) cudaIpcCloseMemHandle(p);
  if (e->tier.copy) cudaStreamSynchronize(e->tier.copy);
  if (e->win.copy) cudaStreamSynchronize(e->win.copy);
  for (void* p : e->allocs) cudaFree(p);
  for (void* p : {(void*)e->tier.host, (void*)e->tier.h_map, (void*)e->tier.h_route, (void*)e->tier.h_tile,
                  (void*)e->tier.h_ids, (void*)e->win.k_cold, (void*)e->win.v_cold})
    if (p) cudaFreeHost(p);
  if (e->tier.copied) cudaEventDestroy(e->tier.copied);
  if (e->tier.copy) cudaStreamDestroy(e->tier.copy);
  for (cudaEvent_t ev : {e->win.start, e->win.staged[0], e->win.staged[1], e->win.used[0], e->win.used[1]})
    if (ev) cudaEventDestroy(ev);
  if (e->win.copy) cudaStreamDestroy(e->win.copy);
  if (e->h_tok) cudaFreeHost(e->h_tok);
  if (e->h_hist) cudaFreeHost(e->h_hist);
  if (e->h_keys) cudaFreeHost(e->h_keys);
  if (e->h_logits) cudaFreeHost(e->h_logits);
  if (e->stream) cudaStreamDestroy(e->stream);
  delete e;
}

void* sfk_engine_stream(sfk_engine* e) { return e ? (void*)e->stream : nullptr; }

sfk_status sfk_engine_create(int device, const sfk_hparams* hp, sfk_engine** out) {
  if (!out) return fail(SFK_ERR_INVALID_ARGUMENT, "null out");
  *out = nullptr;
  sfk_status s = validate_hp(hp);
  if (s) return s;
  int ndev = 0;
  CK(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) return fail(SFK_ERR_INVALID_ARGUMENT, "device %d of %d", device, ndev);
  CK(cudaSetDevice(device));
  sfk_engine* e = new (std::nothrow) sfk_engine();
  if (!e) return fail(SFK_ERR_OUT_OF_MEMORY, "host alloc");
  e->device = device;
  e->hp = *hp;
  e->hd = hp->head_dim > 0 ? hp->head_dim : hp->n_embd / hp->n_head;
  {
    const int N = hp->ep_size > 1 ? hp->ep_size : 1;
    // SFK_HEAD_PARALLEL=0 keeps the attention trunk replicated on every rank
    const char* hpv = getenv("SFK_HEAD_PARALLEL");
    e->head_par = N > 1 && hp->n_head % N == 0 && hp->n_head_kv % N == 0 &&
                  (hp->n_head / N) * e->hd % 256 == 0 &&  // the projection's column slice is whole 256-blocks
                  !(hpv && atoi(hpv) == 0);
    const int R = e->head_par ? hp->ep_rank : 0, NP = e->head_par ? N : 1;
    e->hq_loc = hp->n_head / NP;
    e->hkv_loc = hp->n_head_kv / NP;
    e->q0 = R * e->hq_loc;
    e->kv0 = R * e->hkv_loc;
  }
  e->nq = e->hq_loc * e->hd;  // this rank's query rows (all of them without head parallelism)
  e->nk = e->hkv_loc * e->hd;
  e->nqkv = e->nq + 2 * e->nk;
  e->sm_count = sm_count_of(device);
  e->seq_pos.assign(hp->max_batch, 0);
  e->ep_size = hp->ep_size > 1 ? hp->ep_size : 1;
  e->ep_rank = hp->ep_size > 1 ? hp->ep_rank : 0;
  e->e_loc = hp->n_expert / e->ep_size;
  e->e0 = e->ep_rank * e->e_loc;
#define TRY(x)               \
  do {                       \
    sfk_status s_ = (x);     \
    if (s_) {                \
      sfk_engine_free(e);    \
      return s_;             \
    }                        \
  } while (0)
  {
    cudaError_t ce = cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking);
    if (ce != cudaSuccess) {
      sfk_engine_free(e);
      return fail(SFK_ERR_RUNTIME, "stream create: %s", cudaGetErrorString(ce));
    }
  }
  const int d = hp->n_embd, F = hp->n_ff, E = hp->n_expert, V = hp->n_vocab;
  const int B = hp->max_batch, k = hp->n_expert_used;
  // a bounded expert tier when expert_slots is below the whole working set
  // (engine.cpp:1386-1394: 0 = auto, every expert resident)
  e->tier.on = hp->expert_slots > 0 && (int64_t)hp->expert_slots < (int64_t)hp->n_layer * E;
  if (e->tier.on && e->ep_size > 1) {
    sfk_engine_free(e);
    return fail(SFK_ERR_UNSUPPORTED, "a bounded expert tier (expert_slots %d) needs a single-GPU engine",
                hp->expert_slots);
  }
  if (e->tier.on && hp->expert_slots < std::min(E, B * k)) {
    sfk_engine_free(e);
    return fail(SFK_ERR_INVALID_ARGUMENT,
                "expert_slots %d cannot hold one step's routed experts of a layer (%d): the kernels read the "
                "slots in place",
                hp->expert_slots, std::min(E, B * k));
  }
  // weights (HBM tier)
  TRY(e->alloc(&e->tok_embd, dev_gguf_row_bytes(hp->type_embd, d) * V, &e->weight_bytes));
  TRY(e->alloc(&e->out_norm, sizeof(float) * d, &e->weight_bytes));
  TRY(e->alloc(&e->output, dev_row_bytes(hp->type_output, d) * V, &e->weight_bytes));
  e->L.resize(hp->n_layer);
  for (int l = 0; l < hp->n_layer; ++l) {
    LayerW& W = e->L[l];
    TRY(e->alloc(&W.qkv, dev_row_bytes(hp->type_attn, d) * e->nqkv, &e->weight_bytes));
    TRY(e->alloc(&W.wo, dev_row_bytes(hp->type_attn, e->nq) * d, &e->weight_bytes));
    TRY(e->alloc(&W.attn_norm, sizeof(float) * d, &e->weight_bytes));
    TRY(e->alloc(&W.ffn_norm, sizeof(float) * d, &e->weight_bytes));
    TRY(e->alloc(&W.router, sizeof(float) * d * E, &e->weight_bytes));
    if (e->tier.on) continue;  // the experts live in the pool's slots
    const int El = e->e_loc;  // this rank's experts
    TRY(e->alloc(&W.gate, dev_row_bytes(hp->type_ffn_gu, d) * F * El, &e->weight_bytes));
    TRY(e->alloc(&W.up, dev_row_bytes(hp->type_ffn_gu, d) * F * El, &e->weight_bytes));
    TRY(e->alloc(&W.down, dev_row_bytes(hp->type_ffn_down, F) * d * El, &e->weight_bytes));
  }
  if (e->tier.on) TRY(tier_create(e));
  // paged KV: one pool per layer of B * ceil(n_ctx/16) pages [Hkv][16][hd];
  // pages are handed to sequences in a seeded permuted order (a fragmented
  // pool, as a page allocator produces).
  e->max_pages = (hp->n_ctx + 15) / 16;
  e->win.on = hp->kv_window > 0 && hp->kv_window < hp->n_ctx;
  if (e->win.on) {
    e->win.pages = (hp->kv_window + 15) / 16;
    if (e->win.pages < 2 || e->ep_size > 1) {
      sfk_engine_free(e);
      return fail(e->ep_size > 1 ? SFK_ERR_UNSUPPORTED : SFK_ERR_INVALID_ARGUMENT,
                  "kv_window %d: a window spans at least two 16-token pages, on a single-GPU engine", hp->kv_window);
    }
    if (e->win.pages >= e->max_pages) e->win.on = false;  // the window holds the whole context
  }
  e->n_pages = B * (e->win.on ? e->win.pages : e->max_pages);
  e->kv_layer_elems = (int64_t)e->n_pages * e->hkv_loc * 16 * e->hd;
  const size_t kv_elem = hp->kv_type == SFK_KV_F16 ? 2 : 4;
  TRY(e->alloc(&e->k_pool, kv_elem * e->kv_layer_elems * hp->n_layer, &e->kv_bytes));
  TRY(e->alloc(&e->v_pool, kv_elem * e->kv_layer_elems * hp->n_layer, &e->kv_bytes));
  TRY(e->alloc(&e->page_table, sizeof(int) * B * e->max_pages, &e->kv_bytes));
  {
    // HBM pages handed out in a seeded permuted order (a fragmented pool, as
    // a page allocator produces); with a window, sequence t's ring slot r is
    // page perm[t * pages + r] and logical page j starts in slot j % pages
    std::vector<int> perm(e->n_pages);
    for (int i = 0; i < e->n_pages; ++i) perm[i] = i;
    uint64_t st = 0x5F3759DFull;
    for (int i = e->n_pages - 1; i > 0; --i) {
      st = splitmix64(st);
      const int j = (int)(st % (uint64_t)(i + 1));
      std::swap(perm[i], perm[j]);
    }
    e->pt0 = perm;
    if (e->win.on) {
      sfk_engine::Window& w = e->win;
      w.ring = perm;
      w.cold.assign(B, 0);
      e->pt0.assign((size_t)B * e->max_pages, 0);
      for (int t = 0; t < B; ++t)
        for (int j = 0; j < e->max_pages; ++j)
          e->pt0[(size_t)t * e->max_pages + j] = w.ring[(size_t)t * w.pages + j % w.pages];
      w.page_bytes = (int64_t)e->hkv_loc * 16 * e->hd * kv_elem;
      const size_t stage = (size_t)B * e->max_pages * w.page_bytes;
      for (int i = 0; i < 2; ++i) {
        TRY(e->alloc(&w.k_stage[i], stage, &e->kv_bytes));
        TRY(e->alloc(&w.v_stage[i], stage, &e->kv_bytes));
      }
      CK(cudaHostAlloc(&w.k_cold, stage * hp->n_layer, cudaHostAllocDefault));
      CK(cudaHostAlloc(&w.v_cold, stage * hp->n_layer, cudaHostAllocDefault));
      CK(cudaStreamCreateWithFlags(&w.copy, cudaStreamNonBlocking));
      CK(cudaEventCreateWithFlags(&w.start, cudaEventDisableTiming));
      for (int i = 0; i < 2; ++i) {
        CK(cudaEventCreateWithFlags(&w.staged[i], cudaEventDisableTiming));
        CK(cudaEventCreateWithFlags(&w.used[i], cudaEventDisableTiming));
      }
    }
    TRY(window_table(e));
  }
  e->step_pos.assign(B, 0);
  // step buffers
  e->attn_cluster = attn_cluster_for(e->max_pages * 16);
  e->attn_max_chunk = (e->max_pages + e->attn_cluster - 1) / e->attn_cluster * 16;  // whole pages per CTA
  {
    // 16-CTA clusters (twice the SMs per kv head) when every (sequence, kv
    // head) cluster of a step fits on the GPU at once; SFK_ATTN_CLUSTER
    // forces 8 or 16
    int want = 0;
    if (const char* v = getenv("SFK_ATTN_CLUSTER")) want = atoi(v);
    if (want == 0 && B * e->hkv_loc <= 8 && e->max_pages >= 32) want = 16;
    if (want == 16 && e->attn_cluster != 16) {
      const int mc16 = (e->max_pages + 15) / 16 * 16;
      if (attn_active_clusters(e->hd, hp->kv_type == SFK_KV_F16, hp->n_head / hp->n_head_kv, 16, mc16) >=
          B * e->hkv_loc) {
        e->attn_cluster = 16;
        e->attn_max_chunk = mc16;
      }
    }
    if (want == 8 && e->attn_cluster == 16 && e->max_pages * 16 <= 8 * 2048) {
      e->attn_cluster = 8;
      e->attn_max_chunk = (e->max_pages + 7) / 8 * 16;
    }
  }
  if (attn_smem_bytes(e->hd, hp->n_head / hp->n_head_kv, hp->kv_type == SFK_KV_F16, e->attn_max_chunk) >
      (size_t)SMEM_LIMIT) {
    sfk_engine_free(e);
    return fail(SFK_ERR_UNSUPPORTED, "n_ctx %d too long for the attention kernel's shared memory", hp->n_ctx);
  }
  uint64_t* sb = &e->scratch_bytes;
  TRY(e->alloc(&e->x, sizeof(float) * B * d, sb));
  TRY(e->alloc(&e->ffn_inp, sizeof(float) * B * d, sb));
  TRY(e->alloc(&e->q, sizeof(float) * B * e->nq, sb));
  TRY(e->alloc(&e->attn_out, sizeof(float) * B * e->nq, sb));
  TRY(e->alloc(&e->h, sizeof(float) * B * k * F, sb));
  TRY(e->alloc(&e->logits, sizeof(float) * B * V, sb));
  TRY(e->alloc(&e->rope, sizeof(float) * (size_t)e->max_pages * 16 * e->hd, sb));
  TRY(e->alloc(&e->router_logits, sizeof(float) * B * E, sb));
  TRY(e->alloc(&e->xq_ffn, qact_bytes(d) * B, sb));
  TRY(e->alloc(&e->hq, qact_bytes(F) * B * k, sb));
  TRY(e->alloc(&e->route, sizeof(Route), sb));
  TRY(e->alloc(&e->router_counter, 2 * sizeof(int), sb));
  TRY(e->alloc(&e->grp_counter, sizeof(int) * (F / 256), sb));
  TRY(e->alloc(&e->argmax_key, sizeof(unsigned long long) * B + 16, sb));
  e->status = reinterpret_cast<int*>(e->argmax_key + B);
  TRY(e->alloc(&e->tok_in, sizeof(int) * 2 * B, sb));
  e->pos_in = e->tok_in + B;
  TRY(e->alloc(&e->pos_state, sizeof(int) * B, sb));
  TRY(e->alloc(&e->pos_cur, sizeof(int) * B, sb));
  TRY(e->alloc(&e->tok_hist, sizeof(int) * B, sb));
  if (e->ep_size > 1) {
    // exchange buffer: [layer parity][stage][B][d] partial outputs, then MAXR
    // flag words; its own allocation so that its IPC handle exposes nothing else
    // tail: flag words [MAXR] at +0, head flag words [MAXR] at +128, argmax keys [MAXB] at +256
    const size_t part = sizeof(float) * 4 * (size_t)B * d;
    const size_t tail = 256 + sizeof(unsigned long long) * MAXB;
    TRY(e->alloc(&e->ep_buf, part + tail, sb));
    uint8_t* tb = reinterpret_cast<uint8_t*>(e->ep_buf) + part;
    e->ep_flags = reinterpret_cast<unsigned*>(tb);
    e->ep_head_flags = reinterpret_cast<unsigned*>(tb + 128);
    e->ep_keys = reinterpret_cast<unsigned long long*>(tb + 256);
    {
      // SFK_VOCAB_SHARD=0 keeps the lm_head replicated
      const char* vs = getenv("SFK_VOCAB_SHARD");
      const int N = e->ep_size;
      e->v_loc = (V + N - 1) / N;
      e->v0 = e->ep_rank * e->v_loc;
      e->v_loc = std::max(0, std::min(e->v_loc, V - e->v0));
      e->head_shard = !(vs && vs[0] == '0') && (int64_t)(N - 1) * ((V + N - 1) / N) < V;  // no empty slice
    }
    TRY(e->alloc(&e->ep_step, sizeof(unsigned), sb));
    cudaError_t ce = cudaMemset(e->ep_buf, 0, part + tail);
    if (ce == cudaSuccess) ce = cudaMemset(e->ep_step, 0, sizeof(unsigned));
    if (ce != cudaSuccess) {
      sfk_engine_free(e);
      return fail(SFK_ERR_RUNTIME, "engine init: %s", cudaGetErrorString(ce));
    }
  }
  {
    cudaError_t ce = cudaSuccess;
    ce = cudaMemset(e->router_counter, 0, 2 * sizeof(int));
    if (ce == cudaSuccess) ce = cudaMemset(e->grp_counter, 0, sizeof(int) * (F / 256));
    if (ce == cudaSuccess) ce = cudaMemset(e->argmax_key, 0, sizeof(unsigned long long) * B);
    if (ce == cudaSuccess) ce = cudaMemset(e->pos_state, 0, sizeof(int) * B);
    if (ce == cudaSuccess) ce = cudaMemset(e->status, 0, sizeof(int));
    if (ce == cudaSuccess) ce = cudaMemset(e->k_pool, 0, kv_elem * e->kv_layer_elems * hp->n_layer);
    if (ce == cudaSuccess) ce = cudaMemset(e->v_pool, 0, kv_elem * e->kv_layer_elems * hp->n_layer);
    if (ce == cudaSuccess) ce = cudaMallocHost(&e->h_tok, sizeof(int) * 2 * B);
    if (ce == cudaSuccess) e->h_pos = e->h_tok + B;
    if (ce == cudaSuccess) ce = cudaMallocHost(&e->h_hist, sizeof(int) * B);
    if (ce == cudaSuccess) ce = cudaMallocHost(&e->h_keys, sizeof(unsigned long long) * B + 16);
    if (ce == cudaSuccess) e->h_status = reinterpret_cast<int*>(e->h_keys + B);
    if (ce == cudaSuccess) ce = cudaMallocHost(&e->h_logits, sizeof(float) * B * hp->n_vocab);
    if (ce != cudaSuccess) {
      sfk_engine_free(e);
      return fail(SFK_ERR_RUNTIME, "engine init: %s", cudaGetErrorString(ce));
    }
  }
  {
    // fold the router into the gate/up kernel when its warp-tile form fits:
    // small routers are staged whole in every CTA, large ones (hundreds of
    // experts) are scored a few logits per CTA and exchanged.
    // SFK_ROUTER_KERNEL=1 keeps the separate router kernel.
    const char* rk = getenv("SFK_ROUTER_KERNEL");
    // (a bounded tier reads each layer's routing back before its experts run)
    e->fused_route = !(rk && atoi(rk) == 1) && !e->tier.on;
    // SFK_FUSED_ROUTE_MAX_B moves the step size up to which routing stays fused
    e->fused_route_max_b = 2;
    if (const char* v = getenv("SFK_FUSED_ROUTE_MAX_B")) e->fused_route_max_b = std::max(1, atoi(v));
    e->fused_route_max_b = std::min(e->fused_route_max_b, B);
    StreamParams gp = gateup_params(e, 0, e->fused_route_max_b);
    int grid = 0;
    if (e->fused_route &&
        (plan_stream(gp, e->sm_count, &grid) != SFK_OK || stream2_smem_bytes(gp) > SMEM_LIMIT))
      e->fused_route = false;
  }
  {
    // the persistent step kernel (SFK_PERSISTENT=1): single-GPU engines whose
    // types, expert count and GQA group it covers; by default a step runs as
    // the launch chain, which is faster at the Mixtral shape today
    const char* pv = getenv("SFK_PERSISTENT");
    const int gqa = hp->n_head / hp->n_head_kv;
    int coop = 0;
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device);
    if (pv && atoi(pv) == 1 && coop && e->ep_size == 1 && !e->tier.on && !e->win.on && E <= MEGA_MAXE &&
        gqa <= MEGA_MAXGQA &&
        (gqa & (gqa - 1)) == 0 &&
        mega_types_supported(hp->type_attn, hp->type_ffn_gu, hp->type_ffn_down, hp->type_output)) {
      const int Hq = hp->n_head, Hkv = hp->n_head_kv;
      e->att_nc = (e->max_pages * 16 + MEGA_CH - 1) / MEGA_CH;
      TRY(e->alloc(&e->d_layers, sizeof(MegaLayer) * hp->n_layer, sb));
      TRY(e->alloc(&e->att_y, sizeof(float) * (size_t)B * Hq * hp->n_ctx, sb));
      TRY(e->alloc(&e->att_cmax, sizeof(float) * (size_t)B * Hkv * e->att_nc * gqa, sb));
      TRY(e->alloc(&e->att_stat, sizeof(float) * (size_t)B * Hq * 2, sb));
      TRY(e->alloc(&e->att_opart, sizeof(double) * (size_t)B * Hkv * e->att_nc * gqa * e->hd, sb));
      TRY(e->alloc(&e->att_cnt, sizeof(int) * 2 * B * Hkv, sb));
      TRY(e->alloc(&e->att_ready, sizeof(unsigned) * B * Hkv, sb));
      TRY(e->alloc(&e->gbar, 2 * sizeof(unsigned), sb));
      std::vector<MegaLayer> tab(hp->n_layer);
      for (int l = 0; l < hp->n_layer; ++l) {
        const LayerW& W = e->L[l];
        tab[l] = MegaLayer{W.qkv, W.wo, W.attn_norm, W.ffn_norm, W.router, W.gate, W.up, W.down};
      }
      cudaError_t ce = cudaMemcpy(e->d_layers, tab.data(), sizeof(MegaLayer) * tab.size(), cudaMemcpyHostToDevice);
      if (ce == cudaSuccess) ce = cudaMemset(e->att_cnt, 0, sizeof(int) * 2 * B * Hkv);
      if (ce == cudaSuccess) ce = cudaMemset(e->att_ready, 0, sizeof(unsigned) * B * Hkv);
      if (ce == cudaSuccess) ce = cudaMemset(e->gbar, 0, 2 * sizeof(unsigned));
      if (ce != cudaSuccess) {
        sfk_engine_free(e);
        return fail(SFK_ERR_RUNTIME, "persistent kernel init: %s", cudaGetErrorString(ce));
      }
      e->mega = true;
    }
  }
  {
    // RoPE cos/sin for every position (ggml rope cache, mode NORMAL,
    // freq_scale 1, ext_factor 0): theta_0 = pos, theta_{i+1} = theta_i *
    // powf(base, -2/n_dims), evaluated with the host libm
    const int half = e->hd / 2, npos = e->max_pages * 16;
    std::vector<float> tab((size_t)npos * e->hd);
    const float theta_scale = powf(hp->freq_base, -2.0f / (float)e->hd);
    for (int pos = 0; pos < npos; ++pos) {
      float theta = (float)pos;
      for (int i = 0; i < half; ++i) {
        tab[((size_t)pos * half + i) * 2 + 0] = cosf(theta);
        tab[((size_t)pos * half + i) * 2 + 1] = sinf(theta);
        theta *= theta_scale;
      }
    }
    cudaError_t ce = cudaMemcpy(e->rope, tab.data(), tab.size() * sizeof(float), cudaMemcpyHostToDevice);
    if (ce != cudaSuccess) {
      sfk_engine_free(e);
      return fail(SFK_ERR_RUNTIME, "rope table: %s", cudaGetErrorString(ce));
    }
  }
#undef TRY
  *out = e;
  return SFK_OK;
}

size_t sfk_tensor_bytes(const sfk_engine* e, int tid, int layer) {
  if (!e || tid < 0 || tid > SFK_T_FFN_DOWN_EXPS) return 0;
  if (layered(tid) ? (layer < 0 || layer >= e->hp.n_layer) : layer != 0) return 0;
  return (size_t)dev_gguf_row_bytes(tensor_type(e, tid), tensor_cols(e, tid)) * (size_t)tensor_rows(e, tid);
}

static bool expert_tensor(int tid) {
  return tid == SFK_T_FFN_GATE_EXPS || tid == SFK_T_FFN_UP_EXPS || tid == SFK_T_FFN_DOWN_EXPS;
}

// Bounded tier: a stacked expert tensor's rows, re-laid out, into each
// expert's bundle in the pinned store (gate / up / down part of the slot).
static sfk_status tier_put_stacked(sfk_engine* e, int tid, int layer, const uint8_t* dev_gguf) {
  sfk_engine::Tier& T = e->tier;
  const int type = tensor_type(e, tid), E = e->hp.n_expert;
  const int64_t cols = tensor_cols(e, tid), per = tensor_rows(e, tid) / E;
  const int64_t rs = dev_row_bytes(type, cols);
  const int64_t part = tid == SFK_T_FFN_GATE_EXPS ? 0 : tid == SFK_T_FFN_UP_EXPS ? T.off_up : T.off_down;
  uint8_t* tmp = nullptr;
  CK(cudaMallocAsync(&tmp, (size_t)E * per * rs, e->stream));
  cudaError_t ce = launch_repack(type, dev_gguf, tmp, E * per, (int)cols, e->stream);
  for (int x = 0; x < E && ce == cudaSuccess; ++x)
    ce = cudaMemcpyAsync(tier_bundle(e, layer, x) + part, tmp + (int64_t)x * per * rs, per * rs,
                         cudaMemcpyDeviceToHost, e->stream);
  cudaFreeAsync(tmp, e->stream);
  CK(ce);
  return tier_invalidate(e);
}

static sfk_status put_gguf_device(sfk_engine* e, int tid, int layer, const uint8_t* dev_gguf) {
  if (e->tier.on && expert_tensor(tid)) return tier_put_stacked(e, tid, layer, dev_gguf);
  const int type = tensor_type(e, tid);
  const int64_t rows = tensor_rows(e, tid), cols = tensor_cols(e, tid);
  uint8_t* dst = tensor_dst(e, tid, layer);
  if (relaid(tid)) {
    CK(launch_repack(type, dev_gguf, dst, rows, (int)cols, e->stream));
  } else {
    CK(cudaMemcpyAsync(dst, dev_gguf, sfk_tensor_bytes(e, tid, layer), cudaMemcpyDeviceToDevice, e->stream));
  }
  return SFK_OK;
}

sfk_status sfk_weights_put(sfk_engine* e, int tid, int layer, int ggml_type, const int64_t ne[3], const void* host,
                           size_t n_bytes) {
  if (!e || !host) return fail(SFK_ERR_INVALID_ARGUMENT, "null argument");
  const size_t want = sfk_tensor_bytes(e, tid, layer);
  if (want == 0) return fail(SFK_ERR_INVALID_ARGUMENT, "unknown tensor %d layer %d", tid, layer);
  if (ggml_type != tensor_type(e, tid))
    return fail(SFK_ERR_INVALID_ARGUMENT, "tensor %d: type %d, engine expects %d", tid, ggml_type, tensor_type(e, tid));
  if (ne) {
    const int64_t n_all = ne[0] * std::max<int64_t>(1, ne[1]) * std::max<int64_t>(1, ne[2]);
    if (ne[0] != tensor_cols(e, tid) || n_all != tensor_cols(e, tid) * tensor_rows(e, tid))
      return fail(SFK_ERR_INVALID_ARGUMENT, "tensor %d: shape mismatch", tid);
  }
  if (n_bytes != want) return fail(SFK_ERR_INVALID_ARGUMENT, "tensor %d: %zu bytes, expected %zu", tid, n_bytes, want);
  CK(cudaSetDevice(e->device));
  uint8_t* tmp = nullptr;
  CK(cudaMallocAsync(&tmp, want, e->stream));
  CK(cudaMemcpyAsync(tmp, host, want, cudaMemcpyHostToDevice, e->stream));
  sfk_status s = put_gguf_device(e, tid, layer, tmp);
  cudaFreeAsync(tmp, e->stream);
  if (s) return s;
  CK(cudaStreamSynchronize(e->stream));
  return SFK_OK;
}

sfk_status sfk_expert_put(sfk_engine* e, int layer, int expert, const void* bundle, size_t n_bytes) {
  if (!e || !bundle) return fail(SFK_ERR_INVALID_ARGUMENT, "null argument");
  const sfk_hparams& hp = e->hp;
  if (layer < 0 || layer >= hp.n_layer || expert < 0 || expert >= hp.n_expert)
    return fail(SFK_ERR_INVALID_ARGUMENT, "expert (%d,%d) out of range", layer, expert);
  if (expert < e->e0 || expert >= e->e0 + e->e_loc) return SFK_OK;  // another rank's expert
  expert -= e->e0;
  const size_t gl = dev_gguf_row_bytes(hp.type_ffn_gu, hp.n_embd) * hp.n_ff;
  const size_t dl = dev_gguf_row_bytes(hp.type_ffn_down, hp.n_ff) * hp.n_embd;
  if (n_bytes != 2 * gl + dl) return fail(SFK_ERR_INVALID_ARGUMENT, "bundle %zu bytes, expected %zu", n_bytes, 2 * gl + dl);
  CK(cudaSetDevice(e->device));
  uint8_t* tmp = nullptr;
  CK(cudaMallocAsync(&tmp, n_bytes, e->stream));
  CK(cudaMemcpyAsync(tmp, bundle, n_bytes, cudaMemcpyHostToDevice, e->stream));
  const LayerW& W = e->L[layer];
  const int64_t rs_gu = dev_row_bytes(hp.type_ffn_gu, hp.n_embd), rs_dn = dev_row_bytes(hp.type_ffn_down, hp.n_ff);
  if (e->tier.on) {  // re-laid out into a device bundle, then into the pinned store
    sfk_engine::Tier& T = e->tier;
    uint8_t* slot = nullptr;
    cudaError_t ce = cudaMallocAsync(&slot, T.slot_bytes, e->stream);
    if (ce == cudaSuccess) ce = launch_repack(hp.type_ffn_gu, tmp, slot, hp.n_ff, hp.n_embd, e->stream);
    if (ce == cudaSuccess) ce = launch_repack(hp.type_ffn_gu, tmp + gl, slot + T.off_up, hp.n_ff, hp.n_embd, e->stream);
    if (ce == cudaSuccess)
      ce = launch_repack(hp.type_ffn_down, tmp + 2 * gl, slot + T.off_down, hp.n_embd, hp.n_ff, e->stream);
    if (ce == cudaSuccess)
      ce = cudaMemcpyAsync(tier_bundle(e, layer, expert), slot, T.slot_bytes, cudaMemcpyDeviceToHost, e->stream);
    if (slot) cudaFreeAsync(slot, e->stream);
    cudaFreeAsync(tmp, e->stream);
    CK(ce);
    return tier_invalidate(e);
  }
  CK(launch_repack(hp.type_ffn_gu, tmp, W.gate + (int64_t)expert * hp.n_ff * rs_gu, hp.n_ff, hp.n_embd, e->stream));
  CK(launch_repack(hp.type_ffn_gu, tmp + gl, W.up + (int64_t)expert * hp.n_ff * rs_gu, hp.n_ff, hp.n_embd, e->stream));
  CK(launch_repack(hp.type_ffn_down, tmp + 2 * gl, W.down + (int64_t)expert * hp.n_embd * rs_dn, hp.n_embd, hp.n_ff,
                   e->stream));
  cudaFreeAsync(tmp, e->stream);
  CK(cudaStreamSynchronize(e->stream));
  return SFK_OK;
}

sfk_status sfk_weights_get(sfk_engine* e, int tid, int layer, void* host_out, size_t n_bytes) {
  if (!e || !host_out) return fail(SFK_ERR_INVALID_ARGUMENT, "null argument");
  const size_t want = sfk_tensor_bytes(e, tid, layer);
  if (want == 0 || n_bytes != want) return fail(SFK_ERR_INVALID_ARGUMENT, "tensor %d: bad size", tid);
  CK(cudaSetDevice(e->device));
  const uint8_t* src = tensor_dst(e, tid, layer);
  if (e->tier.on && expert_tensor(tid)) {  // from the pinned store's bundles
    sfk_engine::Tier& T = e->tier;
    const int type = tensor_type(e, tid), E = e->hp.n_expert;
    const int64_t cols = tensor_cols(e, tid), per = tensor_rows(e, tid) / E, rs = dev_row_bytes(type, cols);
    const int64_t part = tid == SFK_T_FFN_GATE_EXPS ? 0 : tid == SFK_T_FFN_UP_EXPS ? T.off_up : T.off_down;
    uint8_t *dev = nullptr, *tmp = nullptr;
    CK(cudaMallocAsync(&dev, (size_t)E * per * rs, e->stream));
    cudaError_t ce = cudaMallocAsync(&tmp, want, e->stream);
    for (int x = 0; x < E && ce == cudaSuccess; ++x)
      ce = cudaMemcpyAsync(dev + (int64_t)x * per * rs, tier_bundle(e, layer, x) + part, per * rs,
                           cudaMemcpyHostToDevice, e->stream);
    if (ce == cudaSuccess) ce = launch_unpack(type, dev, tmp, E * per, (int)cols, e->stream);
    if (ce == cudaSuccess) ce = cudaMemcpyAsync(host_out, tmp, want, cudaMemcpyDeviceToHost, e->stream);
    cudaFreeAsync(dev, e->stream);
    if (tmp) cudaFreeAsync(tmp, e->stream);
    CK(ce);
    CK(cudaStreamSynchronize(e->stream));
    return SFK_OK;
  }
  if (relaid(tid)) {
    uint8_t* tmp = nullptr;
    CK(cudaMallocAsync(&tmp, want, e->stream));
    CK(launch_unpack(tensor_type(e, tid), src, tmp, tensor_rows(e, tid), (int)tensor_cols(e, tid), e->stream));
    CK(cudaMemcpyAsync(host_out, tmp, want, cudaMemcpyDeviceToHost, e->stream));
    cudaFreeAsync(tmp, e->stream);
  } else {
    CK(cudaMemcpyAsync(host_out, src, want, cudaMemcpyDeviceToHost, e->stream));
  }
  CK(cudaStreamSynchronize(e->stream));
  return SFK_OK;
}

sfk_status sfk_weights_synth(sfk_engine* e, uint64_t seed) {
  if (!e) return fail(SFK_ERR_INVALID_ARGUMENT, "null engine");
  CK(cudaSetDevice(e->device));
  size_t maxb = 0;
  for (int tid = 0; tid <= SFK_T_FFN_DOWN_EXPS; ++tid) maxb = std::max(maxb, sfk_tensor_bytes(e, tid, 0));
  uint8_t* tmp = nullptr;
  CK(cudaMallocAsync(&tmp, maxb, e->stream));
  for (int tid = 0; tid <= SFK_T_FFN_DOWN_EXPS; ++tid) {
    const int nl = layered(tid) ? e->hp.n_layer : 1;
    for (int l = 0; l < nl; ++l) {
      const int64_t rows = tensor_rows(e, tid), cols = tensor_cols(e, tid);
      if (tid == SFK_T_OUTPUT_NORM || tid == SFK_T_ATTN_NORM || tid == SFK_T_FFN_NORM) {
        CK(launch_fill_f32(reinterpret_cast<float*>(tensor_dst(e, tid, l)), 1.0f, cols, e->stream));
        continue;
      }
      const int type = tensor_type(e, tid);
      // expert tensors: this rank's rows of the full stacked tensor
      // head-sharded tensors: this rank's rows of Q/K/V, its columns of the
      // output projection
      int64_t row0 = tid == SFK_T_FFN_GATE_EXPS || tid == SFK_T_FFN_UP_EXPS ? (int64_t)e->e0 * e->hp.n_ff
                     : tid == SFK_T_FFN_DOWN_EXPS                          ? (int64_t)e->e0 * e->hp.n_embd
                                                                            : 0;
      int64_t col0 = 0, kfull = 0;
      if (tid == SFK_T_ATTN_Q) row0 = (int64_t)e->q0 * e->hd;
      if (tid == SFK_T_ATTN_K || tid == SFK_T_ATTN_V) row0 = (int64_t)e->kv0 * e->hd;
      if (tid == SFK_T_ATTN_OUT) {
        col0 = (int64_t)e->q0 * e->hd;
        kfull = (int64_t)e->hp.n_head * e->hd;
      }
      CK(launch_synth(type, tensor_seed(seed, tid, l), 0.02f, tmp, rows, (int)cols, e->stream, row0, col0, kfull));
      sfk_status s = put_gguf_device(e, tid, l, tmp);
      if (s) {
        cudaFreeAsync(tmp, e->stream);
        return s;
      }
    }
  }
  cudaFreeAsync(tmp, e->stream);
  CK(cudaStreamSynchronize(e->stream));
  return SFK_OK;
}

sfk_status sfk_kv_reset(sfk_engine* e) {
  if (!e) return fail(SFK_ERR_INVALID_ARGUMENT, "null engine");
  CK(cudaSetDevice(e->device));
  const size_t kv_elem = e->hp.kv_type == SFK_KV_F16 ? 2 : 4;
  CK(cudaMemsetAsync(e->k_pool, 0, kv_elem * e->kv_layer_elems * e->hp.n_layer, e->stream));
  CK(cudaMemsetAsync(e->v_pool, 0, kv_elem * e->kv_layer_elems * e->hp.n_layer, e->stream));
  CK(cudaMemsetAsync(e->pos_state, 0, sizeof(int) * e->hp.max_batch, e->stream));
  CK(cudaStreamSynchronize(e->stream));
  std::fill(e->seq_pos.begin(), e->seq_pos.end(), 0);
  if (e->win.on) return window_table(e);
  return SFK_OK;
}

// full_logits: the caller reads this step's logits (otherwise an
// expert-parallel engine scores only its vocabulary slice and exchanges the
// argmax)
static sfk_status run_step(sfk_engine* e, int b, bool greedy, bool full_logits) {
  e->shard_now = e->head_shard && !full_logits;
  if (e->tier.on || e->win.on) {
    sfk_status s = run_step_direct(e, b, greedy);
    if (s) return s;
    e->steps += 1;
    e->last_b = b;
    return SFK_OK;
  }
  cudaGraphExec_t g = nullptr;
  sfk_status s = get_graph(e, b, greedy, &g);
  if (s) return s;
  CK(cudaGraphLaunch(g, e->stream));
  e->steps += 1;
  e->last_b = b;
  return SFK_OK;
}

sfk_status sfk_forward_batch(sfk_engine* e, int32_t n_seq, const int32_t* tokens, const int32_t* positions,
                             float* logits_host, int32_t* argmax_out) {
  if (!e || !tokens || !positions) return fail(SFK_ERR_INVALID_ARGUMENT, "null argument");
  if (n_seq < 1 || n_seq > e->hp.max_batch) return fail(SFK_ERR_INVALID_ARGUMENT, "n_seq %d", n_seq);
  for (int t = 0; t < n_seq; ++t) {
    if (positions[t] < 0 || positions[t] >= e->hp.n_ctx)
      return fail(SFK_ERR_INVALID_ARGUMENT, "position %d outside [0, n_ctx=%d)", positions[t], e->hp.n_ctx);
    if (tokens[t] < 0 || tokens[t] >= e->hp.n_vocab)
      return fail(SFK_ERR_INVALID_ARGUMENT, "token %d outside the vocabulary", tokens[t]);
  }
  CK(cudaSetDevice(e->device));
  // one upload of tokens | positions, the step, then the logits and keys |
  // status word into pinned memory and a single synchronisation
  const int B = e->hp.max_batch;
  memcpy(e->h_tok, tokens, sizeof(int) * n_seq);
  memcpy(e->h_pos, positions, sizeof(int) * n_seq);
  for (int t = 0; t < n_seq; ++t) e->step_pos[t] = positions[t];
  CK(cudaMemcpyAsync(e->tok_in, e->h_tok, sizeof(int) * 2 * B, cudaMemcpyHostToDevice, e->stream));
  sfk_status s = run_step(e, n_seq, false, logits_host != nullptr);
  if (s) return s;
  const size_t n_logits = (size_t)n_seq * e->hp.n_vocab;
  if (logits_host)
    CK(cudaMemcpyAsync(e->h_logits, e->logits, sizeof(float) * n_logits, cudaMemcpyDeviceToHost, e->stream));
  CK(cudaMemcpyAsync(e->h_keys, e->argmax_key, sizeof(unsigned long long) * B + sizeof(int), cudaMemcpyDeviceToHost,
                     e->stream));
  CK(cudaStreamSynchronize(e->stream));
  if ((s = status_result(e->status, *e->h_status))) {
    reset_counters(e);
    return s;
  }
  if (logits_host) memcpy(logits_host, e->h_logits, sizeof(float) * n_logits);
  for (int t = 0; t < n_seq; ++t) {
    e->seq_pos[t] = positions[t] + 1;
    if (argmax_out) argmax_out[t] = (int32_t)(0xFFFFFFFFu - (uint32_t)(e->h_keys[t] & 0xFFFFFFFFull));
  }
  return SFK_OK;
}

sfk_status sfk_forward(sfk_engine* e, int32_t token, int32_t pos, float* logits_host, int32_t* argmax_out) {
  return sfk_forward_batch(e, 1, &token, &pos, logits_host, argmax_out);
}

namespace {

constexpr int PF_CHUNK = 512;  // prompt tokens per prefill pass

sfk_status prefill_alloc(sfk_engine* e) {
  if (e->pf.cap) return SFK_OK;
  const sfk_hparams& hp = e->hp;
  const int C = std::min(PF_CHUNK, hp.n_ctx);
  const int d = hp.n_embd, F = hp.n_ff, E = hp.n_expert, k = hp.n_expert_used;
  const int np = C * k;
  const int mt = (np + TC_TT - 1) / TC_TT + std::min(E, np);
  const int rows_pad = mt * TC_TT, cpad = (C + TC_TT - 1) / TC_TT * TC_TT;
  const size_t act = std::max(std::max(tc_act_bytes(cpad, d), tc_act_bytes(cpad, e->nq)),
                              std::max(tc_act_bytes(rows_pad, d), tc_act_bytes(rows_pad, F)));
  sfk_engine::Prefill& f = e->pf;
  uint64_t* acct = &e->scratch_bytes;
  sfk_status s;
  if ((s = e->alloc(&f.tok, sizeof(int) * C, acct)) || (s = e->alloc(&f.pos, sizeof(int) * C, acct)) ||
      (s = e->alloc(&f.pt, sizeof(int) * (size_t)C * e->max_pages, acct)) ||
      (s = e->alloc(&f.x, sizeof(float) * (size_t)C * d, acct)) ||
      (s = e->alloc(&f.ffn, sizeof(float) * (size_t)C * d, acct)) ||
      (s = e->alloc(&f.xn, sizeof(float) * (size_t)C * d, acct)) ||
      (s = e->alloc(&f.qkv, sizeof(float) * (size_t)C * e->nqkv, acct)) ||
      (s = e->alloc(&f.q, sizeof(float) * (size_t)C * e->nq, acct)) ||
      (s = e->alloc(&f.att, sizeof(float) * (size_t)C * e->nq, acct)) ||
      (s = e->alloc(&f.h, sizeof(float) * (size_t)rows_pad * F, acct)) ||
      (s = e->alloc(&f.yd, sizeof(float) * (size_t)rows_pad * d, acct)) ||
      (s = e->alloc(&f.w, sizeof(float) * np, acct)) || (s = e->alloc(&f.act, act, acct)) ||
      (s = e->alloc(&f.xqd, (size_t)C * qact_bytes(d), acct)) || (s = e->alloc(&f.ids, sizeof(int) * np, acct)) ||
      (s = e->alloc(&f.pos_of_pair, sizeof(int) * np, acct)) ||
      (s = e->alloc(&f.rows_tok, sizeof(int) * rows_pad, acct)) ||
      (s = e->alloc(&f.rows_self, sizeof(int) * rows_pad, acct)) ||
      (s = e->alloc(&f.tile_expert, sizeof(int) * mt, acct)))
    return s;
  // bounded tier: the down GEMM's activations apart from gate/up's, which
  // every pass over the experts reads again
  if (e->tier.on && (s = e->alloc(&f.act_dn, tc_act_bytes(rows_pad, F), acct))) return s;
  if (pf_attn_supported(e->hd, e->hq_loc, e->hkv_loc)) {
    // score rows of a whole chunk at the longest context, at most 256 MB
    // (longer contexts run the attention in token sub-batches of whole tiles)
    const int qt = 64 / (e->hq_loc / e->hkv_loc);
    const size_t want = pf_attn_scratch_bytes(C, hp.n_ctx - C, e->hq_loc, e->hkv_loc);
    const size_t cap = std::max((size_t)256 << 20, pf_attn_scratch_bytes(qt, hp.n_ctx - qt, e->hq_loc, e->hkv_loc));
    f.score_bytes = std::min(want, cap);
    if ((s = e->alloc(&f.score, f.score_bytes, acct))) return s;
  }
  f.cap = C;
  f.mt = mt;
  return SFK_OK;
}

// One layer over m prompt tokens at positions pos0 .. pos0 + m - 1 of
// sequence `seq`: the reference's per-token layer (engine.cpp:1878-1986) with
// the matrices as tensor-core GEMMs over all m tokens (the routed experts
// grouped by expert) and the attention of every token over its own prefix.
// Bounded tier: the routed gate/up and down GEMMs of a prefill chunk, in
// passes over as many of the chunk's experts as the pool can hold at once.
// Each expert tile is computed exactly as in one pass (tiles are
// independent); a pass's GEMMs see only its own tiles (the others are marked
// -1), and the next pass may reuse the slots once the stream has drained.
sfk_status tier_prefill_experts(sfk_engine* e, int l, int m) {
  const sfk_hparams& hp = e->hp;
  sfk_engine::Prefill& f = e->pf;
  sfk_engine::Tier& T = e->tier;
  cudaStream_t st = e->stream;
  const int d = hp.n_embd, F = hp.n_ff, E = hp.n_expert, k = hp.n_expert_used;
  const int act_gu = act_for(hp.type_ffn_gu), act_dn = act_for(hp.type_ffn_down);
  CK(cudaMemcpyAsync(T.h_tile, f.tile_expert, sizeof(int) * f.mt, cudaMemcpyDeviceToHost, st));
  CK(cudaMemcpyAsync(T.h_ids, f.ids, sizeof(int) * m * k, cudaMemcpyDeviceToHost, st));
  CK(cudaStreamSynchronize(st));
  T.sp->unpin_all();
  std::vector<int> tile(T.h_tile, T.h_tile + f.mt), order;
  for (int i = 0; i < m * k; ++i) {
    if (T.h_ids[i] < 0 || T.h_ids[i] >= E) return fail(SFK_ERR_RUNTIME, "layer %d: routed expert %d", l, T.h_ids[i]);
    T.pred->observe((uint32_t)l, (uint32_t)T.h_ids[i]);
  }
  // the experts in order of their first routed pair (the reference acquires
  // them token by token)
  std::vector<char> seen(E, 0);
  for (int i = 0; i < m * k; ++i)
    if (!seen[T.h_ids[i]]) {
      seen[T.h_ids[i]] = 1;
      order.push_back(T.h_ids[i]);
    }
  std::vector<int> slot_of(E, -1);
  size_t next = 0;
  while (next < order.size()) {
    std::fill(slot_of.begin(), slot_of.end(), -1);
    size_t taken = 0;
    for (; next < order.size(); ++next, ++taken) {
      uint32_t slot = 0;
      sfk_status s = tier_acquire(e, l, order[next], true, &slot);
      if (s) return s;
      if (slot == SlotPool::NONE) break;
      slot_of[order[next]] = (int)slot;
    }
    if (taken == 0) return fail(SFK_ERR_RUNTIME, "layer %d: no free expert slot", l);
    for (int t = 0; t < f.mt; ++t) T.h_tile[t] = tile[t] >= 0 && tile[t] < E ? slot_of[tile[t]] : -1;
    CK(cudaMemcpyAsync(T.d_tile, T.h_tile, sizeof(int) * f.mt, cudaMemcpyHostToDevice, st));
    sfk_status s = tier_fence(e);
    if (s) return s;
    TcGemmParams g{};
    g.w = T.pool;
    g.w2 = T.pool + T.off_up;
    g.rowstride = dev_row_bytes(hp.type_ffn_gu, d);
    g.expert_stride = T.slot_bytes;
    g.rows = F;
    g.K = d;
    g.wtype = hp.type_ffn_gu;
    g.act_type = act_gu;
    g.xq = f.act;
    g.ntile = f.mt;
    g.tile_expert = T.d_tile;
    g.y = f.h;
    g.ldy = F;
    g.epi = TC_EPI_SWIGLU;
    g.status = e->status;
    CK(launch_tc_gemm(g, st));
    CK(launch_tc_quant(act_dn, f.h, F, f.rows_self, f.mt * TC_TT, f.mt * TC_TT, F, f.act_dn, st));
    g = TcGemmParams{};
    g.w = T.pool + T.off_down;
    g.rowstride = dev_row_bytes(hp.type_ffn_down, F);
    g.expert_stride = T.slot_bytes;
    g.rows = d;
    g.K = F;
    g.wtype = hp.type_ffn_down;
    g.act_type = act_dn;
    g.xq = f.act_dn;
    g.ntile = f.mt;
    g.tile_expert = T.d_tile;
    g.y = f.yd;
    g.ldy = d;
    g.epi = TC_EPI_STORE;
    g.status = e->status;
    CK(launch_tc_gemm(g, st));
    if (next < order.size()) {  // the next pass may take these slots back
      CK(cudaStreamSynchronize(st));
      T.sp->unpin_all();
    }
  }
  return SFK_OK;
}

sfk_status prefill_layer(sfk_engine* e, int l, int seq, int m, int pos0) {
  const sfk_hparams& hp = e->hp;
  const LayerW& W = e->L[l];
  sfk_engine::Prefill& f = e->pf;
  cudaStream_t st = e->stream;
  const int d = hp.n_embd, F = hp.n_ff, E = hp.n_expert, k = hp.n_expert_used;
  const int mpad = (m + TC_TT - 1) / TC_TT * TC_TT;
  const int act_attn = act_for(hp.type_attn);
  if (e->win.on) {  // this layer's cold pages of the sequence, for its attention (in stream order)
    bool staged = false;
    sfk_status s = window_stage(e, l, seq, seq + 1, st, &staged);
    if (s) return s;
  }
  // attn_norm -> QKV (engine.cpp:1878-1889)
  CK(launch_pf_norm(f.x, W.attn_norm, m, d, hp.rms_eps, f.xn, st));
  CK(launch_tc_quant(act_attn, f.xn, d, nullptr, m, mpad, d, f.act, st));
  TcGemmParams g{};
  g.w = W.qkv;
  g.rowstride = dev_row_bytes(hp.type_attn, d);
  g.rows = e->nqkv;
  g.K = d;
  g.wtype = hp.type_attn;
  g.act_type = act_attn;
  g.xq = f.act;
  g.n = m;
  g.ntile = mpad / TC_TT;
  g.y = f.qkv;
  g.ldy = e->nqkv;
  g.epi = TC_EPI_STORE;
  g.status = e->status;
  CK(launch_tc_gemm(g, st));
  // RoPE, KV append (engine.cpp:1892-1901,1646-1656)
  KvView kv = kv_view(e, l);
  const int* pt_row = e->page_table + (size_t)seq * e->max_pages;
  CK(launch_pf_rope_kv(f.qkv, m, e->hq_loc, kv, pt_row, e->rope, pos0, f.q, e->status, st));
  // attention of token t over positions 0 .. pos0 + t (engine.cpp:1751-1761)
  if (f.score) {
    // token sub-batches (whole 64-row tiles) whose score rows fit the scratch
    const int qt = 64 / (e->hq_loc / e->hkv_loc);
    const size_t tile_bytes = pf_attn_scratch_bytes(qt, pos0 + m - qt, e->hq_loc, e->hkv_loc);
    const int step = std::max(1, (int)(f.score_bytes / tile_bytes)) * qt;
    for (int c = 0; c < m; c += step) {
      const int mc = std::min(step, m - c);
      CK(launch_pf_attn(f.q + (size_t)c * e->nq, kv, pt_row, mc, pos0 + c, e->hq_loc, f.att + (size_t)c * e->nq,
                        f.score, e->status, st));
    }
  } else {  // other head shapes: the decode kernel, one page-table row per prompt token
    AttnParams a{};
    a.q = f.q;
    a.kv = kv;
    a.kv.page_table = f.pt;
    a.pos = f.pos;
    a.b = m;
    a.n_head = e->hq_loc;
    a.cluster = e->attn_cluster;
    a.max_chunk = e->attn_max_chunk;
    a.out = f.att;
    a.status = e->status;
    CK(launch_attn(a, st, false));
  }
  // O projection + residual (engine.cpp:1905-1906)
  CK(launch_tc_quant(act_attn, f.att, e->nq, nullptr, m, mpad, e->nq, f.act, st));
  g = TcGemmParams{};
  g.w = W.wo;
  g.rowstride = dev_row_bytes(hp.type_attn, e->nq);
  g.rows = d;
  g.K = e->nq;
  g.wtype = hp.type_attn;
  g.act_type = act_attn;
  g.xq = f.act;
  g.n = m;
  g.ntile = mpad / TC_TT;
  g.y = f.ffn;
  g.ldy = d;
  g.res = f.x;
  g.ldres = d;
  g.epi = TC_EPI_RESID;
  g.status = e->status;
  CK(launch_tc_gemm(g, st));
  // ffn_norm, router, top-k (engine.cpp:1909-1924); pairs grouped by expert
  const int act_gu = act_for(hp.type_ffn_gu), act_dn = act_for(hp.type_ffn_down);
  CK(launch_pf_route(f.ffn, W.ffn_norm, W.router, m, d, E, k, hp.rms_eps, act_gu, f.xqd, f.xn, f.ids, f.w, e->status,
                     st));
  CK(launch_pf_group(f.ids, m * k, k, E, f.mt, f.pos_of_pair, f.rows_tok, f.rows_self, f.tile_expert, e->status, st));
  // gate / up + SwiGLU of every routed pair (engine.cpp:1967-1969)
  CK(launch_tc_quant(act_gu, f.xn, d, f.rows_tok, m, f.mt * TC_TT, d, f.act, st));
  if (e->tier.on) {
    sfk_status s = tier_prefill_experts(e, l, m);
    if (s) return s;
    CK(launch_pf_combine(f.yd, f.pos_of_pair, f.w, k, m, d, f.ffn, f.x, st));
    return SFK_OK;
  }
  g = TcGemmParams{};
  g.w = W.gate;
  g.w2 = W.up;
  g.rowstride = dev_row_bytes(hp.type_ffn_gu, d);
  g.expert_stride = (int64_t)F * g.rowstride;
  g.rows = F;
  g.K = d;
  g.wtype = hp.type_ffn_gu;
  g.act_type = act_gu;
  g.xq = f.act;
  g.ntile = f.mt;
  g.tile_expert = f.tile_expert;
  g.y = f.h;
  g.ldy = F;
  g.epi = TC_EPI_SWIGLU;
  g.status = e->status;
  CK(launch_tc_gemm(g, st));
  // down of every routed pair, then the weighted combine + residual
  // (engine.cpp:1970-1986)
  CK(launch_tc_quant(act_dn, f.h, F, f.rows_self, f.mt * TC_TT, f.mt * TC_TT, F, f.act, st));
  g = TcGemmParams{};
  g.w = W.down;
  g.rowstride = dev_row_bytes(hp.type_ffn_down, F);
  g.expert_stride = (int64_t)d * g.rowstride;
  g.rows = d;
  g.K = F;
  g.wtype = hp.type_ffn_down;
  g.act_type = act_dn;
  g.xq = f.act;
  g.ntile = f.mt;
  g.tile_expert = f.tile_expert;
  g.y = f.yd;
  g.ldy = d;
  g.epi = TC_EPI_STORE;
  g.status = e->status;
  CK(launch_tc_gemm(g, st));
  CK(launch_pf_combine(f.yd, f.pos_of_pair, f.w, k, m, d, f.ffn, f.x, st));
  return SFK_OK;
}

// output_norm + lm_head + argmax of one hidden row into sequence seq's logits
// row and argmax key (engine.cpp:2988-3006)
sfk_status lmhead_row(sfk_engine* e, const float* x_row, int seq) {
  const sfk_hparams& hp = e->hp;
  CK(cudaMemsetAsync(e->argmax_key + seq, 0, sizeof(unsigned long long), e->stream));
  StreamParams p{};
  p.w0 = e->output;
  p.rowstride = dev_row_bytes(hp.type_output, hp.n_embd);
  p.rows = hp.n_vocab;
  p.K = hp.n_embd;
  p.wtype = hp.type_output;
  p.nmat = 1;
  p.act_type = act_for(hp.type_output);
  p.row_align = 1;
  p.b = 1; p.k = 1; p.n_pairs = 1; p.n_vec = 1;
  p.pro = PRO_QUANT;
  p.x = x_row;
  p.norm_w = e->out_norm;
  p.eps = hp.rms_eps;
  p.epi = EPI_LMHEAD;
  p.y = e->logits + (size_t)seq * hp.n_vocab;
  p.y_stride = hp.n_vocab;
  p.argmax_key = e->argmax_key + seq;
  p.store_logits = 1;
  p.status = e->status;
  int grid = 0;
  sfk_status s = plan_stream(p, e->sm_count, &grid);
  if (s) return s;
  CK(launch_stream(p, grid, e->stream, false));
  return SFK_OK;
}

}  // namespace

sfk_status sfk_prefill(sfk_engine* e, int32_t seq, const int32_t* tokens, int32_t n, int32_t pos0, float* logits_host,
                       int32_t* argmax_out) {
  if (!e || !tokens) return fail(SFK_ERR_INVALID_ARGUMENT, "null argument");
  const sfk_hparams& hp = e->hp;
  if (seq < 0 || seq >= hp.max_batch) return fail(SFK_ERR_INVALID_ARGUMENT, "sequence %d", seq);
  if (n < 1 || pos0 < 0 || (int64_t)pos0 + n > hp.n_ctx)
    return fail(SFK_ERR_INVALID_ARGUMENT, "positions [%d, %d) outside [0, n_ctx=%d)", pos0, pos0 + n, hp.n_ctx);
  for (int i = 0; i < n; ++i)
    if (tokens[i] < 0 || tokens[i] >= hp.n_vocab)
      return fail(SFK_ERR_INVALID_ARGUMENT, "token %d outside the vocabulary", tokens[i]);
  if (e->ep_size > 1) return fail(SFK_ERR_UNSUPPORTED, "batched prefill runs on one GPU (no expert parallelism)");
  CK(cudaSetDevice(e->device));
  sfk_status s = prefill_alloc(e);
  if (s) return s;
  sfk_engine::Prefill& f = e->pf;
  // with a KV window a chunk spans at most the window's pages, all written
  // in HBM; the pages before them are evicted first
  const int cap = e->win.on ? std::min(f.cap, (e->win.pages - 1) * 16) : f.cap;
  for (int c0 = 0; c0 < n; c0 += cap) {
    const int m = std::min(cap, n - c0);
    if (e->win.on) {
      if ((pos0 + c0) / 16 < e->win.cold[seq])
        return fail(SFK_ERR_INVALID_ARGUMENT, "sequence %d: position %d lies in a page that has left the KV window",
                    seq, pos0 + c0);
      if ((s = window_advance(e, seq, pos0 + c0 + m - 1))) return s;
    }
    CK(cudaMemcpyAsync(f.tok, tokens + c0, sizeof(int) * m, cudaMemcpyHostToDevice, e->stream));
    CK(launch_pf_embed(e->tok_embd, hp.type_embd, hp.n_embd, hp.n_vocab, f.tok, m, pos0 + c0, f.x, f.pos,
                       e->pos_state + seq, e->status, e->stream));
    CK(launch_pf_pt(e->page_table + (size_t)seq * e->max_pages, e->max_pages, m, f.pt, e->stream));
    for (int l = 0; l < hp.n_layer; ++l)
      if ((s = prefill_layer(e, l, seq, m, pos0 + c0))) return s;
    if (c0 + m == n && (s = lmhead_row(e, f.x + (size_t)(m - 1) * hp.n_embd, seq))) return s;
  }
  const int B = hp.max_batch;
  if (logits_host)
    CK(cudaMemcpyAsync(e->h_logits, e->logits + (size_t)seq * hp.n_vocab, sizeof(float) * hp.n_vocab,
                       cudaMemcpyDeviceToHost, e->stream));
  CK(cudaMemcpyAsync(e->h_keys, e->argmax_key, sizeof(unsigned long long) * B + sizeof(int), cudaMemcpyDeviceToHost,
                     e->stream));
  CK(cudaStreamSynchronize(e->stream));
  if ((s = status_result(e->status, *e->h_status))) {
    reset_counters(e);
    return s;
  }
  if (logits_host) memcpy(logits_host, e->h_logits, sizeof(float) * hp.n_vocab);
  if (argmax_out) *argmax_out = (int32_t)(0xFFFFFFFFu - (uint32_t)(e->h_keys[seq] & 0xFFFFFFFFull));
  e->seq_pos[seq] = pos0 + n;
  return SFK_OK;
}

sfk_sampling sfk_sampling_defaults(void) {
  sfk_sampling s{};
  s.temperature = 0.0f;
  s.top_p = 1.0f;
  s.top_k = 0;
  s.seed = 0;
  s.max_tokens = 256;
  s.eos_token = -1;
  return s;
}

sfk_status sfk_generate(sfk_engine* e, const int32_t* prompt, int32_t n_prompt, const sfk_sampling* sampling,
                        int32_t* tokens_out, int32_t cap_out, int32_t* n_out, sfk_token_cb cb, void* user) {
  if (!e || !prompt || !n_out) return fail(SFK_ERR_INVALID_ARGUMENT, "null argument");
  if (n_prompt < 1) return fail(SFK_ERR_INVALID_ARGUMENT, "empty prompt");
  if (tokens_out && cap_out < 0) return fail(SFK_ERR_INVALID_ARGUMENT, "cap_out");
  const sfk_sampling sp = sampling ? *sampling : sfk_sampling_defaults();
  const sfk_hparams& hp = e->hp;
  *n_out = 0;
  const int pos0 = e->seq_pos[0];
  if ((int64_t)pos0 + n_prompt > hp.n_ctx)
    return fail(SFK_ERR_INVALID_ARGUMENT, "prompt of %d tokens at position %d exceeds n_ctx=%d", n_prompt, pos0,
                hp.n_ctx);
  const bool greedy = !(sp.temperature > 0.0f);
  if (!greedy && !e->sample_p) {
    sfk_status s;
    if ((s = e->alloc(&e->sample_p, sizeof(float) * hp.n_vocab, &e->scratch_bytes)) ||
        (s = e->alloc(&e->sample_tok, sizeof(int), &e->scratch_bytes)))
      return s;
  }
  int32_t am = 0;
  sfk_status s = sfk_prefill(e, 0, prompt, n_prompt, pos0, nullptr, &am);
  if (s) return s;
  int limit = sp.max_tokens > 0 ? sp.max_tokens : 256;
  if (tokens_out) limit = std::min(limit, cap_out);
  SampleArgs a{};
  a.temperature = sp.temperature;
  a.top_p = sp.top_p;
  a.top_k = sp.top_k;
  a.seed = sp.seed;
  int n = 0;
  for (int i = 0; i < limit; ++i) {
    // the token after the last forward: its argmax, or a sample of its logits
    // written over the argmax key (the next step's input either way)
    int32_t tok = 0;
    if (greedy) {
      unsigned long long key = 0;
      CK(cudaMemcpyAsync(&key, e->argmax_key, sizeof(key), cudaMemcpyDeviceToHost, e->stream));
      CK(cudaStreamSynchronize(e->stream));
      tok = (int32_t)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
    } else {
      CK(launch_sample(e->logits, hp.n_vocab, a, i, e->sample_p, e->argmax_key, e->sample_tok, e->stream));
      CK(cudaMemcpyAsync(&tok, e->sample_tok, sizeof(int), cudaMemcpyDeviceToHost, e->stream));
      CK(cudaStreamSynchronize(e->stream));
    }
    if (tok == sp.eos_token) break;
    if (tok < 0 || tok >= hp.n_vocab) return fail(SFK_ERR_RUNTIME, "sampled token %d outside the vocabulary", tok);
    if (tokens_out) tokens_out[n] = tok;
    ++n;
    if (cb && cb(tok, user) != 0) break;
    if (i + 1 == limit || e->seq_pos[0] + 1 > hp.n_ctx) break;
    // one decode step on the token (device greedy-loop form: the key holds it)
    e->step_pos[0] = e->seq_pos[0];
    if ((s = run_step(e, 1, true, true))) return s;
    if ((s = engine_check(e))) return s;
    e->seq_pos[0] += 1;
  }
  *n_out = n;
  return SFK_OK;
}

sfk_status sfk_decode_greedy(sfk_engine* e, int32_t n_seq, int32_t n_steps, int32_t* tokens_out) {
  if (!e) return fail(SFK_ERR_INVALID_ARGUMENT, "null engine");
  if (n_seq < 1 || n_seq > e->hp.max_batch || n_steps < 0) return fail(SFK_ERR_INVALID_ARGUMENT, "n_seq / n_steps");
  for (int t = 0; t < n_seq; ++t)
    if (e->seq_pos[t] + n_steps > e->hp.n_ctx)
      return fail(SFK_ERR_INVALID_ARGUMENT, "sequence %d would exceed n_ctx", t);
  CK(cudaSetDevice(e->device));
  for (int i = 0; i < n_steps; ++i) {
    for (int t = 0; t < n_seq; ++t) e->step_pos[t] = e->seq_pos[t] + i;
    sfk_status s = run_step(e, n_seq, true, false);
    if (s) return s;
    if (tokens_out) {
      // token consumed by this step = previous argmax
      CK(cudaMemcpyAsync(tokens_out + (int64_t)i * n_seq, e->tok_hist, sizeof(int) * n_seq, cudaMemcpyDeviceToHost,
                         e->stream));
    }
  }
  sfk_status s = engine_check(e);
  if (s) return s;
  for (int t = 0; t < n_seq; ++t) e->seq_pos[t] += n_steps;
  return SFK_OK;
}

sfk_status sfk_route_get(sfk_engine* e, int32_t* ids_out, float* w_out, size_t n) {
  if (!e || !ids_out || !w_out) return fail(SFK_ERR_INVALID_ARGUMENT, "null argument");
  const size_t np = (size_t)std::max(1, e->last_b) * e->hp.n_expert_used;
  if (n < np) return fail(SFK_ERR_INVALID_ARGUMENT, "need %zu entries", np);
  CK(cudaSetDevice(e->device));
  CK(cudaMemcpyAsync(ids_out, e->route->ids, np * sizeof(int), cudaMemcpyDeviceToHost, e->stream));
  CK(cudaMemcpyAsync(w_out, e->route->w, np * sizeof(float), cudaMemcpyDeviceToHost, e->stream));
  CK(cudaStreamSynchronize(e->stream));
  return SFK_OK;
}

sfk_status sfk_debug_get(sfk_engine* e, int32_t which, float* host_out, size_t n_floats) {
  if (!e || !host_out) return fail(SFK_ERR_INVALID_ARGUMENT, "null argument");
  const size_t b = (size_t)std::max(1, e->last_b);
  const float* src = nullptr;
  size_t n = 0;
  switch (which) {
    case 0: src = e->attn_out; n = b * e->nq; break;
    case 1: src = e->ffn_inp; n = b * e->hp.n_embd; break;
    case 2: src = e->q; n = b * e->nq; break;
    case 3: src = e->h; n = b * e->hp.n_expert_used * e->hp.n_ff; break;
    default: return fail(SFK_ERR_INVALID_ARGUMENT, "unknown buffer %d", which);
  }
  if (n_floats < n) return fail(SFK_ERR_INVALID_ARGUMENT, "need %zu floats", n);
  CK(cudaSetDevice(e->device));
  CK(cudaMemcpyAsync(host_out, src, n * sizeof(float), cudaMemcpyDeviceToHost, e->stream));
  CK(cudaStreamSynchronize(e->stream));
  return SFK_OK;
}

// ---- per-layer entry points ---------------------------------------------------
static sfk_status layer_call_check(sfk_engine* e, int32_t n_tok, const void* hidden) {
  if (!e || !hidden) return fail(SFK_ERR_INVALID_ARGUMENT, "null argument");
  if (n_tok < 1 || n_tok > e->hp.max_batch) return fail(SFK_ERR_INVALID_ARGUMENT, "n_tok %d", n_tok);
  if (e->ep_size > 1) return fail(SFK_ERR_UNSUPPORTED, "per-layer calls run on single-GPU engines");
  CK(cudaSetDevice(e->device));
  return SFK_OK;
}

// tokens / positions into the step's device inputs (and the host mirror the
// KV window reads)
static sfk_status layer_positions(sfk_engine* e, const int32_t* positions, int32_t n_tok) {
  for (int t = 0; t < n_tok; ++t)
    if (positions[t] < 0 || positions[t] >= e->hp.n_ctx)
      return fail(SFK_ERR_INVALID_ARGUMENT, "position %d outside [0, n_ctx=%d)", positions[t], e->hp.n_ctx);
  memcpy(e->h_pos, positions, sizeof(int) * n_tok);
  for (int t = 0; t < n_tok; ++t) e->step_pos[t] = positions[t];
  return SFK_OK;
}

sfk_status sfk_embed(sfk_engine* e, const int32_t* tokens, const int32_t* positions, int32_t n_tok, float* hidden) {
  sfk_status s = layer_call_check(e, n_tok, hidden);
  if (s) return s;
  if (!tokens || !positions) return fail(SFK_ERR_INVALID_ARGUMENT, "null argument");
  for (int t = 0; t < n_tok; ++t)
    if (tokens[t] < 0 || tokens[t] >= e->hp.n_vocab)
      return fail(SFK_ERR_INVALID_ARGUMENT, "token %d outside the vocabulary", tokens[t]);
  if ((s = layer_positions(e, positions, n_tok))) return s;
  memcpy(e->h_tok, tokens, sizeof(int) * n_tok);
  const int B = e->hp.max_batch;
  CK(cudaMemcpyAsync(e->tok_in, e->h_tok, sizeof(int) * 2 * B, cudaMemcpyHostToDevice, e->stream));
  if ((s = launch_one(e, K_EMBED, 0, n_tok, false, false))) return s;
  CK(cudaMemcpyAsync(hidden, e->x, sizeof(float) * n_tok * e->hp.n_embd, cudaMemcpyDeviceToDevice, e->stream));
  return engine_check(e);
}

sfk_status sfk_decode_layer_attn(sfk_engine* e, int32_t layer, const int32_t* positions, int32_t n_tok,
                                 float* hidden) {
  sfk_status s = layer_call_check(e, n_tok, hidden);
  if (s) return s;
  if (!positions || layer < 0 || layer >= e->hp.n_layer) return fail(SFK_ERR_INVALID_ARGUMENT, "layer %d", layer);
  if ((s = layer_positions(e, positions, n_tok))) return s;
  const int B = e->hp.max_batch, d = e->hp.n_embd;
  // positions as the embedding kernel leaves them (pos_cur), then the layer
  CK(cudaMemcpyAsync(e->pos_in, e->h_pos, sizeof(int) * B, cudaMemcpyHostToDevice, e->stream));
  CK(cudaMemcpyAsync(e->pos_cur, e->pos_in, sizeof(int) * n_tok, cudaMemcpyDeviceToDevice, e->stream));
  CK(cudaMemcpyAsync(e->x, hidden, sizeof(float) * n_tok * d, cudaMemcpyDeviceToDevice, e->stream));
  if (e->win.on) {
    for (int t = 0; t < n_tok && !s; ++t) s = window_advance(e, t, positions[t]);
    bool staged = false;
    if (!s) s = window_stage(e, layer, 0, n_tok, e->stream, &staged);
    if (s) return s;
  }
  for (int c = K_QKV; c <= K_OPROJ && !s; ++c) s = launch_one(e, c, layer, n_tok, false, c != K_QKV);
  if (s) return s;
  CK(cudaMemcpyAsync(hidden, e->ffn_inp, sizeof(float) * n_tok * d, cudaMemcpyDeviceToDevice, e->stream));
  if ((s = engine_check(e))) return s;
  for (int t = 0; t < n_tok; ++t) e->seq_pos[t] = std::max(e->seq_pos[t], positions[t] + 1);
  e->last_b = n_tok;
  return SFK_OK;
}

sfk_status sfk_decode_layer_moe(sfk_engine* e, int32_t layer, int32_t n_tok, float* hidden, int32_t* ids_out,
                                float* w_out) {
  sfk_status s = layer_call_check(e, n_tok, hidden);
  if (s) return s;
  if (layer < 0 || layer >= e->hp.n_layer) return fail(SFK_ERR_INVALID_ARGUMENT, "layer %d", layer);
  const int d = e->hp.n_embd, k = e->hp.n_expert_used;
  CK(cudaMemcpyAsync(e->ffn_inp, hidden, sizeof(float) * n_tok * d, cudaMemcpyDeviceToDevice, e->stream));
  if (!route_fused(e, n_tok)) s = launch_one(e, K_ROUTER, layer, n_tok, false, false);
  if (!s && e->tier.on) {
    e->tier.warmed_now.clear();
    s = tier_route_layer(e, layer, n_tok);
  }
  if (!s) s = launch_one(e, K_GATEUP, layer, n_tok, false, false);
  if (!s) s = launch_one(e, K_DOWN, layer, n_tok, false, true);
  if (!s && e->tier.on) s = tier_prefetch(e, layer + 1);
  if (s) return s;
  CK(cudaMemcpyAsync(hidden, e->x, sizeof(float) * n_tok * d, cudaMemcpyDeviceToDevice, e->stream));
  if (ids_out)
    CK(cudaMemcpyAsync(ids_out, reinterpret_cast<const uint8_t*>(e->route) + offsetof(Route, ids),
                       sizeof(int) * n_tok * k, cudaMemcpyDeviceToDevice, e->stream));
  if (w_out)
    CK(cudaMemcpyAsync(w_out, reinterpret_cast<const uint8_t*>(e->route) + offsetof(Route, w),
                       sizeof(float) * n_tok * k, cudaMemcpyDeviceToDevice, e->stream));
  e->last_b = n_tok;
  return engine_check(e);
}

sfk_status sfk_lm_head(sfk_engine* e, const float* hidden, int32_t n_tok, float* logits_out, int32_t* argmax_out) {
  sfk_status s = layer_call_check(e, n_tok, hidden);
  if (s) return s;
  const int B = e->hp.max_batch, V = e->hp.n_vocab;
  CK(cudaMemcpyAsync(e->x, hidden, sizeof(float) * n_tok * e->hp.n_embd, cudaMemcpyDeviceToDevice, e->stream));
  CK(cudaMemsetAsync(e->argmax_key, 0, sizeof(unsigned long long) * n_tok, e->stream));
  if ((s = launch_one(e, K_LMHEAD, 0, n_tok, false, false))) return s;
  if (logits_out)
    CK(cudaMemcpyAsync(logits_out, e->logits, sizeof(float) * n_tok * V, cudaMemcpyDeviceToDevice, e->stream));
  CK(cudaMemcpyAsync(e->h_keys, e->argmax_key, sizeof(unsigned long long) * B + sizeof(int), cudaMemcpyDeviceToHost,
                     e->stream));
  CK(cudaStreamSynchronize(e->stream));
  if ((s = status_result(e->status, *e->h_status))) {
    reset_counters(e);
    return s;
  }
  if (argmax_out)
    for (int t = 0; t < n_tok; ++t)
      argmax_out[t] = (int32_t)(0xFFFFFFFFu - (uint32_t)(e->h_keys[t] & 0xFFFFFFFFull));
  return SFK_OK;
}

sfk_status sfk_hidden_get(sfk_engine* e, float* host_out, size_t n_floats) {
  if (!e || !host_out) return fail(SFK_ERR_INVALID_ARGUMENT, "null argument");
  const size_t n = (size_t)std::max(1, e->last_b) * e->hp.n_embd;
  if (n_floats < n) return fail(SFK_ERR_INVALID_ARGUMENT, "need %zu floats", n);
  CK(cudaSetDevice(e->device));
  CK(cudaMemcpyAsync(host_out, e->x, n * sizeof(float), cudaMemcpyDeviceToHost, e->stream));
  CK(cudaStreamSynchronize(e->stream));
  return SFK_OK;
}

}  // extern "C"

namespace sfk {
// This engine's share of a sharded model (library-internal, for the .strata
// loader): the head split (query heads [q0, q0 + hq_loc), kv heads
// [kv0, kv0 + hkv_loc), head width hd) and the local experts [e0, e0 + e_loc).
void engine_shard(const sfk_engine* e, EngineShard* out) {
  out->head_split = e->head_par ? 1 : 0;
  out->q0 = e->q0;
  out->hq_loc = e->hq_loc;
  out->kv0 = e->kv0;
  out->hkv_loc = e->hkv_loc;
  out->hd = e->hd;
  out->e0 = e->e0;
  out->e_loc = e->e_loc;
}
}  // namespace sfk

extern "C" {

sfk_status sfk_get_stats(const sfk_engine* e, sfk_stats* out) {
  if (!e || !out) return fail(SFK_ERR_INVALID_ARGUMENT, "null argument");
  const sfk_hparams& hp = e->hp;
  out->weight_bytes_hbm = e->weight_bytes;
  out->kv_bytes_hbm = e->kv_bytes;
  out->scratch_bytes_hbm = e->scratch_bytes;
  out->steps = e->steps;
  out->kernels_per_step = e->kernels_per_step;
  const uint64_t d = hp.n_embd, F = hp.n_ff;
  uint64_t per_layer = (uint64_t)dev_gguf_row_bytes(hp.type_attn, d) * e->nqkv +
                       (uint64_t)dev_gguf_row_bytes(hp.type_attn, e->nq) * d + 4ull * d * hp.n_expert +
                       (uint64_t)hp.n_expert_used * (2ull * dev_gguf_row_bytes(hp.type_ffn_gu, d) * F +
                                                     (uint64_t)dev_gguf_row_bytes(hp.type_ffn_down, F) * d);
  out->active_bytes_per_token = per_layer * hp.n_layer + (uint64_t)dev_gguf_row_bytes(hp.type_output, d) * hp.n_vocab;
  const sfk_engine::Tier& T = e->tier;
  out->pool_slots = T.on ? T.n_slots : 0;
  out->pool_hits = T.on ? T.sp->stats().hits : 0;
  out->pool_misses = T.on ? T.sp->stats().misses : 0;
  out->pool_evictions = T.on ? T.sp->stats().evictions : 0;
  out->h2d_expert_bytes = T.h2d;
  out->prefetch_warmed = T.warmed;
  out->prefetch_used = T.used;
  out->kv_window_pages = e->win.on ? (uint64_t)e->win.pages : 0;
  out->kv_pages_evicted = e->win.evicted;
  out->kv_staged_bytes = e->win.staged_bytes;
  return SFK_OK;
}

sfk_status sfk_time_kernels(sfk_engine* e, int32_t n_seq, int32_t iters, float* ms_out, int32_t n_out) {
  if (!e || !ms_out || n_out < K_NCLASS || iters < 1 || n_seq < 1 || n_seq > e->hp.max_batch)
    return fail(SFK_ERR_INVALID_ARGUMENT, "time_kernels arguments");
  if (e->steps == 0) return fail(SFK_ERR_INVALID_ARGUMENT, "run a decode step first");
  if (e->tier.on || e->win.on)
    return fail(SFK_ERR_UNSUPPORTED, "per-kernel timing needs every expert and the whole KV resident");
  e->shard_now = false;  // the whole lm_head, as the replicated engine runs it
  CK(cudaSetDevice(e->device));
  cudaEvent_t a = nullptr, z = nullptr;
  CK(cudaEventCreate(&a));
  CK(cudaEventCreate(&z));
  sfk_status s = SFK_OK;
  for (int c = 0; c < K_NCLASS && !s; ++c) {
    // greedy-mode embed would advance positions; time it in host-token mode
    CK(cudaEventRecord(a, e->stream));
    for (int i = 0; i < iters && !s; ++i) s = launch_one(e, c, i % e->hp.n_layer, n_seq, false, false);
    CK(cudaEventRecord(z, e->stream));
    CK(cudaEventSynchronize(z));
    float ms = 0.0f;
    CK(cudaEventElapsedTime(&ms, a, z));
    ms_out[c] = (c == K_ROUTER && route_fused(e, n_seq)) ? 0.0f : ms / iters;  // routing is inside gate/up
  }
  cudaEventDestroy(a);
  cudaEventDestroy(z);
  if (s) return s;
  return engine_check(e);
}

sfk_status sfk_ep_handle(sfk_engine* e, void* handle_out, size_t n_bytes) {
  if (!e || !handle_out) return fail(SFK_ERR_INVALID_ARGUMENT, "null argument");
  if (e->ep_size <= 1) return fail(SFK_ERR_INVALID_ARGUMENT, "engine is not expert-parallel");
  if (n_bytes < sizeof(cudaIpcMemHandle_t) || n_bytes < SFK_EP_HANDLE_BYTES)
    return fail(SFK_ERR_INVALID_ARGUMENT, "handle buffer of %zu bytes", n_bytes);
  CK(cudaSetDevice(e->device));
  cudaIpcMemHandle_t h;
  CK(cudaIpcGetMemHandle(&h, e->ep_buf));
  memcpy(handle_out, &h, sizeof(h));
  return SFK_OK;
}

sfk_status sfk_ep_connect(sfk_engine* e, const void* handles, int32_t n_ranks) {
  if (!e || !handles) return fail(SFK_ERR_INVALID_ARGUMENT, "null argument");
  if (e->ep_size <= 1) return fail(SFK_ERR_INVALID_ARGUMENT, "engine is not expert-parallel");
  if (n_ranks != e->ep_size) return fail(SFK_ERR_INVALID_ARGUMENT, "%d handles for %d ranks", n_ranks, e->ep_size);
  if (e->ep_connected) return fail(SFK_ERR_INVALID_ARGUMENT, "already connected");
  CK(cudaSetDevice(e->device));
  const size_t part = sizeof(float) * 4 * (size_t)e->hp.max_batch * e->hp.n_embd;
  for (int r = 0; r < n_ranks; ++r) {
    uint8_t* base = nullptr;
    if (r == e->ep_rank) {
      base = reinterpret_cast<uint8_t*>(e->ep_buf);
    } else {
      cudaIpcMemHandle_t h;
      memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)r * SFK_EP_HANDLE_BYTES, sizeof(h));
      void* p = nullptr;
      cudaError_t ce = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
      if (ce != cudaSuccess) return fail(SFK_ERR_RUNTIME, "rank %d buffer: %s", r, cudaGetErrorString(ce));
      e->ep_opened.push_back(p);
      base = static_cast<uint8_t*>(p);
    }
    e->ep_parts[r] = reinterpret_cast<const float*>(base);
    e->ep_peer_flags[r] = reinterpret_cast<unsigned*>(base + part);
    e->ep_peer_head_flags[r] = reinterpret_cast<unsigned*>(base + part + 128);
    e->ep_peer_keys[r] = reinterpret_cast<const unsigned long long*>(base + part + 256);
  }
  e->ep_connected = true;
  return SFK_OK;
}

// ---- operator-level -------------------------------------------------------
int64_t sfk_dev_row_bytes(int t, int64_t K) {
  if (!quant_ok(t) || K % 256) return 0;
  return dev_row_bytes(t, (int)K);
}

sfk_status sfk_repack(int t, const void* src, void* dst, int64_t nrows, int64_t K, void* stream) {
  if (!quant_ok(t) || K % 256 || !src || !dst) return fail(SFK_ERR_INVALID_ARGUMENT, "repack arguments");
  CK(launch_repack(t, (const uint8_t*)src, (uint8_t*)dst, nrows, (int)K, (cudaStream_t)stream));
  return SFK_OK;
}

sfk_status sfk_unpack(int t, const void* src, void* dst, int64_t nrows, int64_t K, void* stream) {
  if (!quant_ok(t) || K % 256 || !src || !dst) return fail(SFK_ERR_INVALID_ARGUMENT, "unpack arguments");
  CK(launch_unpack(t, (const uint8_t*)src, (uint8_t*)dst, nrows, (int)K, (cudaStream_t)stream));
  return SFK_OK;
}

sfk_status sfk_dequantize(int t, const void* src, float* dst, int64_t n, void* stream) {
  if (!src || !dst || n < 0) return fail(SFK_ERR_INVALID_ARGUMENT, "dequantize arguments");
  const int qk = (t == T_Q8_0) ? 32 : ((t == T_Q4_K || t == T_Q6_K) ? 256 : 1);
  if (!(quant_ok(t) || t == T_F32 || t == T_F16) || n % qk) return fail(SFK_ERR_INVALID_ARGUMENT, "type / size");
  if (n == 0) return SFK_OK;
  CK(launch_dequant(t, (const uint8_t*)src, dst, n, (cudaStream_t)stream));
  return SFK_OK;
}

sfk_status sfk_quantize_act(int act_type, const float* x, int32_t b, int64_t K, void* out, void* stream) {
  if (!x || !out || b < 0 || K % 256 || (act_type != T_Q8_K && act_type != T_Q8_0))
    return fail(SFK_ERR_INVALID_ARGUMENT, "quantize_act arguments");
  if (b == 0) return SFK_OK;
  CK(launch_quant_act_gguf(act_type, x, b, (int)K, (uint8_t*)out, (cudaStream_t)stream));
  return SFK_OK;
}

sfk_status sfk_mul_mat_tc(int t, const void* w, int64_t rows, int64_t K, const float* x, int32_t n, float* y,
                          void* stream) {
  if (!quant_ok(t) || K % 256 || !w || !x || !y || n < 1 || rows < 1 || rows > (1 << 30))
    return fail(SFK_ERR_INVALID_ARGUMENT, "mul_mat_tc arguments");
  const int act = act_for(t);
  const int npad = (n + TC_TT - 1) / TC_TT * TC_TT;
  const size_t need = tc_act_bytes(npad, (int)K);
  OpScratch* sc = nullptr;
  sfk_status s = op_scratch(need, 1, &sc);
  if (s) return s;
  cudaStream_t st = (cudaStream_t)stream;
  uint8_t* buf = static_cast<uint8_t*>(sc->buf);
  CK(launch_tc_quant(act, x, K, nullptr, n, npad, (int)K, buf, st));
  TcGemmParams p{};
  p.w = (const uint8_t*)w;
  p.rowstride = dev_row_bytes(t, (int)K);
  p.rows = (int)rows;
  p.K = (int)K;
  p.wtype = t;
  p.act_type = act;
  p.xq = buf;
  p.n = n;
  p.ntile = npad / TC_TT;
  p.y = y;
  p.ldy = rows;
  p.epi = TC_EPI_STORE;
  p.status = sc->status;
  CK(launch_tc_gemm(p, st));
  return check_status_word(sc->status, st);
}

sfk_status sfk_mul_mat_id_tc(int t, const void* w, int32_t n_expert, int64_t rows, int64_t K, const float* x,
                             int32_t x_per_pair, const int32_t* ids, int32_t b, int32_t k, float* y, void* stream) {
  if (!quant_ok(t) || K % 256 || !w || !x || !ids || !y || b < 1 || k < 1 || (int64_t)b * k > (1 << 20) ||
      n_expert < 1 || n_expert > 1024 || rows < 1 || rows > 65535 * 128)
    return fail(SFK_ERR_INVALID_ARGUMENT, "mul_mat_id_tc arguments");
  const int act = act_for(t);
  const int np = b * k;
  // every expert's pairs in whole 64-row tiles: at most one partial tile per
  // routed expert beyond the full ones
  const int mt = (np + TC_TT - 1) / TC_TT + std::min(n_expert, np);
  const int rows_pad = mt * TC_TT;
  auto up = [](size_t v) { return (v + 255) & ~(size_t)255; };
  const size_t act_b = up(tc_act_bytes(rows_pad, (int)K));
  const size_t ypad_b = up(sizeof(float) * (size_t)rows_pad * (size_t)rows);
  const size_t ints_b = up(sizeof(int) * ((size_t)np + 2 * (size_t)rows_pad + (size_t)mt));
  OpScratch* sc = nullptr;
  sfk_status s = op_scratch(act_b + ypad_b + ints_b, 1, &sc);
  if (s) return s;
  cudaStream_t st = (cudaStream_t)stream;
  uint8_t* buf = static_cast<uint8_t*>(sc->buf);
  float* ypad = reinterpret_cast<float*>(buf + act_b);
  int* pos_of_pair = reinterpret_cast<int*>(buf + act_b + ypad_b);
  int* rows_tok = pos_of_pair + np;
  int* rows_self = rows_tok + rows_pad;
  int* tile_expert = rows_self + rows_pad;
  // group the pairs by expert; the activation row of pair i is token i / k,
  // or pair i itself when every pair has its own row
  CK(launch_pf_group(ids, np, x_per_pair ? 1 : k, n_expert, mt, pos_of_pair, rows_tok, rows_self, tile_expert,
                     sc->status, st));
  CK(launch_tc_quant(act, x, K, rows_tok, x_per_pair ? np : b, rows_pad, (int)K, buf, st));
  TcGemmParams p{};
  p.w = (const uint8_t*)w;
  p.rowstride = dev_row_bytes(t, (int)K);
  p.expert_stride = rows * p.rowstride;
  p.rows = (int)rows;
  p.K = (int)K;
  p.wtype = t;
  p.act_type = act;
  p.xq = buf;
  p.ntile = mt;
  p.tile_expert = tile_expert;
  p.y = ypad;
  p.ldy = rows;
  p.epi = TC_EPI_STORE;
  p.status = sc->status;
  CK(launch_tc_gemm(p, st));
  CK(launch_pf_ungroup(ypad, pos_of_pair, np, rows, y, st));
  return check_status_word(sc->status, st);
}

sfk_status sfk_sample_logits(const float* logits, int32_t V, const sfk_sampling* sp, int32_t step, int32_t* token_out,
                             void* stream) {
  if (!logits || !sp || !token_out || V < 1 || step < 0 || !(sp->temperature > 0.0f))
    return fail(SFK_ERR_INVALID_ARGUMENT, "sample_logits arguments");
  // scratch: V floats, the key, the token
  const size_t need = ((sizeof(float) * (size_t)V + 15) & ~(size_t)15) + 16 + 16;
  OpScratch* sc = nullptr;
  sfk_status s = op_scratch(need, 1, &sc);
  if (s) return s;
  uint8_t* buf = static_cast<uint8_t*>(sc->buf);
  float* p = reinterpret_cast<float*>(buf);
  unsigned long long* key = reinterpret_cast<unsigned long long*>(buf + ((sizeof(float) * (size_t)V + 15) & ~(size_t)15));
  int* tok = reinterpret_cast<int*>(key + 2);
  SampleArgs a{};
  a.temperature = sp->temperature;
  a.top_p = sp->top_p;
  a.top_k = sp->top_k;
  a.seed = sp->seed;
  cudaStream_t st = (cudaStream_t)stream;
  CK(launch_sample(logits, V, a, step, p, key, tok, st));
  int h = 0;
  CK(cudaMemcpyAsync(&h, tok, sizeof(int), cudaMemcpyDeviceToHost, st));
  if ((s = check_status_word(sc->status, st))) return s;
  *token_out = h;
  return SFK_OK;
}

sfk_status sfk_mul_mat(int t, const void* w, int64_t rows, int64_t K, const float* x, int32_t b, float* y,
                       void* stream) {
  if (!quant_ok(t) || K % 256 || !w || !x || !y || b < 1 || b > MAXB || rows < 1)
    return fail(SFK_ERR_INVALID_ARGUMENT, "mul_mat arguments");
  OpScratch* sc = nullptr;
  sfk_status s = op_scratch(16, 1, &sc);
  if (s) return s;
  StreamParams p{};
  p.w0 = (const uint8_t*)w;
  p.rowstride = dev_row_bytes(t, (int)K);
  p.rows = (int)rows;
  p.K = (int)K;
  p.wtype = t;
  p.nmat = 1;
  p.act_type = act_for(t);
  p.row_align = 1;
  p.b = b; p.k = 1; p.n_pairs = b; p.n_vec = b;
  p.pro = PRO_QUANT;
  p.x = x;
  p.epi = EPI_STORE;
  p.y = y;
  p.y_stride = rows;
  p.status = sc->status;
  int dev = 0, grid = 0;
  CK(cudaGetDevice(&dev));
  s = plan_stream(p, sm_count_of(dev), &grid);
  if (s) return s;
  CK(launch_stream(p, grid, (cudaStream_t)stream, false));
  return check_status_word(sc->status, (cudaStream_t)stream);
}

sfk_status sfk_mul_mat_id(int t, const void* w, int32_t n_expert, int64_t rows, int64_t K, const float* x,
                          int32_t x_per_pair, const int32_t* ids, int32_t b, int32_t k, float* y, void* stream) {
  if (!quant_ok(t) || K % 256 || !w || !x || !ids || !y || b < 1 || b > MAXB || k < 1 || b * k > MAXP ||
      n_expert < 1 || rows < 1)
    return fail(SFK_ERR_INVALID_ARGUMENT, "mul_mat_id arguments");
  const size_t qbytes = (size_t)qact_bytes((int)K) * b * k;
  OpScratch* sc = nullptr;
  sfk_status s = op_scratch(qbytes, 1, &sc);
  if (s) return s;
  cudaStream_t st = (cudaStream_t)stream;
  CK(launch_route_build(ids, nullptr, b, k, n_expert, sc->route, sc->status, st));
  const int nvec = x_per_pair ? b * k : b;
  CK(launch_quant_act(act_for(t), x, nvec, (int)K, (uint8_t*)sc->buf, st));
  StreamParams p{};
  p.w0 = (const uint8_t*)w;
  p.rowstride = dev_row_bytes(t, (int)K);
  p.expert_stride = rows * p.rowstride;
  p.rows = (int)rows;
  p.K = (int)K;
  p.wtype = t;
  p.nmat = 1;
  p.act_type = act_for(t);
  p.row_align = 1;
  p.b = b; p.k = k; p.n_pairs = b * k; p.n_vec = nvec;
  p.route = sc->route;
  p.pro = PRO_LOAD;
  p.qact = (const uint8_t*)sc->buf;
  p.qact_stride = qact_bytes((int)K);
  p.xq_by_pair = x_per_pair ? 1 : 0;
  p.epi = EPI_STORE;
  p.y = y;
  p.y_stride = rows;
  p.status = sc->status;
  int dev = 0, grid = 0;
  CK(cudaGetDevice(&dev));
  s = plan_stream(p, sm_count_of(dev), &grid);
  if (s) return s;
  CK(launch_stream(p, grid, st, false));
  return check_status_word(sc->status, st);
}

sfk_status sfk_moe_ffn(int type_gu, int type_down, const void* gate, const void* up, const void* down,
                       int32_t n_expert, int64_t d, int64_t F, const float* x, const float* res, const int32_t* ids,
                       const float* wts, int32_t b, int32_t k, float* out, void* stream) {
  if (!quant_ok(type_gu) || !quant_ok(type_down) || d % 256 || F % 256 || !gate || !up || !down || !x || !ids ||
      !wts || !out || b < 1 || b > MAXB || k < 1 || b * k > MAXP || n_expert < 1)
    return fail(SFK_ERR_INVALID_ARGUMENT, "moe_ffn arguments");
  const size_t xq_b = (size_t)qact_bytes((int)d) * b;
  const size_t h_b = sizeof(float) * (size_t)b * k * F;
  const size_t hq_b = (size_t)qact_bytes((int)F) * b * k;
  OpScratch* sc = nullptr;
  sfk_status s = op_scratch(xq_b + h_b + hq_b + 256, (size_t)(F / 256), &sc);
  if (s) return s;
  cudaStream_t st = (cudaStream_t)stream;
  uint8_t* xq = (uint8_t*)sc->buf;
  float* h = (float*)(xq + ((xq_b + 255) & ~(size_t)255));
  uint8_t* hq = (uint8_t*)h + ((h_b + 255) & ~(size_t)255);
  if ((size_t)(hq - (uint8_t*)sc->buf) + hq_b > sc->bytes) {
    s = op_scratch((size_t)(hq - (uint8_t*)sc->buf) + hq_b, (size_t)(F / 256), &sc);
    if (s) return s;
    xq = (uint8_t*)sc->buf;
    h = (float*)(xq + ((xq_b + 255) & ~(size_t)255));
    hq = (uint8_t*)h + ((h_b + 255) & ~(size_t)255);
  }
  CK(launch_route_build(ids, wts, b, k, n_expert, sc->route, sc->status, st));
  CK(launch_quant_act(act_for(type_gu), x, b, (int)d, xq, st));
  int dev = 0, grid = 0;
  CK(cudaGetDevice(&dev));
  const int sms = sm_count_of(dev);
  {
    StreamParams p{};
    p.w0 = (const uint8_t*)gate;
    p.w1 = (const uint8_t*)up;
    p.rowstride = dev_row_bytes(type_gu, (int)d);
    p.expert_stride = F * p.rowstride;
    p.rows = (int)F;
    p.K = (int)d;
    p.wtype = type_gu;
    p.nmat = 2;
    p.act_type = act_for(type_gu);
    p.row_align = 1;
    p.b = b; p.k = k; p.n_pairs = b * k; p.n_vec = b;
    p.route = sc->route;
    p.pro = PRO_LOAD;
    p.qact = xq;
    p.qact_stride = qact_bytes((int)d);
    p.epi = EPI_GATEUP;
    p.h = h;
    p.hq = hq;
    p.grp_counter = sc->counters;
    p.h_act_type = act_for(type_down);
    p.status = sc->status;
    s = plan_stream(p, sms, &grid);
    if (s) return s;
    CK(launch_stream(p, grid, st, false));
  }
  {
    StreamParams p{};
    p.w0 = (const uint8_t*)down;
    p.rowstride = dev_row_bytes(type_down, (int)F);
    p.expert_stride = d * p.rowstride;
    p.rows = (int)d;
    p.K = (int)F;
    p.wtype = type_down;
    p.nmat = 1;
    p.act_type = act_for(type_down);
    p.row_align = 1;
    p.b = b; p.k = k; p.n_pairs = b * k; p.n_vec = b * k;
    p.route = sc->route;
    p.pro = PRO_LOAD;
    p.qact = hq;
    p.qact_stride = qact_bytes((int)F);
    p.xq_by_pair = 1;
    p.epi = EPI_DOWN;
    p.y = out;
    p.res = res;
    p.y_stride = d;
    p.status = sc->status;
    s = plan_stream(p, sms, &grid);
    if (s) return s;
    CK(launch_stream(p, grid, st, false));
  }
  return check_status_word(sc->status, st);
}

sfk_status sfk_attn_decode_paged(const float* q, const void* kp, const void* vp, int32_t kv_type, int32_t n_pages,
                                 const int32_t* page_table, int32_t max_pages, const int32_t* positions, int32_t b,
                                 int32_t n_head, int32_t n_head_kv, int32_t head_dim, float* out, void* stream) {
  if (!q || !kp || !vp || !page_table || !positions || !out || b < 1 || b > MAXB || n_head_kv < 1 || n_pages < 1 ||
      max_pages < 1 ||
      n_head % n_head_kv || (head_dim != 32 && head_dim != 64 && head_dim != 128 && head_dim != 256) ||
      (kv_type != SFK_KV_F16 && kv_type != SFK_KV_F32))
    return fail(SFK_ERR_INVALID_ARGUMENT, "attn_decode_paged arguments");
  OpScratch* sc = nullptr;
  sfk_status s = op_scratch(16, 1, &sc);
  if (s) return s;
  AttnParams a{};
  a.q = q;
  a.kv.k = const_cast<void*>(kp);
  a.kv.v = const_cast<void*>(vp);
  a.kv.page_table = page_table;
  a.kv.max_pages = max_pages;
  a.kv.n_pages = n_pages;
  a.kv.n_head_kv = n_head_kv;
  a.kv.head_dim = head_dim;
  a.kv.f16 = kv_type == SFK_KV_F16 ? 1 : 0;
  a.pos = positions;
  a.b = b;
  a.n_head = n_head;
  a.cluster = attn_cluster_for(max_pages * 16);
  a.max_chunk = (max_pages + a.cluster - 1) / a.cluster * 16;  // whole pages per CTA
  if (attn_smem_bytes(head_dim, n_head / n_head_kv, a.kv.f16, a.max_chunk) > (size_t)SMEM_LIMIT)
    return fail(SFK_ERR_UNSUPPORTED, "context of %d pages too long", max_pages);
  a.out = out;
  a.status = sc->status;
  CK(launch_attn(a, (cudaStream_t)stream, false));
  return check_status_word(sc->status, (cudaStream_t)stream);
}

}  // extern "C"
