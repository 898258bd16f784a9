// sfk_mega.cuh -- parameter block of the persistent decode-step kernel
// (sfk_mega.cu), shared with the host orchestration in sfk_api.cu.
//
// One cooperative launch runs a whole decode step (embedding, every layer,
// lm_head) on one CTA per SM.  The phases of a layer are separated by grid
// barriers; every warp streams the weight tiles of its share of each phase
// through its own ring of shared-memory slots, and the ring runs ahead across
// phase boundaries, so the next matrix's tiles are already arriving while the
// CTAs wait at a barrier or compute attention.
#pragma once
#include <cstdint>

#include "sfk_kernels.cuh"

namespace sfk {

constexpr int MEGA_NWS = 16;        // warps per CTA: 15 consumer warps and the producer warp
constexpr int MEGA_NC = MEGA_NWS - 1;  // consumer warps (each owns a ring of weight-tile slots)
constexpr int MEGA_MAXS = 4;        // ring slots per warp (at most)
constexpr int MEGA_MAXE = 64;       // experts the kernel routes itself
constexpr int MEGA_MAXGQA = 8;      // query heads per kv head (whole warps per head in the softmax sums)
constexpr int MEGA_RED = 128;       // doubles of reduction scratch
// weight phases of the tile plan
enum : int { MEGA_PK_QKV = 0, MEGA_PK_O = 1, MEGA_PK_GU = 2, MEGA_PK_DN = 3, MEGA_PK_OUT = 4 };

// Per-layer weights (device array, read-only).
struct MegaLayer {
  const uint8_t* qkv;      // [nq + 2 nk] rows of K = d (device layout)
  const uint8_t* wo;       // [d] rows of K = nq
  const float* attn_norm;  // [d]
  const float* ffn_norm;   // [d]
  const float* router;     // [E][d] F32
  const uint8_t* gate;     // [E][F] rows of K = d
  const uint8_t* up;
  const uint8_t* down;     // [E][d] rows of K = F
};

struct MegaParams {
  const MegaLayer* layers;
  int n_layer;
  // shape
  int d, nq, nk, nqkv, hd, n_head, n_head_kv, gqa, F, E, k, V, b, n_ctx;
  float eps, att_scale;
  int t_embd, t_attn, t_gu, t_down, t_out;
  int a_attn, a_gu, a_down, a_out;  // activation (dot) types: Q8_K or Q8_0
  int64_t rs_attn, rs_o, rs_gu, rs_down, rs_out;  // device row strides
  // plan (host): ring, tile rows, rows per CTA, shared-memory offsets
  int S, slot;
  // per weight phase (MEGA_PK_*): rows per tile R; a row longer than a slot
  // is cut into H tiles of gpp column groups each (then R = 1)
  int R[5], H[5], gpp[5];
  int rpc_qkv, rpc_o, rpc_gu, rpc_down, rpc_out;
  int rt_parts;       // router: parts per expert row (items = E * rt_parts)
  int att_ch;         // attention positions per work item (multiple of 16)
  int att_nc;         // chunks per (sequence, kv head) at n_ctx
  int S_log2;         // S = 1 << S_log2 ring slots per warp
  int lookahead;      // streamed phases a warp's ring may run ahead of the CTA's current step
  int off_ring, off_xq, off_acc, off_route, off_red, off_probs, off_att, off_misc, off_layers, smem;
  int xq_bytes;       // bytes of the xq region (activations; attention staging)
  // embedding / head
  const uint8_t* tok_embd;  // GGUF layout
  const float* out_norm;
  const uint8_t* output;
  // tokens and positions (the embed kernel's duties)
  const int* tok_in;
  const int* pos_in;        // host positions, or null: pos_state (greedy loop)
  int greedy;
  int* pos_state;
  int* pos_cur;
  int* tok_hist;
  unsigned long long* argmax_key;
  // KV cache and RoPE
  void* k_pool;
  void* v_pool;
  int64_t kv_layer_bytes;   // bytes of one layer's K (or V) pool
  const int* page_table;    // [b][max_pages]
  int max_pages, n_pages, kv_f16;
  const float* rope;        // [n_ctx][hd/2] (cos, sin)
  // step buffers (device)
  float* x;         // [b][d] layer input / output
  float* ffn_inp;   // [b][d]
  float* q;         // [b][nq] after RoPE
  float* attn_out;  // [b][nq]
  float* h;         // [b*k][F] SwiGLU
  uint8_t* hq;      // [b*k] qact(F)
  float* logits;    // [b][V]
  int* grp_counter; // [F/256], self-resetting
  Route* route_out; // routing of the last layer (host read-back)
  // attention exchange (device scratch)
  float* att_y;        // [b][Hq][n_ctx] scaled scores
  float* att_cmax;     // [b][Hkv][att_nc][gqa] chunk maxima
  float* att_stat;     // [b][Hq][2] (max, 1/sum)
  double* att_opart;   // [b][Hkv][att_nc][gqa][hd] chunk partial outputs
  int* att_cnt;        // [2][b][Hkv] arrival counters, self-resetting
  unsigned* att_ready; // [b][Hkv] softmax statistics ready (layer + 1), cleared at exit
  unsigned* gbar;      // [2] grid-barrier arrivals, exits; cleared at exit
  int* status;
  int store_logits;
};

// Host: launch one step (cooperative, one CTA per SM).  `grid` CTAs; returns
// cudaErrorNotSupported for a type combination without an instantiation.
cudaError_t launch_mega(const MegaParams& p, int grid, cudaStream_t st);
// Host: the weight-type combinations with a compiled kernel.
bool mega_types_supported(int t_attn, int t_gu, int t_down, int t_out);

}  // namespace sfk
