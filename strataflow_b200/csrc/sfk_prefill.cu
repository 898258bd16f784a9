// sfk_prefill.cu -- per-token kernels of the batched prompt prefill.
//
// The reference feeds a prompt one position per Engine::forward call
// (tests/test_engine_oracle.cpp:182-187, src/model/engine/engine.cpp:1961).
// The prefill here runs a chunk of prompt tokens through each layer at once:
// the matrices on the tensor cores (sfk_tc.cu), these kernels for what lies
// between them.  Each kernel restates the arithmetic of the decode path's
// fused epilogues and prologues for many tokens, so a prompt token's values
// differ from token-by-token decode only in the fp32 order of the GEMMs'
// block sums.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include "sfk_dequant.cuh"
#include "sfk_device.cuh"
#include "sfk_prefill.cuh"
#include "sfk_route.cuh"
#include "sfk_tc.cuh"

namespace sfk {
namespace {

// ---- embedding ---------------------------------------------------------------
__global__ void __launch_bounds__(256) pf_embed_kernel(const uint8_t* tok_embd, int type, int d, int V,
                                                       const int* tok, int n, int pos0, float* x, int* pos,
                                                       int* pos_next, int* status) {
  const int t = blockIdx.y;
  int id = tok[t];
  if (id < 0 || id >= V) {
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(status, ERR_BAD_ID);
    id = 0;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    pos[t] = pos0 + t;
    if (t == 0 && pos_next) *pos_next = pos0 + n;
  }
  const uint8_t* row = tok_embd + (int64_t)id * dev_gguf_row_bytes(type, d);
  const int i = blockIdx.x * 256 + threadIdx.x;
  if (i < d) x[(int64_t)t * d + i] = gguf_dequant_one(type, row, i);
}

// ---- RMSNorm ---------------------------------------------------------------------
// squares summed in double, mean = (float)(sum / d), scale = 1 / sqrtf(mean +
// eps), y = (x * scale) * w: the formula of the decode prologues
// (engine.cpp:1878-1879, ggml_rms_norm + ggml_mul)
__global__ void __launch_bounds__(256) pf_norm_kernel(const float* x, const float* w, int d, float eps, float* y) {
  const int t = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const float* xr = x + (int64_t)t * d;
  __shared__ double red[8];
  double s = 0.0;
  for (int c = tid; c < d; c += 256) {
    const float v = xr[c];
    s += (double)__fmul_rn(v, v);
  }
  s = warp_sum_d(s);
  if (lane == 0) red[warp] = s;
  __syncthreads();
  double tot = 0.0;
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float mean = (float)(tot / (double)d);
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
  for (int c = tid; c < d; c += 256) y[(int64_t)t * d + c] = __fmul_rn(__fmul_rn(xr[c], scale), w[c]);
}

// ---- RoPE + KV append ------------------------------------------------------------
// ggml rope NORMAL (engine.cpp:1892-1897): rows (r, r + 1) rotated by
// theta_i = pos * theta_scale^i from the host-built table; K and V appended
// at the token's position (engine.cpp:1646-1656)
__global__ void __launch_bounds__(256) pf_rope_kv_kernel(const float* qkv, int n, int nq, KvView kv,
                                                         const int* pt_row, const float* rope, int pos0, float* q_out,
                                                         int* status) {
  const int hd = kv.head_dim, Hkv = kv.n_head_kv;
  const int nk = Hkv * hd, nqkv = nq + 2 * nk, half_rows = nqkv / 2;
  const int64_t idx = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (idx >= (int64_t)n * half_rows) return;
  const int t = (int)(idx / half_rows);
  const int r = 2 * (int)(idx % half_rows);
  const int pos = pos0 + t;
  const float x0 = qkv[(int64_t)t * nqkv + r], x1 = qkv[(int64_t)t * nqkv + r + 1];
  float o0 = x0, o1 = x1;
  if (r < nq + nk) {
    const int i = (r % hd) >> 1;
    const float2 cs = reinterpret_cast<const float2*>(rope)[(int64_t)pos * (hd >> 1) + i];
    o0 = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
    o1 = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
  }
  if (r < nq) {
    q_out[(int64_t)t * nq + r] = o0;
    q_out[(int64_t)t * nq + r + 1] = o1;
    return;
  }
  const bool is_k = r < nq + nk;
  const int rr = r - nq - (is_k ? 0 : nk);
  const int h = rr / hd, i0 = rr % hd;
  const int page = pt_row[pos / 16];
  if (!kv_page_writable(kv, page)) {  // never write outside the pool
    atomicExch(status, ERR_BAD_PAGE);
    return;
  }
  const int64_t off = (((int64_t)page * Hkv + h) * 16 + (pos & 15)) * hd + i0;
  void* base = is_k ? kv.k : kv.v;
  if (kv.f16) {
    __half* kb = reinterpret_cast<__half*>(base);
    kb[off] = __float2half_rn(o0);
    kb[off + 1] = __float2half_rn(o1);
  } else {
    float* kb = reinterpret_cast<float*>(base);
    kb[off] = o0;
    kb[off + 1] = o1;
  }
}

__global__ void pf_pt_kernel(const int* pt_row, int max_pages, int n, int* pt_out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < (int64_t)n * max_pages) pt_out[i] = pt_row[i % max_pages];
}

// ---- routing ---------------------------------------------------------------------
constexpr int PF_RT_THREADS = 1024;
constexpr int PF_RT_MAXE = 512;
struct PfBlockSync {
  __device__ void operator()() const { __syncthreads(); }
};

__global__ void __launch_bounds__(PF_RT_THREADS) pf_route_kernel(const float* x, const float* norm_w,
                                                                 const float* w_r, int d, int E, int k, float eps,
                                                                 int act_type, uint8_t* xq, float* xn_out, int* ids,
                                                                 float* w) {
  const int t = blockIdx.x;
  extern __shared__ __align__(16) uint8_t rsm[];
  float* xn = reinterpret_cast<float*>(rsm);  // [d]
  __shared__ double red[PF_RT_THREADS / 32 + 1];
  __shared__ float probs[PF_RT_MAXE];
  __shared__ double seg[PF_RT_MAXE * 4];
  route_one<PF_RT_THREADS / 32>(x + (int64_t)t * d, norm_w, w_r, d, E, k, eps, act_type, xq + (int64_t)t * qact_bytes(d),
                                xn, seg, probs, red, ids + (int64_t)t * k, w + (int64_t)t * k,
                                xn_out + (int64_t)t * d, PfBlockSync{});
}

// ---- expert grouping -------------------------------------------------------------
// One CTA.  Counts per expert, 64-aligned segment starts, then the rank of each
// pair among its expert's pairs in pair order: per 1024-pair round, lanes with
// the same expert find each other with match_any, and per-warp histograms are
// prefix-summed across the warps (and the earlier rounds).
constexpr int PF_GROUP_THREADS = 1024;

__global__ void __launch_bounds__(PF_GROUP_THREADS) pf_group_kernel(const int* ids, int np, int k, int E, int max_tiles,
                                                                    int* pos_of_pair, int* rows_tok, int* rows_self,
                                                                    int* tile_expert, int* status) {
  extern __shared__ int gsm[];
  int* cnt = gsm;         // [E]
  int* off = cnt + E;     // [E]
  int* run = off + E;     // [E] pairs of each expert placed in earlier rounds
  int* hist = run + E;    // [32][E]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int e = tid; e < E; e += PF_GROUP_THREADS) {
    cnt[e] = 0;
    run[e] = 0;
  }
  __syncthreads();
  for (int i = tid; i < np; i += PF_GROUP_THREADS) {
    int e = ids[i];
    if (e < 0 || e >= E) {
      atomicExch(status, ERR_BAD_ID);
      e = 0;
    }
    atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  if (tid == 0) {
    int o = 0, tile = 0;
    for (int e = 0; e < E; ++e) {
      off[e] = o;
      const int nt = (cnt[e] + TC_TT - 1) / TC_TT;
      for (int j = 0; j < nt && tile < max_tiles; ++j) tile_expert[tile++] = e;
      o += nt * TC_TT;
    }
    for (; tile < max_tiles; ++tile) tile_expert[tile] = -1;
  }
  for (int p = tid; p < max_tiles * TC_TT; p += PF_GROUP_THREADS) {
    rows_tok[p] = -1;
    rows_self[p] = -1;
  }
  __syncthreads();
  for (int r0 = 0; r0 < np; r0 += PF_GROUP_THREADS) {
    const int i = r0 + tid;
    int e = -1;
    if (i < np) {
      e = ids[i];
      if (e < 0 || e >= E) e = 0;
    }
    for (int j = tid; j < 32 * E; j += PF_GROUP_THREADS) hist[j] = 0;
    __syncthreads();
    const unsigned same = __match_any_sync(0xffffffffu, e);
    const int rank_w = __popc(same & ((1u << lane) - 1u));
    if (e >= 0 && rank_w == 0) hist[warp * E + e] = __popc(same);
    __syncthreads();
    for (int x = tid; x < E; x += PF_GROUP_THREADS) {  // exclusive prefix over the warps
      int acc = run[x];
      for (int w = 0; w < 32; ++w) {
        const int c = hist[w * E + x];
        hist[w * E + x] = acc;
        acc += c;
      }
      run[x] = acc;
    }
    __syncthreads();
    if (e >= 0) {
      const int p = off[e] + hist[warp * E + e] + rank_w;
      if (p < max_tiles * TC_TT) {
        pos_of_pair[i] = p;
        rows_tok[p] = i / k;
        rows_self[p] = p;
      } else {
        atomicExch(status, ERR_BAD_ID);
        pos_of_pair[i] = 0;
      }
    }
    __syncthreads();
  }
}

// ---- combine ---------------------------------------------------------------------
__global__ void __launch_bounds__(256) pf_combine_kernel(const float* yd, const int* pos_of_pair, const float* w,
                                                         int k, int n, int d, const float* res, float* x) {
  const int64_t idx = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (idx >= (int64_t)n * d) return;
  const int t = (int)(idx / d), c = (int)(idx % d);
  // experts * weights, then moe_out = e0 + e1 + ..., then + ffn_inp
  float a = __fmul_rn(yd[(int64_t)pos_of_pair[t * k] * d + c], w[t * k]);
  for (int j = 1; j < k; ++j) a = __fadd_rn(a, __fmul_rn(yd[(int64_t)pos_of_pair[t * k + j] * d + c], w[t * k + j]));
  x[idx] = __fadd_rn(a, res[idx]);
}

unsigned blocks_for(int64_t items, int per) { return (unsigned)((items + per - 1) / per); }

__global__ void __launch_bounds__(256) pf_ungroup_kernel(const float4* src, const int* pos_of_pair, int np,
                                                         int64_t rows4, float4* y) {
  const int64_t idx = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (idx >= (int64_t)np * rows4) return;
  const int64_t i = idx / rows4, c = idx % rows4;
  y[idx] = src[(int64_t)pos_of_pair[i] * rows4 + c];
}

__global__ void __launch_bounds__(256) pf_ungroup1_kernel(const float* src, const int* pos_of_pair, int np,
                                                          int64_t rows, float* y) {
  const int64_t idx = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (idx >= (int64_t)np * rows) return;
  const int64_t i = idx / rows, c = idx % rows;
  y[idx] = src[(int64_t)pos_of_pair[i] * rows + c];
}

// ---- causal attention over the paged KV -----------------------------------------
// The arithmetic of the reference's per-token attention as the CPU oracle and
// the decode kernel compute it (engine.cpp:1751-1761: ggml_mul_mat(k, q),
// ggml_soft_max_ext, ggml_mul_mat(v, kq)): scores are fp32 products summed in
// double, y = (float)score * scale; p = e * (float)(1 / sum e) with
// e = exp(y - max y) (the shared exp, sfk_expf) and the sum in double; the
// output is fp32 products v * p summed in double.  Every prompt token gets
// exactly the values a token-by-token prompt gets.
//
// One CTA per (64 query rows, kv head): the rows are QT = 64 / gqa prompt
// tokens x the gqa query heads sharing the kv head.  Three passes over the
// keys, 64 positions at a time through shared memory (read through the
// sequence's page table):
//   1. S = Q K^T on 4 x 4 register tiles (thread (ty, tx) owns rows ty + 16a
//      and keys tx + 16c, so eight consecutive tx read eight padded K rows in
//      different banks); y to a scratch row, and the row maxima.
//   2. e = exp(y - max) over the thread's own scratch entries; row sums.
//   3. P = e * inv into shared memory, O += P V for the thread's 4 rows x
//      HD/16 columns.
constexpr int PA_R = 64;   // query rows per CTA
constexpr int PA_KB = 64;  // keys per block

struct PfAttnParams {
  const float* q;       // [n][nq]
  KvView kv;
  const int* pt_row;    // the sequence's page table
  float* out;           // [n][nq]
  float* scratch;       // [row tiles][Hkv][64][ld] scores, then exponentials
  int64_t ld;           // keys per scratch row (>= pos0 + n, a multiple of 64)
  int n, pos0, n_head, nq;
  float scale;
  int* status;
};

template <int HD, int F16>
struct PaSmem {
  using KT = typename std::conditional<F16 != 0, __half, float>::type;
  static constexpr int QS = HD + 4;  // floats
  static constexpr int KS = HD + 4;  // elements
  static constexpr int PS = PA_KB + 4;  // floats
  static constexpr size_t q_off = 0;
  static constexpr size_t k_off = q_off + sizeof(float) * PA_R * QS;   // K in pass 1, V in pass 3
  static constexpr size_t p_off = k_off + sizeof(KT) * PA_KB * KS;
  static constexpr size_t bytes = p_off + sizeof(float) * PA_R * PS;
};

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 ld4(const __half* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

// the thread's O columns of V row `row`: 4 tx + 64 e + i (HD >= 64) or 2 tx + i
template <int HD, typename KT>
__device__ __forceinline__ void load_vrow(const KT* row, int tx, float (&v)[HD / 16]) {
  if constexpr (HD == 32) {
    if constexpr (sizeof(KT) == 2) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(row + 2 * tx));
      v[0] = f.x;
      v[1] = f.y;
    } else {
      const float2 f = *reinterpret_cast<const float2*>(row + 2 * tx);
      v[0] = f.x;
      v[1] = f.y;
    }
  } else {
#pragma unroll
    for (int e = 0; e < HD / 64; ++e) {
      const float4 f = ld4(row + 4 * tx + 64 * e);
      v[4 * e] = f.x;
      v[4 * e + 1] = f.y;
      v[4 * e + 2] = f.z;
      v[4 * e + 3] = f.w;
    }
  }
}

// Stage rows kb*64 .. +63 of the kv head's K (or V) pool into `dst` (row
// stride `stride` elements); positions past qpos_max read as zero.
template <int HD, typename KT>
__device__ __forceinline__ void stage_kv(KT* dst, int stride, int isv, const PfAttnParams& p, int kvh, int kb,
                                         int qpos_max) {
  constexpr int VEC = 16 / sizeof(KT);  // elements per 16 bytes
  const int Hkv = p.kv.n_head_kv;
  for (int idx = threadIdx.x; idx < PA_KB * HD / VEC; idx += 256) {
    const int j = idx / (HD / VEC), c = idx % (HD / VEC);
    const int kp = kb * PA_KB + j;
    uint4 v4 = make_uint4(0, 0, 0, 0);
    if (kp <= qpos_max) {
      const int page = p.pt_row[kp >> 4];
      if (page < 0 || (p.kv.n_pages > 0 && page >= p.kv.n_pages)) {
        atomicExch(p.status, ERR_BAD_PAGE);
      } else {
        const int64_t off = (((int64_t)kvh * 16 + (kp & 15)) * HD + c * VEC) * (int64_t)sizeof(KT);
        const int64_t page_bytes = (int64_t)Hkv * 16 * HD * (int64_t)sizeof(KT);
        v4 = __ldg(reinterpret_cast<const uint4*>(kv_page(p.kv, isv, page, page_bytes) + off));
      }
    }
    // padded rows keep 8-byte alignment: two 8-byte stores
    uint2* d = reinterpret_cast<uint2*>(dst + j * stride + c * VEC);
    d[0] = make_uint2(v4.x, v4.y);
    d[1] = make_uint2(v4.z, v4.w);
  }
}

template <int HD, int F16>
__global__ void __launch_bounds__(256, HD >= 256 ? 1 : 2) pf_attn_kernel(const PfAttnParams p) {
  static_assert(HD == 32 || HD % 64 == 0, "head widths of 32, 64, 128, 256");
  using SM = PaSmem<HD, F16>;
  using KT = typename SM::KT;
  constexpr int QS = SM::QS, KS = SM::KS, PS = SM::PS;
  constexpr int CPT = HD / 16;  // O columns per thread
  extern __shared__ __align__(16) uint8_t pa_smem[];
  float* Qs = reinterpret_cast<float*>(pa_smem + SM::q_off);
  KT* KVs = reinterpret_cast<KT*>(pa_smem + SM::k_off);
  float* Ps = reinterpret_cast<float*>(pa_smem + SM::p_off);

  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int Hkv = p.kv.n_head_kv, gqa = p.n_head / Hkv, QT = PA_R / gqa;
  const int tile = gridDim.x - 1 - blockIdx.x;  // the longest prefixes first
  const int kvh = blockIdx.y;
  const int t0 = tile * QT;
  const int t_end = min(t0 + QT, p.n);
  const int qpos_max = p.pos0 + t_end - 1;
  const int nkb = qpos_max / PA_KB + 1;
  float* ysc = p.scratch + ((int64_t)tile * Hkv + kvh) * PA_R * p.ld;

  // Q rows: row r = token t0 + r / gqa, head kvh * gqa + r % gqa
  for (int idx = tid; idx < PA_R * HD / 4; idx += 256) {
    const int r = idx / (HD / 4), c4 = idx % (HD / 4);
    const int t = t0 + r / gqa, h = kvh * gqa + r % gqa;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (t < p.n) v = *reinterpret_cast<const float4*>(p.q + (int64_t)t * p.nq + h * HD + 4 * c4);
    *reinterpret_cast<float4*>(Qs + r * QS + 4 * c4) = v;
  }
  int qpos[4];
#pragma unroll
  for (int a = 0; a < 4; ++a) qpos[a] = p.pos0 + t0 + (ty + 16 * a) / gqa;

  // pass 1: y = (float)(sum_d (double)(k_d q_d)) * scale, row maxima
  float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
  for (int kb = 0; kb < nkb; ++kb) {
    __syncthreads();  // the previous block's K is consumed
    stage_kv<HD>(KVs, KS, 0, p, kvh, kb, qpos_max);
    __syncthreads();
    double s[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int c = 0; c < 4; ++c) s[a][c] = 0.0;
#pragma unroll 2
    for (int d0 = 0; d0 < HD; d0 += 4) {
      float4 qa[4], kc[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) qa[a] = ld4(Qs + (ty + 16 * a) * QS + d0);
#pragma unroll
      for (int c = 0; c < 4; ++c) kc[c] = ld4(KVs + (tx + 16 * c) * KS + d0);
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          s[a][c] += (double)__fmul_rn(kc[c].x, qa[a].x);
          s[a][c] += (double)__fmul_rn(kc[c].y, qa[a].y);
          s[a][c] += (double)__fmul_rn(kc[c].z, qa[a].z);
          s[a][c] += (double)__fmul_rn(kc[c].w, qa[a].w);
        }
    }
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int kp = kb * PA_KB + tx + 16 * c;
        if (kp <= qpos[a]) {
          const float y = __fmul_rn((float)s[a][c], p.scale);
          ysc[(int64_t)(ty + 16 * a) * p.ld + kp] = y;
          mx[a] = fmaxf(mx[a], y);
        }
      }
  }
  // pass 2: e = exp(y - max) in place, sums in double
  double sum[4];
#pragma unroll
  for (int a = 0; a < 4; ++a) {
#pragma unroll
    for (int off = 1; off < 16; off <<= 1) mx[a] = fmaxf(mx[a], __shfl_xor_sync(0xffffffffu, mx[a], off));
    float* yr = ysc + (int64_t)(ty + 16 * a) * p.ld;
    double sm = 0.0;
    for (int kp = tx; kp <= qpos[a]; kp += 16) {
      const float e = sfk_expf(__fsub_rn(yr[kp], mx[a]));
      yr[kp] = e;
      sm += (double)e;
    }
#pragma unroll
    for (int off = 1; off < 16; off <<= 1) sm += __shfl_xor_sync(0xffffffffu, sm, off);
    sum[a] = sm;
  }
  float inv[4];
#pragma unroll
  for (int a = 0; a < 4; ++a) inv[a] = (float)(1.0 / sum[a]);
  // pass 3: O = sum_j (double)(v_j * p_j), p = e * inv
  double o[4][CPT];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int i = 0; i < CPT; ++i) o[a][i] = 0.0;
  for (int kb = 0; kb < nkb; ++kb) {
    __syncthreads();  // the previous block's V and P are consumed
    stage_kv<HD>(KVs, HD, 1, p, kvh, kb, qpos_max);
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int kp = kb * PA_KB + tx + 16 * c;
        Ps[(ty + 16 * a) * PS + tx + 16 * c] =
            kp <= qpos[a] ? __fmul_rn(ysc[(int64_t)(ty + 16 * a) * p.ld + kp], inv[a]) : 0.0f;
      }
    __syncthreads();
    const int jmax = min(PA_KB, qpos_max - kb * PA_KB + 1);
    for (int j0 = 0; j0 < jmax; j0 += 4) {
      float4 pa[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) pa[a] = *reinterpret_cast<const float4*>(Ps + (ty + 16 * a) * PS + j0);
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        float v[CPT];
        load_vrow<HD>(KVs + (j0 + jj) * HD, tx, v);
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          const float pj = jj == 0 ? pa[a].x : (jj == 1 ? pa[a].y : (jj == 2 ? pa[a].z : pa[a].w));
#pragma unroll
          for (int i = 0; i < CPT; ++i) o[a][i] += (double)__fmul_rn(v[i], pj);
        }
      }
    }
  }
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int r = ty + 16 * a;
    const int t = t0 + r / gqa, h = kvh * gqa + r % gqa;
    if (t >= p.n) continue;
    float* dst = p.out + (int64_t)t * p.nq + h * HD;
    if constexpr (HD == 32) {
      *reinterpret_cast<float2*>(dst + 2 * tx) = make_float2((float)o[a][0], (float)o[a][1]);
    } else {
#pragma unroll
      for (int e = 0; e < HD / 64; ++e)
        *reinterpret_cast<float4*>(dst + 4 * tx + 64 * e) =
            make_float4((float)o[a][4 * e], (float)o[a][4 * e + 1], (float)o[a][4 * e + 2], (float)o[a][4 * e + 3]);
    }
  }
}

template <int HD, int F16>
cudaError_t launch_pf_attn_t(const PfAttnParams& p, cudaStream_t st) {
  auto kern = pf_attn_kernel<HD, F16>;
  const size_t smem = PaSmem<HD, F16>::bytes;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int gqa = p.n_head / p.kv.n_head_kv, QT = PA_R / gqa;
  kern<<<dim3((unsigned)((p.n + QT - 1) / QT), (unsigned)p.kv.n_head_kv), 256, smem, st>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_pf_embed(const uint8_t* tok_embd, int type, int d, int V, const int* tok, int n, int pos0, float* x,
                            int* pos, int* pos_next, int* status, cudaStream_t st) {
  pf_embed_kernel<<<dim3((unsigned)((d + 255) / 256), (unsigned)n), 256, 0, st>>>(tok_embd, type, d, V, tok, n, pos0,
                                                                                 x, pos, pos_next, status);
  return cudaGetLastError();
}

cudaError_t launch_pf_norm(const float* x, const float* w, int n, int d, float eps, float* y, cudaStream_t st) {
  pf_norm_kernel<<<n, 256, 0, st>>>(x, w, d, eps, y);
  return cudaGetLastError();
}

cudaError_t launch_pf_rope_kv(const float* qkv, int n, int n_head, const KvView& kv, const int* pt_row,
                              const float* rope, int pos0, float* q_out, int* status, cudaStream_t st) {
  const int nqkv = n_head * kv.head_dim + 2 * kv.n_head_kv * kv.head_dim;
  pf_rope_kv_kernel<<<blocks_for((int64_t)n * (nqkv / 2), 256), 256, 0, st>>>(
      qkv, n, n_head * kv.head_dim, kv, pt_row, rope, pos0, q_out, status);
  return cudaGetLastError();
}

bool pf_attn_supported(int head_dim, int n_head, int n_head_kv) {
  if (n_head_kv < 1 || n_head % n_head_kv) return false;
  const int gqa = n_head / n_head_kv;
  return (head_dim == 32 || head_dim == 64 || head_dim == 128 || head_dim == 256) && gqa <= PA_R && PA_R % gqa == 0;
}

size_t pf_attn_scratch_bytes(int n, int pos0, int n_head, int n_head_kv) {
  const int gqa = n_head / n_head_kv, QT = PA_R / gqa;
  const int64_t ld = ((int64_t)pos0 + n + PA_KB - 1) / PA_KB * PA_KB;
  return (size_t)((n + QT - 1) / QT) * n_head_kv * PA_R * ld * sizeof(float);
}

cudaError_t launch_pf_attn(const float* q, const KvView& kv, const int* pt_row, int n, int pos0, int n_head,
                           float* out, float* scratch, int* status, cudaStream_t st) {
  if (!pf_attn_supported(kv.head_dim, n_head, kv.n_head_kv)) return cudaErrorInvalidValue;
  PfAttnParams p{};
  p.scratch = scratch;
  p.ld = ((int64_t)pos0 + n + PA_KB - 1) / PA_KB * PA_KB;
  p.q = q;
  p.kv = kv;
  p.pt_row = pt_row;
  p.out = out;
  p.n = n;
  p.pos0 = pos0;
  p.n_head = n_head;
  p.nq = n_head * kv.head_dim;
  p.scale = 1.0f / sqrtf((float)kv.head_dim);
  p.status = status;
  switch (kv.head_dim * 2 + (kv.f16 ? 1 : 0)) {
    case 64: return launch_pf_attn_t<32, 0>(p, st);
    case 65: return launch_pf_attn_t<32, 1>(p, st);
    case 128: return launch_pf_attn_t<64, 0>(p, st);
    case 129: return launch_pf_attn_t<64, 1>(p, st);
    case 256: return launch_pf_attn_t<128, 0>(p, st);
    case 257: return launch_pf_attn_t<128, 1>(p, st);
    case 512: return launch_pf_attn_t<256, 0>(p, st);
    case 513: return launch_pf_attn_t<256, 1>(p, st);
    default: return cudaErrorInvalidValue;
  }
}

__global__ void pt_set_kernel(int* pt, int idx, int id) { pt[idx] = id; }

cudaError_t launch_pt_set(int* page_table, int idx, int id, cudaStream_t st) {
  pt_set_kernel<<<1, 1, 0, st>>>(page_table, idx, id);
  return cudaGetLastError();
}

cudaError_t launch_pf_pt(const int* pt_row, int max_pages, int n, int* pt_out, cudaStream_t st) {
  pf_pt_kernel<<<blocks_for((int64_t)n * max_pages, 256), 256, 0, st>>>(pt_row, max_pages, n, pt_out);
  return cudaGetLastError();
}

cudaError_t launch_pf_route(const float* x, const float* norm_w, const float* w_r, int n, int d, int E, int k,
                            float eps, int act_type, uint8_t* xq_scratch, float* xn, int* ids, float* w, int* status,
                            cudaStream_t st) {
  (void)status;
  if (E > PF_RT_MAXE || k > E) return cudaErrorInvalidValue;
  const size_t smem = (size_t)d * sizeof(float);
  cudaError_t e = cudaFuncSetAttribute(pf_route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  pf_route_kernel<<<n, PF_RT_THREADS, smem, st>>>(x, norm_w, w_r, d, E, k, eps, act_type, xq_scratch, xn, ids, w);
  return cudaGetLastError();
}

cudaError_t launch_pf_group(const int* ids, int np, int k, int E, int max_tiles, int* pos_of_pair, int* rows_tok,
                            int* rows_self, int* tile_expert, int* status, cudaStream_t st) {
  const size_t smem = (size_t)(3 + 32) * E * sizeof(int);
  cudaError_t e = cudaFuncSetAttribute(pf_group_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  pf_group_kernel<<<1, PF_GROUP_THREADS, smem, st>>>(ids, np, k, E, max_tiles, pos_of_pair, rows_tok, rows_self,
                                                     tile_expert, status);
  return cudaGetLastError();
}

cudaError_t launch_pf_ungroup(const float* src, const int* pos_of_pair, int np, int64_t rows, float* y,
                              cudaStream_t st) {
  if (rows % 4 == 0 && ((uintptr_t)src | (uintptr_t)y) % 16 == 0)
    pf_ungroup_kernel<<<blocks_for((int64_t)np * (rows / 4), 256), 256, 0, st>>>(
        (const float4*)src, pos_of_pair, np, rows / 4, (float4*)y);
  else
    pf_ungroup1_kernel<<<blocks_for((int64_t)np * rows, 256), 256, 0, st>>>(src, pos_of_pair, np, rows, y);
  return cudaGetLastError();
}

cudaError_t launch_pf_combine(const float* yd, const int* pos_of_pair, const float* w, int k, int n, int d,
                              const float* res, float* x, cudaStream_t st) {
  pf_combine_kernel<<<blocks_for((int64_t)n * d, 256), 256, 0, st>>>(yd, pos_of_pair, w, k, n, d, res, x);
  return cudaGetLastError();
}

}  // namespace sfk
