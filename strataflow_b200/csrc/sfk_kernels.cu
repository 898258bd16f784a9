// sfk_kernels.cu -- the sm_100a decode kernels.
//
//   stream_kernel  : HBM-streaming quantized GEMV / mul_mat_id.  One CTA per SM,
//                    one producer thread moving weight tiles with 1-D TMA bulk
//                    copies (cp.async.bulk) into an mbarrier ring, 8 consumer
//                    warps doing dp4a sub-block dots against ggml-quantized
//                    activations.  Weight tiles that do not depend on the
//                    previous kernel are requested before griddepcontrol.wait,
//                    so the next GEMV's weights stream while the previous
//                    kernel drains (programmatic dependent launch).
//                    Fused prologues (RMSNorm + activation quantization) and
//                    epilogues (RoPE + paged-KV append, residual, SwiGLU +
//                    Q8_K requantization, routed combine, argmax).
//   attn_kernel    : split-K GQA decode attention over the paged KV cache.
//   router_kernel  : ffn_norm + activation quantization + softmax router +
//                    top-k + renormalisation + slot lists.
//   embed_kernel   : token (host or greedy argmax) -> dequantized embedding row.
//
// Reference op order: src/model/engine/engine.cpp of Coaade-Inc/strataflow,
// router segment :1854-1947, attention :1633-1762, experts :1956-1989,
// embedding :2708-2723, head :2988-3006.  Elementwise steps use explicit
// round-to-nearest intrinsics (no FMA contraction) so they round exactly as
// the ggml CPU code does.
#include <cuda_runtime.h>
#include <cooperative_groups.h>
#include <cuda_fp16.h>
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstdlib>

#include "sfk_act.cuh"
#include "sfk_device.cuh"
#include "sfk_kernels.cuh"
#include "sfk_dequant.cuh"
#include "sfk_route.cuh"

namespace sfk {

// ---------------------------------------------------------------------------
// shared-memory plan of the streaming kernel (host and device agree on it)
// ---------------------------------------------------------------------------
struct StreamPlan {
  int n_stages, stage_bytes, rows_per_warp, rt, rows_tile;
  int ring_off, xq_off, acc_off, red_off, total;
  int xq_vec_bytes;
};

__host__ __device__ inline StreamPlan make_plan(const StreamParams& p) {
  StreamPlan s;
  const int U = p.K / UNIT;
  const int gb = group_bytes(p.wtype, U < GROUP_UNITS ? U : GROUP_UNITS);
  int R = (24 * 1024) / (NW * gb);
  if (R < 1) R = 1;
  if (R > 8) R = 8;
  if (p.nmat == 2 && ((NW * R) & 1)) R += 1;
  s.rows_per_warp = R;
  s.rt = NW * R;
  s.rows_tile = s.rt / p.nmat;
  s.stage_bytes = s.rt * gb;
  int ns = RING_BYTES / s.stage_bytes;
  if (ns < 2) ns = 2;
  if (ns > 8) ns = 8;
  s.n_stages = ns;
  s.ring_off = 128;
  s.xq_off = s.ring_off + ns * s.stage_bytes;
  s.xq_vec_bytes = p.xq_resident ? (int)qact_bytes(p.K) : qact_group_bytes(U < GROUP_UNITS ? U : GROUP_UNITS);
  s.acc_off = s.xq_off + ((p.n_vec * s.xq_vec_bytes + 15) & ~15);
  s.red_off = s.acc_off + ((p.rows_per_cta * p.n_pairs * p.nmat * 4 + 15) & ~15);
  s.total = s.red_off + 64 * 8;  // reduction scratch: 64 doubles / u64
  return s;
}

int stream2_smem_bytes(const StreamParams& p);

int stream_smem_bytes(const StreamParams& p, int* n_stages, int* stage_bytes, int* rows_per_warp) {
  const StreamPlan s = make_plan(p);
  if (n_stages) *n_stages = s.n_stages;
  if (stage_bytes) *stage_bytes = s.stage_bytes;
  if (rows_per_warp) *rows_per_warp = s.rows_per_warp;
  const int v2 = stream2_smem_bytes(p);
  return v2 <= 227 * 1024 ? v2 : s.total;
}

// consumer-only named barrier (the producer warp never joins it)
template <int NWS>
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"r"(NWS * 32) : "memory"); }

// Tile walk shared by producer and consumers.  Row-outer when the whole
// activation is resident in shared memory, group-outer otherwise (then the
// consumers reload one group of every activation vector per group).
struct TileWalk {
  int n_rb, n_slots, G, group_outer;
  int rb, si, g;
  __device__ void begin() { rb = 0; si = 0; g = 0; }
  __device__ bool done() const { return group_outer ? (g >= G) : (rb >= n_rb); }
  __device__ void next() {
    if (group_outer) {
      if (++si < n_slots) return;
      si = 0;
      if (++rb < n_rb) return;
      rb = 0;
      ++g;
    } else {
      if (++g < G) return;
      g = 0;
      if (++si < n_slots) return;
      si = 0;
      ++rb;
    }
  }
};

__device__ __forceinline__ int slot_expert(const StreamParams& p, int si) {
  return p.route ? p.route->slot_expert[si] : 0;
}
// Where expert e's matrices sit: e itself, or its slot of the bounded pool
// (a slot outside the pool reads slot 0 and reports).
__device__ __forceinline__ int expert_home(const StreamParams& p, int e) {
  if (!p.slot_map) return e;
  const int s = p.slot_map[e];
  if (s < 0 || s >= p.n_map_slots) {
    atomicExch(p.status, ERR_BAD_ID);
    return 0;
  }
  return s;
}

template <int WT>
__device__ __forceinline__ float unit_dot(const uint8_t* wg, const uint8_t* xg, int ng, int lane) {
  XQ8 x;
  x.load(xg, ng, lane);
  if constexpr (WT == T_Q4_K) {
    WQ4K w;
    w.load(wg, ng, lane);
    return dot_unit_q4k(w, x, lane);
  } else if constexpr (WT == T_Q6_K) {
    WQ6K w;
    w.load(wg, ng, lane);
    return dot_unit_q6k(w, x);
  } else {
    WQ80 w;
    w.load(wg, ng, lane);
    return dot_unit_q80(w, x);
  }
}

// Prologue PRO_QUANT: (RMSNorm(x) * w) or x, quantized to the activation type,
// written to shared memory for every group.  ggml rms_norm: squares summed in
// double, mean = (float)(sum/n), scale = 1/sqrtf(mean+eps), y = x*scale, then
// ggml_mul by the weight (engine.cpp:1878-1879).
struct NoOp {
  __device__ void operator()() const {}
};

// `after_loads` runs once the first vector's loads are in flight (a caller
// queues its weight copies behind them).
template <int NWS, int RB = 32 / NWS, typename F = NoOp>
__device__ void prologue_quant(const StreamParams& p, uint8_t* xq, int xq_vec_bytes, double* red,
                               F after_loads = F{}) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = p.K;
  const int nblk = K / QK_K;
  for (int t = 0; t < p.n_vec; ++t) {
    const float* x = p.x + (int64_t)t * K;
    uint8_t* qa = xq + (int64_t)t * xq_vec_bytes;
    if (nblk <= RB * NWS) {  // RB 256-column blocks per warp held in registers
      // this warp's blocks of x (and of the norm weight), one round trip
      float xv[RB][8], wv[RB][8];
#pragma unroll
      for (int i = 0; i < RB; ++i) {
        const int blk = warp + i * NWS;
        if (blk < nblk) {
          const float4* xp = reinterpret_cast<const float4*>(x + blk * QK_K + lane * 8);
          const float4 x0 = xp[0], x1 = xp[1];
          xv[i][0] = x0.x; xv[i][1] = x0.y; xv[i][2] = x0.z; xv[i][3] = x0.w;
          xv[i][4] = x1.x; xv[i][5] = x1.y; xv[i][6] = x1.z; xv[i][7] = x1.w;
          if (p.norm_w) {
            const float4* wp = reinterpret_cast<const float4*>(p.norm_w + blk * QK_K + lane * 8);
            const float4 w0 = wp[0], w1 = wp[1];
            wv[i][0] = w0.x; wv[i][1] = w0.y; wv[i][2] = w0.z; wv[i][3] = w0.w;
            wv[i][4] = w1.x; wv[i][5] = w1.y; wv[i][6] = w1.z; wv[i][7] = w1.w;
          }
        }
      }
      if (t == 0) after_loads();
      float scale = 1.0f;
      if (p.norm_w) {
        double s = 0.0;
#pragma unroll
        for (int i = 0; i < RB; ++i)
          if (warp + i * NWS < nblk) {
#pragma unroll
            for (int j = 0; j < 8; ++j) s += (double)__fmul_rn(xv[i][j], xv[i][j]);
          }
        s = warp_sum_d(s);
        if (lane == 0) red[warp] = s;
        consumer_sync<NWS>();
        double tot = 0.0;
        for (int w = 0; w < NWS; ++w) tot += red[w];  // every thread, same order
        const float mean = (float)(tot / (double)K);
        scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
        consumer_sync<NWS>();  // red is reused by the next vector
      }
      float vn[RB][8];
#pragma unroll
      for (int i = 0; i < RB; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) vn[i][j] = p.norm_w ? __fmul_rn(__fmul_rn(xv[i][j], scale), wv[i][j]) : xv[i][j];
      const int nb = warp < nblk ? (nblk - warp + NWS - 1) / NWS : 0;
      if (p.act_type == T_Q8_K) {
        qact_put_q8k_blocks<RB>(qa, K, warp, NWS, nb < RB ? nb : RB, vn, lane);
      } else {
#pragma unroll
        for (int i = 0; i < RB; ++i)
          if (i < nb) qact_put(p.act_type, qa, K, warp + i * NWS, vn[i], lane);
      }
      continue;
    }
    if (t == 0) after_loads();
    float scale = 1.0f;
    if (p.norm_w) {
      double s = 0.0;
      for (int c = tid; c < K; c += NWS * 32) {
        const float v = x[c];
        s += (double)__fmul_rn(v, v);
      }
      s = warp_sum_d(s);
      if (lane == 0) red[warp] = s;
      consumer_sync<NWS>();
      if (tid == 0) {
        double tot = 0.0;
        for (int w = 0; w < NWS; ++w) tot += red[w];
        red[NWS] = tot;
      }
      consumer_sync<NWS>();
      const float mean = (float)(red[NWS] / (double)K);
      scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
      consumer_sync<NWS>();
    }
    for (int blk = warp; blk < nblk; blk += NWS) {
      float v[8];
      const float4 a = *reinterpret_cast<const float4*>(x + blk * QK_K + lane * 8);
      const float4 b = *reinterpret_cast<const float4*>(x + blk * QK_K + lane * 8 + 4);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      if (p.norm_w) {
        const float4 wa = *reinterpret_cast<const float4*>(p.norm_w + blk * QK_K + lane * 8);
        const float4 wb = *reinterpret_cast<const float4*>(p.norm_w + blk * QK_K + lane * 8 + 4);
        const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(__fmul_rn(v[i], scale), wv[i]);
      }
      qact_put(p.act_type, qa, K, blk, v, lane);
    }
  }
}

// Copy qact vectors (all groups, or group g only) from global to shared.
template <int NWS>
__device__ void prologue_load(const StreamParams& p, uint8_t* xq, int xq_vec_bytes, int g_only) {
  const int tid = threadIdx.x;
  for (int vi = 0; vi < p.n_vec; ++vi) {
    const uint8_t* src = p.qact + (int64_t)vi * p.qact_stride;
    uint8_t* dst = xq + (int64_t)vi * xq_vec_bytes;
    int64_t nbytes;
    if (g_only < 0) {
      nbytes = qact_bytes(p.K);
    } else {
      // a group is ng * 148 bytes; round the copy up to 16 B (the bytes past
      // the group belong to the next group or to the vector's 128-byte pad)
      src += qact_group_offset(g_only);
      nbytes = (qact_group_bytes(group_units(p.K, g_only)) + 15) & ~15;
    }
    for (int64_t o = tid * 16; o < nbytes; o += NWS * 32 * 16)
      *reinterpret_cast<uint4*>(dst + o) = __ldcg(reinterpret_cast<const uint4*>(src + o));
  }
}

// ---------------------------------------------------------------------------
// epilogues
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned int ordered_f32(float v) {
  const unsigned int b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

template <int NWS>
__device__ void epi_qkv(const StreamParams& p, const float* acc, int r0, int r1) {
  const int hd = p.kv.head_dim, Hkv = p.kv.n_head_kv;
  const int nq = p.n_head * hd, nk = Hkv * hd;
  const int npair_rows = (r1 - r0) / 2;
  for (int idx = threadIdx.x; idx < npair_rows * p.b; idx += NWS * 32) {
    const int t = idx / npair_rows;
    const int r = r0 + 2 * (idx % npair_rows);
    const float x0 = acc[((r - r0) * p.n_pairs + t)];
    const float x1 = acc[((r + 1 - r0) * p.n_pairs + t)];
    const int pos = p.pos[t];
    float o0 = x0, o1 = x1;
    if (r < nq + nk) {
      // ggml rope NORMAL (engine.cpp:1892-1897): rotate (x0, x1) by theta_i,
      // theta_i = pos * theta_scale^i; cos/sin come from a host-built table
      // evaluated exactly like ggml's rope cache
      const int i = (r % hd) >> 1;
      const float2 cs = reinterpret_cast<const float2*>(p.rope)[(int64_t)pos * (hd >> 1) + i];
      o0 = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
      o1 = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
    }
    if (r < nq) {
      p.y[(int64_t)t * nq + r] = o0;
      p.y[(int64_t)t * nq + r + 1] = o1;
    } else {
      const bool is_k = r < nq + nk;
      const int rr = r - nq - (is_k ? 0 : nk);
      const int h = rr / hd, i0 = rr % hd;
      const int page = p.kv.page_table[t * p.kv.max_pages + pos / 16];
      if (!kv_page_writable(p.kv, page)) {  // never write outside the pool
        atomicExch(p.status, ERR_BAD_PAGE);
        continue;
      }
      const int64_t off = (((int64_t)page * Hkv + h) * 16 + (pos & 15)) * hd + i0;
      void* base = is_k ? p.kv.k : p.kv.v;
      if (p.kv.f16) {
        __half* kb = reinterpret_cast<__half*>(base);
        kb[off] = __float2half_rn(o0);
        kb[off + 1] = __float2half_rn(o1);
      } else {
        float* kb = reinterpret_cast<float*>(base);
        kb[off] = o0;
        kb[off + 1] = o1;
      }
    }
  }
}

template <int NWS>
__device__ void epi_gateup(const StreamParams& p, const float* acc, int r0, int r1, int* flags) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nr = r1 - r0;
  // h = silu(gate) * up  (ggml_swiglu_split(gate, up), engine.cpp:1969)
  for (int idx = tid; idx < nr * p.n_pairs; idx += NWS * 32) {
    const int row = idx % nr, pr = idx / nr;
    const float g = acc[(row * p.n_pairs + pr) * 2 + 0];
    const float u = acc[(row * p.n_pairs + pr) * 2 + 1];
    const float sl = __fdiv_rn(g, __fadd_rn(1.0f, sfk_expf(-g)));
    p.h[(int64_t)pr * p.rows + r0 + row] = __fmul_rn(sl, u);
  }
  __threadfence();
  consumer_sync<NWS>();
  // 256-row groups completed by this CTA's rows get requantized (Q8_K / Q8_0)
  // by whichever CTA adds the last rows to the group's counter.
  const int q0 = r0 / QK_K, q1 = (r1 - 1) / QK_K;
  if (tid == 0) {
    for (int q = q0; q <= q1; ++q) {
      const int lo = max(r0, q * QK_K), hi = min(r1, (q + 1) * QK_K);
      const int old = atomicAdd(&p.grp_counter[q], hi - lo);
      flags[q - q0] = (old + (hi - lo) == QK_K) ? 1 : 0;
    }
  }
  consumer_sync<NWS>();
  for (int q = q0; q <= q1; ++q) {
    if (!flags[q - q0]) continue;
    __threadfence();
    for (int pr = warp; pr < p.n_pairs; pr += NWS) {
      const float* hp = p.h + (int64_t)pr * p.rows + q * QK_K + lane * 8;
      const float4 a = __ldcg(reinterpret_cast<const float4*>(hp));
      const float4 b = __ldcg(reinterpret_cast<const float4*>(hp + 4));
      const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
      qact_put(p.h_act_type, p.hq + (int64_t)pr * qact_bytes(p.rows), p.rows, q, v, lane);
    }
    if (tid == 0) atomicExch(&p.grp_counter[q], 0);
  }
}

template <int NWS>
__device__ void epi_down(const StreamParams& p, const float* acc, int r0, int r1) {
  const int nr = r1 - r0;
  const int k = p.k;
  for (int idx = threadIdx.x; idx < nr * p.b; idx += NWS * 32) {
    const int row = idx % nr, t = idx / nr;
    // experts * weights, then moe_out = e0 + e1 + ..., then + ffn_inp
    // (engine.cpp:1973-1986)
    float a;
    if (p.ep_eloc == 0) {
      a = __fmul_rn(acc[row * p.n_pairs + t * k], p.route->w[t * k]);
      for (int j = 1; j < k; ++j) a = __fadd_rn(a, __fmul_rn(acc[row * p.n_pairs + t * k + j], p.route->w[t * k + j]));
    } else {  // this rank's experts only; the ranks' partials are added by the combine
      a = 0.0f;
      for (int j = 0; j < k; ++j) {
        const int id = p.route->ids[t * k + j];
        if (id >= p.ep_e0 && id < p.ep_e0 + p.ep_eloc)
          a = __fadd_rn(a, __fmul_rn(acc[row * p.n_pairs + t * k + j], p.route->w[t * k + j]));
      }
    }
    if (p.res) a = __fadd_rn(a, p.res[(int64_t)t * p.rows + r0 + row]);
    p.y[(int64_t)t * p.y_stride + r0 + row] = a;
  }
}

template <int NWS>
__device__ void epi_lmhead(const StreamParams& p, const float* acc, int r0, int r1, unsigned long long* red) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nr = r1 - r0;
  for (int t = 0; t < p.b; ++t) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int row = tid; row < nr; row += NWS * 32) {
      const float v = acc[row * p.n_pairs + t];
      if (p.store_logits) p.y[(int64_t)t * p.y_stride + r0 + row] = v;
      if (v > best) { best = v; bi = p.argmax_base + r0 + row; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if (lane == 0)
      red[warp] = bi == 0x7fffffff ? 0ull
                                   : (((unsigned long long)ordered_f32(best) << 32) |
                                      (unsigned long long)(0xFFFFFFFFu - (unsigned)bi));
    consumer_sync<NWS>();
    if (tid == 0) {
      unsigned long long m = 0;
      for (int w = 0; w < NWS; ++w) m = red[w] > m ? red[w] : m;
      if (m) atomicMax(&p.argmax_key[t], m);
    }
    consumer_sync<NWS>();
  }
}

template <int NWS>
__device__ void run_epilogue(const StreamParams& p, const float* acc, int r0, int r1, double* red) {
  switch (p.epi) {
    case EPI_STORE: {
      const int nr = r1 - r0;
      for (int idx = threadIdx.x; idx < nr * p.n_pairs; idx += NWS * 32) {
        const int row = idx % nr, pr = idx / nr;
        p.y[(int64_t)pr * p.y_stride + r0 + row] = acc[row * p.n_pairs + pr];
      }
      break;
    }
    case EPI_RESID: {
      const int nr = r1 - r0;
      for (int idx = threadIdx.x; idx < nr * p.b; idx += NWS * 32) {
        const int row = idx % nr, t = idx / nr;
        const float v = acc[row * p.n_pairs + t];
        p.y[(int64_t)t * p.y_stride + r0 + row] = p.res ? __fadd_rn(v, p.res[(int64_t)t * p.y_stride + r0 + row]) : v;
      }
      break;
    }
    case EPI_QKV: epi_qkv<NWS>(p, acc, r0, r1); break;
    case EPI_GATEUP: epi_gateup<NWS>(p, acc, r0, r1, reinterpret_cast<int*>(red)); break;
    case EPI_DOWN: epi_down<NWS>(p, acc, r0, r1); break;
    case EPI_LMHEAD: epi_lmhead<NWS>(p, acc, r0, r1, reinterpret_cast<unsigned long long*>(red)); break;
    default: break;
  }
}

// ---------------------------------------------------------------------------
// the streaming kernel
// ---------------------------------------------------------------------------
template <int WT>
__global__ void __launch_bounds__((NW + 1) * 32, 1) stream_kernel(const StreamParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const StreamPlan pl = make_plan(p);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + pl.n_stages;
  uint8_t* ring = smem + pl.ring_off;
  uint8_t* xq = smem + pl.xq_off;
  float* acc = reinterpret_cast<float*>(smem + pl.acc_off);
  double* red = reinterpret_cast<double*>(smem + pl.red_off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = blockIdx.x * p.rows_per_cta;
  const int r1 = min(p.rows, r0 + p.rows_per_cta);
  const int G = n_groups(p.K);
  const int ng_full = group_units(p.K, 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < pl.n_stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NW);
    }
    fence_mbar_init();
  }
  __syncthreads();

  TileWalk tw;
  tw.n_rb = r0 < r1 ? (r1 - r0 + pl.rows_tile - 1) / pl.rows_tile : 0;
  tw.G = G;
  tw.group_outer = p.xq_resident ? 0 : 1;
  tw.n_slots = 1;

  if (warp == NW) {
    // ------------------------------ producer ------------------------------
    if (lane != 0) return;
    bool waited = false;
    if (p.route) {
      pdl_wait();  // routed experts are known only after the router ran
      pdl_launch_dependents();
      waited = true;
      tw.n_slots = p.route->n_slots;
    }
    uint32_t it = 0;
    for (tw.begin(); !tw.done(); tw.next(), ++it) {
      const int s = it % pl.n_stages;
      if (it >= (uint32_t)pl.n_stages) {
        if (!waited) {  // the ring is full: from here on the consumers pace the copies
          pdl_wait();
          pdl_launch_dependents();
          waited = true;
        }
        if (!mbar_wait_bounded(&empty[s], ((it / pl.n_stages) - 1) & 1, p.status)) break;
      }
      const int ng = group_units(p.K, tw.g);
      const int gb = group_bytes(WT, ng);
      const int rbase = r0 + tw.rb * pl.rows_tile;
      const int nrows = min(pl.rows_tile, r1 - rbase);
      mbar_arrive_expect_tx(&full[s], (uint32_t)(nrows * p.nmat * gb));
      const int64_t eoff =
          (int64_t)expert_home(p, slot_expert(p, tw.si)) * p.expert_stride + group_offset(WT, p.K, tw.g);
      uint8_t* dst = ring + (int64_t)s * pl.stage_bytes;
      for (int m = 0; m < p.nmat; ++m) {
        const uint8_t* base = (m == 0 ? p.w0 : p.w1) + eoff;
        for (int r = 0; r < nrows; ++r)
          bulk_g2s(dst + (m * pl.rows_tile + r) * gb, base + (int64_t)(rbase + r) * p.rowstride, gb, &full[s]);
      }
    }
    if (!waited) {
      pdl_wait();
      pdl_launch_dependents();
    }
    return;
  }

  // ------------------------------ consumers ------------------------------
  pdl_wait();
  pdl_launch_dependents();
  if (p.clear_keys && blockIdx.x == 0 && threadIdx.x < p.clear_n) p.clear_keys[threadIdx.x] = 0ull;
  const int nacc = (r1 > r0 ? (r1 - r0) : 0) * p.n_pairs * p.nmat;
  for (int i = threadIdx.x; i < nacc; i += NW * 32) acc[i] = 0.0f;
  if (p.route) tw.n_slots = p.route->n_slots;
  if (p.xq_resident) {
    if (p.pro == PRO_QUANT)
      prologue_quant<NW>(p, xq, pl.xq_vec_bytes, red);
    else
      prologue_load<NW>(p, xq, pl.xq_vec_bytes, -1);
  }
  consumer_sync<NW>();

  uint32_t it = 0;
  int cur_g = -1;
  bool ok = true;
  for (tw.begin(); !tw.done(); tw.next(), ++it) {
    if (!p.xq_resident && tw.g != cur_g) {
      consumer_sync<NW>();
      prologue_load<NW>(p, xq, pl.xq_vec_bytes, tw.g);
      consumer_sync<NW>();
      cur_g = tw.g;
    }
    const int s = it % pl.n_stages;
    if (!mbar_wait_bounded(&full[s], (it / pl.n_stages) & 1, p.status)) { ok = false; break; }
    const int ng = group_units(p.K, tw.g);
    const int gb = group_bytes(WT, ng);
    const int rbase = r0 + tw.rb * pl.rows_tile;
    const uint8_t* tile = ring + (int64_t)s * pl.stage_bytes;
    int pb = 0, pe = p.b;
    if (p.route) { pb = p.route->slot_off[tw.si]; pe = p.route->slot_off[tw.si + 1]; }
    const int xq_goff = p.xq_resident ? (int)qact_group_offset(tw.g) : 0;
    for (int i = 0; i < pl.rows_per_warp; ++i) {
      const int rm = warp + NW * i;
      const int m = rm / pl.rows_tile;
      const int row = rbase + rm % pl.rows_tile;
      if (row >= r1) continue;
      const uint8_t* wg = tile + rm * gb;
      for (int pi = pb; pi < pe; ++pi) {
        const int pair = p.route ? p.route->slot_pairs[pi] : pi;
        const int vi = p.xq_by_pair ? pair : (p.route ? pair / p.k : pair);
        float part = 0.0f;
        if (lane < ng) part = unit_dot<WT>(wg, xq + (int64_t)vi * pl.xq_vec_bytes + xq_goff, ng, lane);
        part = warp_sum(part);
        if (lane == 0) acc[((row - r0) * p.n_pairs + pair) * p.nmat + m] += part;
      }
    }
    // the slot's generic reads are ordered before the bulk copy that refills it
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  (void)ng_full;
  (void)ok;
  consumer_sync<NW>();
  if (*(volatile int*)p.status == ERR_TIMEOUT || r0 >= r1) return;  // uniform across the consumers

  run_epilogue<NW>(p, acc, r0, r1, red);
}

// ---------------------------------------------------------------------------
// stream2_kernel: warp-owned tiles, each warp its own copy issuer.  A tile is
// R consecutive full rows (all groups of K) of each of the nmat matrices of
// one expert; tiles go to the consumer warps round-robin and every warp keeps
// S of its tiles in flight in its own ring slots, issuing the next tile's bulk
// copies itself as soon as it is done with a slot.  One thread can keep only
// about one 1-D bulk copy per quarter microsecond going, so a single producer
// thread caps the SM at ~1.1 TB/s/148 with 2 KB copies; eight issuing warps
// stream at HBM speed with 2-8 KB copies.  The row sums keep the fixed order
// of the other kernel (unit partials -> 32-lane butterfly per group -> groups
// added in order): the butterflies of a tile's up to 8 (row, matrix, group)
// values run together (9 shuffles instead of 40), then each (row, matrix)
// adds its group sums in order.
// ---------------------------------------------------------------------------
constexpr int S2_MAXSTAGES = 4;
constexpr int S2_TILE = 16 * 1024;  // default tile target (bytes)
constexpr int S2_SMEM = 227 * 1024;

__host__ __device__ inline int al16i(int64_t v) { return (int)((v + 15) & ~(int64_t)15); }

inline Plan2 make_plan2(const StreamParams& p, int NWS, int occ) {
  Plan2 q;
  q.nws = NWS;
  q.occ = occ;
  const int S2_BUDGET = occ == 2 ? 113 * 1024 : S2_SMEM;
  const int64_t rs = p.rowstride;
  q.G = n_groups(p.K);
  const int64_t xq_all = (int64_t)p.n_vec * qact_bytes(p.K);
  q.xq_smem = (p.pro == PRO_QUANT) || (p.pro == PRO_ROUTE) || (xq_all <= 64 * 1024) ? 1 : 0;
  q.xq_vec_bytes = (int)qact_bytes(p.K);
  const bool rt = p.pro == PRO_ROUTE;
  const bool routed = rt || p.route != nullptr;  // the routing is kept in shared memory
  const int xq_b = q.xq_smem ? al16i(xq_all) : 0;
  const int acc_b = al16i((int64_t)p.rows_per_cta * p.n_pairs * p.nmat * 4);
  const int route_b = (routed ? al16i(sizeof(Route)) : 0) + (rt ? p.K * 4 + al16i(p.b * p.n_expert * 4) : 0);
  const int bars = al16i(NWS * S2_MAXSTAGES * 8 + 16);  // per-warp full[] | router-weights | prologue
  const int fixed = bars + xq_b + acc_b + 64 * 8 + route_b;
  int rmax = 8 / (p.nmat * q.G);
  if (rmax < 1) rmax = 1;
  int R = (int)((p.s2_tile > 0 ? p.s2_tile : S2_TILE) / (p.nmat * rs));
  R = R < 1 ? 1 : (R > rmax ? rmax : R);
  // bigger tiles over deeper rings: with 16 warps each holding one tile,
  // the per-tile work (butterfly, bookkeeping, copy issue) amortises over
  // more rows (measured: gate/up 43 -> 39 us, QKV 12.5 -> 11.2 us)
  const int min_stages = p.s2_stages >= 2 ? 2 : 1;
  while (R > 1 && (S2_BUDGET - fixed) / ((int64_t)NWS * p.nmat * R * rs) < min_stages) --R;
  q.R = R;
  q.tile_bytes = (int)(p.nmat * R * rs);
  int S = (int)((S2_BUDGET - fixed) / ((int64_t)NWS * q.tile_bytes));
  if (S > S2_MAXSTAGES) S = S2_MAXSTAGES;
  if (p.s2_stages > 0 && S > p.s2_stages) S = p.s2_stages;
  if (S < 1) S = 1;
  q.stages = S;
  q.ring_off = bars;
  q.xq_off = q.ring_off + NWS * S * q.tile_bytes;
  q.acc_off = q.xq_off + xq_b;
  q.red_off = q.acc_off + acc_b;
  q.route_off = q.red_off + 64 * 8;
  q.xn_off = q.route_off + (routed ? al16i(sizeof(Route)) : 0);
  q.seg_off = q.xn_off + (rt ? p.K * 4 : 0);
  q.probs_off = q.seg_off;
  q.total = q.probs_off + (rt ? al16i(p.b * p.n_expert * 4) : 0);
  return q;
}

template <int NWS>
struct ConsumerSync {
  __device__ void operator()() const { consumer_sync<NWS>(); }
};

// Sum 8 lane-distributed values over the warp with the 32-lane butterfly
// (p + p^16, then ^8, ^4, ^2, ^1) applied to each value, exchanging two values
// per shuffle while lanes still split them.  Value v ends in the lanes with
// bit 2 = v>>2, bit 3 = (v>>1)&1, bit 4 = v&1.
__device__ __forceinline__ float reduce8(const float v[8], int lane) {
  const bool b16 = lane & 16, b8 = lane & 8, b4 = lane & 4;
  float w[4], x[2];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float A = v[2 * i], B = v[2 * i + 1];
    const float r = __shfl_xor_sync(0xffffffffu, b16 ? A : B, 16);
    w[i] = b16 ? __fadd_rn(B, r) : __fadd_rn(A, r);
  }
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const float A = w[2 * j], B = w[2 * j + 1];
    const float r = __shfl_xor_sync(0xffffffffu, b8 ? A : B, 8);
    x[j] = b8 ? __fadd_rn(B, r) : __fadd_rn(A, r);
  }
  float y;
  {
    const float r = __shfl_xor_sync(0xffffffffu, b4 ? x[0] : x[1], 4);
    y = b4 ? __fadd_rn(x[1], r) : __fadd_rn(x[0], r);
  }
  y = __fadd_rn(y, __shfl_xor_sync(0xffffffffu, y, 2));
  y = __fadd_rn(y, __shfl_xor_sync(0xffffffffu, y, 1));
  return y;
}

// shared memory of the warp-tile kernel, or more than any SM has when a tile
// cannot hold all of one row's group sums (nmat * groups > 8)
// Warp count and plan of the warp-tile kernel: 16 consumer warps when their
// rings fit, else 8 (SFK_STREAM_WARPS forces 8 or 16);
// nws = 0 when a tile cannot hold all of one row's group sums or the rings
// do not fit.
static int stream_warps_forced() {
  static const int v = [] {
    const char* e = getenv("SFK_STREAM_WARPS");
    return e ? atoi(e) : 0;
  }();
  return v;
}
Plan2 choose_plan2(const StreamParams& p) {
  Plan2 none{};
  none.nws = 0;
  if (p.nmat != 1 && p.nmat != 2) return none;
  if (p.s2_occ == 2) {  // two 8-warp CTAs per SM
    const Plan2 q = make_plan2(p, 8, 2);
    if (p.nmat * q.G <= 8 && q.total <= 113 * 1024) return q;
    return none;
  }
  // 16 warps whenever their rings fit, even with one slot each: sixteen
  // warps with one tile in flight beat eight with two (measured on the
  // Mixtral down projection, 8 KB rows)
  const int forced = stream_warps_forced();
  for (int nws : {16, 8}) {
    if (forced && forced != nws) continue;
    const Plan2 q = make_plan2(p, nws, 1);
    if (p.nmat * q.G > 8 || q.total > S2_SMEM) continue;
    return q;
  }
  return none;
}

int stream2_occupancy(const StreamParams& p) {
  const Plan2 q = choose_plan2(p);
  return q.nws ? q.occ : 0;
}

// shared memory of the warp-tile kernel, or more than any SM has when it
// cannot run the launch
int stream2_smem_bytes(const StreamParams& p) {
  const Plan2 q = choose_plan2(p);
  return q.nws ? q.total : 1 << 30;
}

template <int WT>
__device__ __forceinline__ float unit_dot_x(const uint8_t* wg, const XQ8& x, int ng, int lane) {
  if constexpr (WT == T_Q4_K) {
    WQ4K w;
    w.load(wg, ng, lane);
    return dot_unit_q4k(w, x, lane);
  } else if constexpr (WT == T_Q6_K) {
    WQ6K w;
    w.load(wg, ng, lane);
    return dot_unit_q6k(w, x);
  } else {
    WQ80 w;
    w.load(wg, ng, lane);
    return dot_unit_q80(w, x);
  }
}

template <int WT, int NMAT, int NWS, int MINB>
__global__ void __launch_bounds__(NWS * 32, MINB) stream2_kernel(const StreamParams p) {
  constexpr int RBV = MINB >= 2 ? 2 : 32 / NWS;  // register blocks of the activation prologues
  extern __shared__ __align__(128) uint8_t smem[];
  const Plan2& pl = p.pl;  // planned on the host: no divisions before the first copy
  const int S = pl.stages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem) + warp * S;  // this warp's [S]
  uint64_t* pro_bar = reinterpret_cast<uint64_t*>(smem) + NWS * S2_MAXSTAGES;  // prologue copies landed
  uint8_t* ring_all = smem + pl.ring_off;
  uint8_t* ring = ring_all + (int64_t)warp * S * pl.tile_bytes;
  uint8_t* xq_s = smem + pl.xq_off;
  float* acc = reinterpret_cast<float*>(smem + pl.acc_off);
  double* red = reinterpret_cast<double*>(smem + pl.red_off);
  Route* sroute = reinterpret_cast<Route*>(smem + pl.route_off);
  const bool self_route = p.pro == PRO_ROUTE;
  const bool routed = self_route || p.route != nullptr;
  const Route* rt = sroute;  // the routing, in shared memory once known
  const int r0 = blockIdx.x * p.rows_per_cta;
  const int r1 = min(p.rows, r0 + p.rows_per_cta);
  const int G = pl.G;
  const int R = pl.R;
  const int64_t rs = p.rowstride;
  const int n_rb = r0 < r1 ? (r1 - r0 + R - 1) / R : 0;

  if (lane == 0) {
    for (int i = 0; i < S; ++i) mbar_init(&full[i], 1);
    if (warp == 0) mbar_init(pro_bar, NWS);
    fence_mbar_init();
  }
  __syncthreads();
  // lane 0: bring tile `it` (row block it / n_slots of slot expert it % n_slots) into ring slot s
  auto issue = [&](int it, int s, int n_slots) {
    const int rb = it / n_slots, si = it % n_slots;
    const int rbase = r0 + rb * R;
    const uint32_t bytes = (uint32_t)(min(R, r1 - rbase) * rs);
    mbar_arrive_expect_tx(&full[s], bytes * NMAT);
    const int expert = routed ? expert_home(p, rt->slot_expert[si]) : 0;
    const int64_t eoff = (int64_t)expert * p.expert_stride + (int64_t)rbase * rs;
    uint8_t* dst = ring + (int64_t)s * pl.tile_bytes;
    const uint64_t pol = l2_evict_first_policy();
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
      bulk_g2s_hint(dst + (int64_t)m * R * rs, (m == 0 ? p.w0 : p.w1) + eoff, bytes, &full[s], pol);
  };

  // routing: CTA c scores the (token, expert) logits q = c, c + grid, ...;
  // the router weights are static, so the first row slice is loaded before
  // the wait on the previous kernel
  const int nq = self_route ? p.b * p.n_expert : 0;
  // columns of a logit per warp: a multiple of 4 (16-byte loads), the last
  // warp's range clipped at K
  const int rcols = ((p.K + NWS - 1) / NWS + 3) & ~3;
  const int rc0 = min(p.K, warp * rcols), rc1 = min(p.K, rc0 + rcols);
  // When the whole router fits in the ring (idle until the experts are
  // known), every CTA copies it in before the wait and scores all logits
  // itself: no exchange between CTAs.
  const bool wr_local = self_route && (int64_t)p.n_expert * p.K * 4 <= (int64_t)NWS * S * pl.tile_bytes;
  float* wr_s = reinterpret_cast<float*>(smem + pl.ring_off);
  if (wr_local && lane == 0) {
    uint32_t mine = 0;
    for (int e = warp; e < p.n_expert; e += NWS) mine += (uint32_t)(p.K * 4);
    mbar_arrive_expect_tx(pro_bar, mine);
    for (int e = warp; e < p.n_expert; e += NWS)
      bulk_g2s(wr_s + (int64_t)e * p.K, p.w_r + (int64_t)e * p.K, (uint32_t)(p.K * 4), pro_bar);
  }
  constexpr int WPRE = 4;
  float4 wpre[WPRE];
  const bool pre = !wr_local && (int)blockIdx.x < nq && rcols % 128 == 0 && rcols / 128 <= WPRE &&
                   rc1 - rc0 == rcols;
  if (pre) {
    const float* wr = p.w_r + (int64_t)(blockIdx.x % p.n_expert) * p.K + rc0 + lane * 4;
#pragma unroll
    for (int i = 0; i < WPRE; ++i)
      if (i < rcols / 128) wpre[i] = *reinterpret_cast<const float4*>(wr + i * 128);
  }
  // An unrouted matrix's weights do not depend on the previous kernel: with
  // early_fill its first ring fill goes out before the wait.  The CTAs of a
  // kernel can be resident long before their predecessor ends (the output
  // projection's beside the attention's), and the fill then lands in that
  // time instead of after it.
  const bool early = p.early_fill && !routed;
  if (early && lane == 0)
    for (int k = 0; k < S && warp + k * NWS < n_rb; ++k) issue(warp + k * NWS, k, 1);
  pdl_wait();
  pdl_launch_dependents();
  // inputs written by the previous kernels: the routing (when another kernel
  // routed) and precomputed activations, by bulk copies issued from every warp
  const bool bulk_xq = !self_route && p.pro == PRO_LOAD && pl.xq_smem && (p.qact_stride % 16) == 0 &&
                       (reinterpret_cast<uintptr_t>(p.qact) % 16) == 0;
  const bool bulk_pro = bulk_xq || (routed && !self_route);
  if (bulk_pro && lane == 0) {
    uint32_t mine = 0;
    if (routed && !self_route && warp == 0) mine += (uint32_t)sizeof(Route);
    if (bulk_xq)
      for (int vi = warp; vi < p.n_vec; vi += NWS) mine += (uint32_t)pl.xq_vec_bytes;
    mbar_arrive_expect_tx(pro_bar, mine);
    if (routed && !self_route && warp == 0) bulk_g2s(sroute, p.route, (uint32_t)sizeof(Route), pro_bar);
    if (bulk_xq)
      for (int vi = warp; vi < p.n_vec; vi += NWS)
        bulk_g2s(xq_s + (int64_t)vi * pl.xq_vec_bytes, p.qact + (int64_t)vi * p.qact_stride,
                 (uint32_t)pl.xq_vec_bytes, pro_bar);
  }
  if (p.clear_keys && blockIdx.x == 0 && threadIdx.x < p.clear_n) p.clear_keys[threadIdx.x] = 0ull;
  int depart_old = -1;
  if (self_route && wr_local) {
    float* xn_s = reinterpret_cast<float*>(smem + pl.xn_off);
    float* probs_s = reinterpret_cast<float*>(smem + pl.probs_off);  // [b][E]
    for (int t = 0; t < p.b; ++t) {
      route_norm<NWS, RBV>(p.x + (int64_t)t * p.K, p.norm_w, p.K, p.eps, p.act_type, xq_s + (int64_t)t * pl.xq_vec_bytes,
                           xn_s, red, nullptr, ConsumerSync<NWS>{});
      if (t == 0) mbar_wait_bounded(pro_bar, 0, p.status);  // the router rows are in
      // logit e = sum_c (double)(w_r[e][c] * xn[c]); with at least two
      // warps per expert each takes half the columns (four chains each), the
      // halves added in order
      const int wpe = (p.n_expert * 2 <= NWS && p.n_expert * 2 <= 64) ? 2 : 1;
      const int span = p.K / wpe;
      for (int item = warp; item < p.n_expert * wpe; item += NWS) {
        const int e = item / wpe, part = item % wpe;
        const float* wr = wr_s + (int64_t)e * p.K + part * span;
        const float* xs = xn_s + part * span;
        double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
        for (int c = lane * 4; c < span; c += 128) {
          const float4 w4 = *reinterpret_cast<const float4*>(wr + c);
          const float4 x4 = *reinterpret_cast<const float4*>(xs + c);
          a0 += (double)__fmul_rn(w4.x, x4.x);
          a1 += (double)__fmul_rn(w4.y, x4.y);
          a2 += (double)__fmul_rn(w4.z, x4.z);
          a3 += (double)__fmul_rn(w4.w, x4.w);
        }
        const double a = warp_sum_d((a0 + a1) + (a2 + a3));
        if (wpe == 1) {
          if (lane == 0) probs_s[t * p.n_expert + e] = (float)a;
        } else if (lane == 0) {
          red[item] = a;
        }
      }
      consumer_sync<NWS>();
      if (wpe == 2)
        for (int e = threadIdx.x; e < p.n_expert; e += NWS * 32)
          probs_s[t * p.n_expert + e] = (float)(red[2 * e] + red[2 * e + 1]);
      consumer_sync<NWS>();  // xn and red are rewritten by the next token
    }
    for (int t = warp; t < p.b; t += NWS)
      route_select(probs_s + t * p.n_expert, p.n_expert, p.k, &sroute->ids[t * p.k], &sroute->w[t * p.k], lane);
    consumer_sync<NWS>();
    if (p.b * p.k <= 32 && (p.ep_eloc > 0 ? p.ep_eloc : p.n_expert) <= 64) {
      if (warp == 0) build_slots_warp(sroute->ids, p.b * p.k, sroute, lane, p.ep_e0, p.ep_eloc);
    } else if (threadIdx.x == 0) {
      build_slots(sroute->ids, p.b * p.k, sroute, p.ep_e0, p.ep_eloc);
    }
    if (threadIdx.x == 0) {
      sroute->k = p.k;
      sroute->b = p.b;
    }
    consumer_sync<NWS>();
    if (blockIdx.x == 0) {  // publish the routing for the down kernel and the host
      const int* src = reinterpret_cast<const int*>(sroute);
      int* dst = reinterpret_cast<int*>(const_cast<Route*>(p.route));
      for (int i = threadIdx.x; i < (int)(sizeof(Route) / 4); i += NWS * 32) dst[i] = src[i];
    }
  } else if (self_route) {
    float* xn_s = reinterpret_cast<float*>(smem + pl.xn_off);
    float* probs_s = reinterpret_cast<float*>(smem + pl.probs_off);  // [b][E]
    const int tid = threadIdx.x;
    for (int t = 0; t < p.b; ++t) {
      // ffn_norm + quantize token t (every CTA needs its activations)
      route_norm<NWS, RBV>(p.x + (int64_t)t * p.K, p.norm_w, p.K, p.eps, p.act_type, xq_s + (int64_t)t * pl.xq_vec_bytes,
                     xn_s, red, nullptr, ConsumerSync<NWS>{});
      for (int q = blockIdx.x; q < nq; q += gridDim.x) {
        if (q / p.n_expert != t) continue;
        // logit = sum_c (double)(w_r[e][c] * xn[c]): warp w sums its column
        // slice in four chains, the slices are added in order
        const float* wr = p.w_r + (int64_t)(q % p.n_expert) * p.K + rc0;
        const float* xs = xn_s + rc0;
        double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
        if (pre && q == (int)blockIdx.x) {
#pragma unroll
          for (int i = 0; i < WPRE; ++i)
            if (i < rcols / 128) {
              const float4 x4 = *reinterpret_cast<const float4*>(xs + i * 128 + lane * 4);
              a0 += (double)__fmul_rn(wpre[i].x, x4.x);
              a1 += (double)__fmul_rn(wpre[i].y, x4.y);
              a2 += (double)__fmul_rn(wpre[i].z, x4.z);
              a3 += (double)__fmul_rn(wpre[i].w, x4.w);
            }
        } else {
          for (int c = lane * 4; c < rc1 - rc0; c += 128) {
            const float4 w4 = *reinterpret_cast<const float4*>(wr + c);
            const float4 x4 = *reinterpret_cast<const float4*>(xs + c);
            a0 += (double)__fmul_rn(w4.x, x4.x);
            a1 += (double)__fmul_rn(w4.y, x4.y);
            a2 += (double)__fmul_rn(w4.z, x4.z);
            a3 += (double)__fmul_rn(w4.w, x4.w);
          }
        }
        const double a = warp_sum_d((a0 + a1) + (a2 + a3));
        if (lane == 0) red[warp] = a;
        consumer_sync<NWS>();
        if (tid == 0) {
          double tot = 0.0;
          for (int w = 0; w < NWS; ++w) tot += red[w];
          p.logits[q] = (float)tot;
          __threadfence();
          atomicAdd(&p.rsync[0], 1);  // release: this logit is visible
        }
        consumer_sync<NWS>();
      }
    }
    // every logit of the step, from every scoring CTA (bounded wait)
    if (tid == 0) {
      const long long t0 = clock64();
      while (ld_acquire(&p.rsync[0]) < nq) {
        __nanosleep(64);
        if (clock64() - t0 > (1ll << 31)) {
          atomicExch(p.status, ERR_TIMEOUT);
          break;
        }
      }
    }
    consumer_sync<NWS>();
    for (int i = tid; i < nq; i += NWS * 32) probs_s[i] = __ldcg(&p.logits[i]);
    consumer_sync<NWS>();
    for (int t = warp; t < p.b; t += NWS)
      route_select(probs_s + t * p.n_expert, p.n_expert, p.k, &sroute->ids[t * p.k], &sroute->w[t * p.k], lane);
    consumer_sync<NWS>();
    if (tid == 0) {
      build_slots(sroute->ids, p.b * p.k, sroute, p.ep_e0, p.ep_eloc);
      sroute->k = p.k;
      sroute->b = p.b;
      // departure count; its result is looked at only when the CTA is done,
      // so the round trip stays off the critical path
      depart_old = atomicAdd(&p.rsync[1], 1);
    }
    consumer_sync<NWS>();
    if (blockIdx.x == 0) {  // publish the routing for the down kernel and the host
      const int* src = reinterpret_cast<const int*>(sroute);
      int* dst = reinterpret_cast<int*>(const_cast<Route*>(p.route));
      for (int i = threadIdx.x; i < (int)(sizeof(Route) / 4); i += NWS * 32) dst[i] = src[i];
    }
  } else if (bulk_pro) {
    mbar_wait_bounded(pro_bar, 0, p.status);  // routing and/or activations are in shared memory
  }
  const int n_slots = routed ? rt->n_slots : 1;
  const int n_tiles = n_rb * n_slots;
  if (routed && lane == 0) {  // the routed experts are known now
    for (int k = 0; k < S && warp + k * NWS < n_tiles; ++k) issue(warp + k * NWS, k, n_slots);
  }
  // the first ring fill of an unrouted matrix goes out right behind the
  // activation loads (copied ahead of them, it would delay them by the time
  // the whole GPU's first fill takes to drain)
  auto first_fill = [&]() {
    if (!routed && !early && lane == 0)
      for (int k = 0; k < S && warp + k * NWS < n_tiles; ++k) issue(warp + k * NWS, k, 1);
  };
  if (!self_route && pl.xq_smem && p.pro == PRO_QUANT) {
    prologue_quant<NWS, RBV>(p, xq_s, pl.xq_vec_bytes, red, first_fill);
  } else {
    first_fill();
    if (!self_route && pl.xq_smem && !bulk_xq) prologue_load<NWS>(p, xq_s, pl.xq_vec_bytes, -1);
  }
  consumer_sync<NWS>();
  const uint8_t* xbase = pl.xq_smem ? xq_s : p.qact;
  const int64_t xstride = pl.xq_smem ? (int64_t)pl.xq_vec_bytes : p.qact_stride;
  XQ8 xc;
  int cached = -1;  // vi * G + g of the activation group in xc
  for (int kk = 0, it = warp; it < n_tiles; ++kk, it += NWS) {
    const int s = kk % S;
    if (!mbar_wait_bounded(&full[s], (kk / S) & 1, p.status)) break;
    const int rb = it / n_slots, si = it % n_slots;
    const int rbase = r0 + rb * R;
    const int nrows = min(R, r1 - rbase);
    const int RM = nrows * NMAT;  // (row, matrix) pairs; values v = rm * G + g
    const uint8_t* tile = ring + (int64_t)s * pl.tile_bytes;
    int pb = 0, pe = p.b;
    if (routed) { pb = rt->slot_off[si]; pe = rt->slot_off[si + 1]; }
    for (int pi = pb; pi < pe; ++pi) {
      const int pair = routed ? rt->slot_pairs[pi] : pi;
      const int vi = p.xq_by_pair ? pair : (routed ? pair / p.k : pair);
      float part[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) part[j] = 0.0f;
      if (G == 1 && RM == 4) {
        // the common tile (4 row-matrices of one 32-unit group): four
        // independent unit dots in one basic block, so their dp4a chains
        // interleave
        const int ng = group_units(p.K, 0);
        if (vi != cached) {
          if (lane < ng) {
            const uint8_t* xg = xbase + (int64_t)vi * xstride;
            if (pl.xq_smem)
              xc.load(xg, ng, lane);
            else
              xc.load_any(xg, ng, lane);
          }
          cached = vi;
        }
        if (lane < ng) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int r = NMAT == 2 ? (q >> 1) : q, m = NMAT == 2 ? (q & 1) : 0;
            part[q] = unit_dot_x<WT>(tile + ((int64_t)m * R + r) * rs, xc, ng, lane);
          }
        }
      } else {
      // one unit dot in the loop body (a small hot loop stays in the
      // instruction cache); value j = rm * G + g lands in part[j]
      int j = 0;
#pragma unroll 1
      for (int rm = 0; rm < RM; ++rm) {
        const int r = NMAT == 2 ? (rm >> 1) : rm, m = NMAT == 2 ? (rm & 1) : 0;
        const uint8_t* wrow = tile + ((int64_t)m * R + r) * rs;
#pragma unroll 1
        for (int g = 0; g < G; ++g, ++j) {
          const int ng = group_units(p.K, g);
          if (vi * G + g != cached) {
            if (lane < ng) {
              const uint8_t* xg = xbase + (int64_t)vi * xstride + qact_group_offset(g);
              if (pl.xq_smem)
                xc.load(xg, ng, lane);
              else
                xc.load_any(xg, ng, lane);
            }
            cached = vi * G + g;
          }
          float d = 0.0f;
          if (lane < ng) d = unit_dot_x<WT>(wrow + group_offset(WT, p.K, g), xc, ng, lane);
#pragma unroll
          for (int q = 0; q < 8; ++q) part[q] = (q == j) ? d : part[q];
        }
      }
      }
      const float sum = reduce8(part, lane);
      // (row, matrix) rm = lane adds its group sums in order; value v sits in
      // lane ((v >> 2) & 1) << 2 | ((v >> 1) & 1) << 3 | (v & 1) << 4
      float tot = 0.0f;
      for (int g = 0; g < G; ++g) {
        const int v = lane * G + g;
        const int src = ((v >> 2) & 1) << 2 | ((v >> 1) & 1) << 3 | (v & 1) << 4;
        const float sg = __shfl_sync(0xffffffffu, sum, src);
        tot = __fadd_rn(tot, sg);
      }
      if (lane < RM) {
        const int r = NMAT == 2 ? (lane >> 1) : lane, m = NMAT == 2 ? (lane & 1) : 0;
        acc[((rbase - r0 + r) * p.n_pairs + pair) * NMAT + m] = tot;
      }
    }
    __syncwarp();
    const int nxt = it + S * NWS;  // this slot's next tile
    if (lane == 0 && nxt < n_tiles) issue(nxt, s, n_slots);
  }
  consumer_sync<NWS>();
  // the last CTA past the routing wait re-arms the counters for the next launch
  if (depart_old == (int)gridDim.x - 1) {
    atomicExch(&p.rsync[0], 0);
    atomicExch(&p.rsync[1], 0);
  }
  if (*(volatile int*)p.status == ERR_TIMEOUT || r0 >= r1) return;  // uniform across the consumers
  run_epilogue<NWS>(p, acc, r0, r1, red);
}

// ---------------------------------------------------------------------------
// GQA decode attention over the paged KV cache, ggml's op order exactly
// (engine.cpp:1751-1761):
//   kq_j  = (float) sum_i (double)(k_ji * q_i)          ggml_mul_mat F32
//   s_j   = kq_j * (1/sqrt(hd)); M = max_j s_j          ggml_soft_max_ext
//   p_j   = exp(s_j - M); S = sum_j (double) p_j; p'_j = p_j * (float)(1/S)
//   o_i   = (float) sum_j (double)(v_ji * p'_j)         ggml_mul_mat F32
// One thread-block cluster per (token, kv head); CTA r of the cluster owns a
// contiguous run of whole pages.  A KV page of one head ([16][hd], 4 KB in f16
// at hd 128) is contiguous in the pool, so each page arrives in shared memory
// by one bulk copy into a ring of page slots (one ring for K, one for V).
// Pages that earlier steps wrote are requested before the wait on the previous
// kernel; only the page holding the current position waits for it.  The
// cross-CTA steps (global max, global sum, the output reduction) are pushes
// into the other CTAs' shared memory, each closed by one mbarrier arrival per
// CTA pair, so the two-pass softmax is exact in one kernel without cluster-wide
// barriers.  The GQA group's query heads share every K/V page.
// ---------------------------------------------------------------------------
constexpr int ATT_NW = 8;
constexpr int ATT_THREADS = ATT_NW * 32;
constexpr int ATT_MAXG = 16;       // max query heads per kv head
constexpr int ATT_MAXC = 16;       // max CTAs per cluster
constexpr int ATT_RING = 64 * 1024;  // bytes of K + V page slots
constexpr int ATT_PG = 4;            // pages between block barriers (slots refilled per group)

struct AttnPlan {
  int ns, slot_bytes;
  int kring, vring, qs, sc, lsum, gstd, lmax, invs, gst, ored, total;
};

__host__ __device__ inline int al16(int v) { return (v + 15) & ~15; }

__host__ __device__ inline AttnPlan make_attn_plan(int hd, int gqa, int f16, int max_chunk) {
  AttnPlan a;
  a.slot_bytes = 16 * hd * (f16 ? 2 : 4);
  int ns = ATT_RING / (2 * a.slot_bytes);
  ns = ns < 2 ? 2 : (ns > 32 ? 32 : ns);
  a.ns = ns;
  a.kring = ((2 * ns + 3) * 8 + 127) & ~127;  // kfull[ns] | vfull[ns] | xbar[3]
  a.vring = a.kring + ns * a.slot_bytes;
  a.qs = a.vring + ns * a.slot_bytes;
  a.sc = a.qs + al16(gqa * hd * 4);
  a.lsum = a.sc + al16(gqa * max_chunk * 4);
  a.gstd = a.lsum + al16(gqa * 8);
  a.lmax = a.gstd + ATT_MAXC * gqa * 8;
  a.invs = a.lmax + al16(gqa * 4);
  a.gst = a.invs + al16(gqa * 4);
  a.ored = a.gst + al16(ATT_MAXC * gqa * 4);
  a.total = a.ored + (gqa * hd + ATT_MAXC) * 8;  // [C][ceil(gqa*hd/C)] partial outputs received
  return a;
}

template <int HD, int F16>
__global__ void __launch_bounds__(ATT_THREADS) attn_kernel(const AttnParams p) {
  namespace cg = cooperative_groups;
  extern __shared__ __align__(128) uint8_t asmem[];
  cg::cluster_group cl = cg::this_cluster();
  const int C = (int)cl.num_blocks();
  const int rank = (int)cl.block_rank();
  const int hk = blockIdx.x / C, t = blockIdx.y;
  const int Hkv = p.kv.n_head_kv;
  const int gqa = p.n_head / Hkv;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int mc = p.max_chunk;
  const AttnPlan pl = make_attn_plan(HD, gqa, F16, mc);
  uint64_t* kfull = reinterpret_cast<uint64_t*>(asmem);
  uint64_t* vfull = kfull + pl.ns;
  uint8_t* kring = asmem + pl.kring;
  uint8_t* vring = asmem + pl.vring;
  float* qs = reinterpret_cast<float*>(asmem + pl.qs);
  float* sc = reinterpret_cast<float*>(asmem + pl.sc);
  double* lsum = reinterpret_cast<double*>(asmem + pl.lsum);
  double* gstd = reinterpret_cast<double*>(asmem + pl.gstd);
  float* lmax = reinterpret_cast<float*>(asmem + pl.lmax);
  float* invs = reinterpret_cast<float*>(asmem + pl.invs);
  float* gst = reinterpret_cast<float*>(asmem + pl.gst);
  double* ored = reinterpret_cast<double*>(asmem + pl.ored);
  uint64_t* xbar = vfull + pl.ns;  // [3]: maxima, sums, partial outputs received from the cluster
  const int nout = gqa * HD, per = (nout + C - 1) / C;

  // Positions and the page table were written before the previous kernel
  // started (every kernel of the step lets its successor launch only after
  // its own wait on its predecessor), so they are read before the wait.
  // this sequence's page ids (up to 256), loaded alongside the position so
  // the page copies do not wait for two dependent round trips
  __shared__ int ptab_s[256];
  {
    const int* prow = p.kv.page_table + (int64_t)t * p.kv.max_pages;
    if (tid < min(p.kv.max_pages, 256)) ptab_s[tid] = prow[tid];
  }
  int n_kv = p.pos[t] + 1;
  if (n_kv < 1 || n_kv > p.kv.max_pages * 16) {  // outside the page table: no access, report
    if (tid == 0 && rank == 0) atomicExch(p.status, ERR_BAD_POS);
    n_kv = 0;
  }
  if ((((n_kv + 15) >> 4) + C - 1) / C * 16 > mc) {  // score buffer too small: no access, report
    if (tid == 0 && rank == 0) atomicExch(p.status, ERR_BAD_POS);
    n_kv = 0;
  }
  const int np_tot = (n_kv + 15) >> 4;
  const int ppc = (np_tot + C - 1) / C;
  const int pb = min(np_tot, rank * ppc);
  const int np = min(np_tot, pb + ppc) - pb;
  const int nloc = max(0, min(n_kv, (pb + np) * 16) - pb * 16);
  const int last_page = (n_kv - 1) >> 4;  // the page this step's K/V row lands in
  const int* ptab = p.kv.page_table + (int64_t)t * p.kv.max_pages;
  const int64_t page_stride = (int64_t)Hkv * pl.slot_bytes;
  const int64_t head_off = (int64_t)hk * pl.slot_bytes;

  // thread 0: bring page i (local index) of K or V into its ring slot
  auto issue = [&](int isv, int i) {
    const int slot = i % pl.ns;
    uint64_t* bar = (isv ? vfull : kfull) + slot;
    const int pg = pb + i < 256 ? ptab_s[pb + i] : ptab[pb + i];
    if (pg < 0 || (p.kv.n_pages > 0 && pg >= p.kv.n_pages)) {  // never copy from outside the pool
      atomicExch(p.status, ERR_BAD_PAGE);
      mbar_arrive(bar);
      return;
    }
    mbar_arrive_expect_tx(bar, (uint32_t)pl.slot_bytes);
    const uint8_t* src = kv_page(p.kv, isv, pg, page_stride) + head_off;
    bulk_g2s((isv ? vring : kring) + (int64_t)slot * pl.slot_bytes, src, (uint32_t)pl.slot_bytes, bar);
  };

  if (tid == 0) {
    for (int i = 0; i < pl.ns; ++i) {
      mbar_init(&kfull[i], 1);
      mbar_init(&vfull[i], 1);
    }
    // exchange barriers: one local arrival that expects every byte the
    // cluster will push (maxima, sums, this CTA's slice of the outputs)
    for (int i = 0; i < 3; ++i) mbar_init(&xbar[i], 1);
    mbar_arrive_expect_tx(&xbar[0], (uint32_t)(gqa * C * 4));
    mbar_arrive_expect_tx(&xbar[1], (uint32_t)(gqa * C * 8));
    mbar_arrive_expect_tx(&xbar[2], (uint32_t)(max(0, min(nout, rank * per + per) - rank * per) * C * 8));
    fence_mbar_init();
  }
  __syncthreads();
  cluster_arrive();  // barriers initialised; waited on before the first remote push
  // page copies are issued by every warp's lane 0 (one thread keeps only
  // about one bulk copy per quarter microsecond going)
  const int npre = min(np, pl.ns);
  if (lane == 0) {
    for (int i = warp; i < npre; i += ATT_NW)
      if (pb + i < last_page) issue(0, i);
    for (int i = warp; i < npre; i += ATT_NW)
      if (pb + i < last_page) issue(1, i);
  }
  pdl_wait();
  pdl_launch_dependents();
  if (lane == 0) {
    for (int i = warp; i < npre; i += ATT_NW)
      if (pb + i >= last_page) issue(0, i);
    for (int i = warp; i < npre; i += ATT_NW)
      if (pb + i >= last_page) issue(1, i);
  }
  const float scale = __fdiv_rn(1.0f, sqrtf((float)HD));
  for (int i = tid; i < gqa * HD; i += ATT_THREADS) qs[i] = p.q[((int64_t)t * p.n_head + hk * gqa) * HD + i];
  __syncthreads();

  // ---- K pages: scores.  LP lanes per position, 8 dims per lane
  {
    constexpr int LP = HD / 8;
    constexpr int PPW = 32 / LP;
    const int sub = lane / LP, dl = (lane % LP) * 8;
    const int pg = max(1, min(ATT_PG, pl.ns / 2));  // half the ring: the next group's copies are in flight
    for (int i0 = 0; i0 < np; i0 += pg) {
      const int ig = min(pg, np - i0);
      for (int i = i0; i < i0 + ig; ++i) {
        const int slot = i % pl.ns;
        mbar_wait_bounded(&kfull[slot], (uint32_t)((i / pl.ns) & 1), p.status);
        const uint8_t* kp = kring + (int64_t)slot * pl.slot_bytes;
        for (int base = warp * PPW; base < 16; base += ATT_NW * PPW) {
          const int jj = base + sub;
          const int jl = i * 16 + jj;
          float kf[8];
          if constexpr (F16) {
            const uint4 raw = lds128(kp + (jj * HD + dl) * 2);
            const __half2* hv = reinterpret_cast<const __half2*>(&raw);
  #pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = __half22float2(hv[e]);
              kf[2 * e] = f.x;
              kf[2 * e + 1] = f.y;
            }
          } else {
            const uint4 r0 = lds128(kp + (jj * HD + dl) * 4);
            const uint4 r1 = lds128(kp + (jj * HD + dl) * 4 + 16);
            kf[0] = __uint_as_float(r0.x); kf[1] = __uint_as_float(r0.y);
            kf[2] = __uint_as_float(r0.z); kf[3] = __uint_as_float(r0.w);
            kf[4] = __uint_as_float(r1.x); kf[5] = __uint_as_float(r1.y);
            kf[6] = __uint_as_float(r1.z); kf[7] = __uint_as_float(r1.w);
          }
          // four heads at a time, two accumulation chains each (the double
          // sums are order-free at this length), so the chains overlap
          for (int h0 = 0; h0 < gqa; h0 += 4) {
            double r[4];
  #pragma unroll
            for (int hh = 0; hh < 4; ++hh) {
              r[hh] = 0.0;
              if (h0 + hh < gqa) {
                const float4 qa = *reinterpret_cast<const float4*>(qs + (h0 + hh) * HD + dl);
                const float4 qb = *reinterpret_cast<const float4*>(qs + (h0 + hh) * HD + dl + 4);
                double a0 = (double)__fmul_rn(kf[0], qa.x), a1 = (double)__fmul_rn(kf[1], qa.y);
                a0 += (double)__fmul_rn(kf[2], qa.z);
                a1 += (double)__fmul_rn(kf[3], qa.w);
                a0 += (double)__fmul_rn(kf[4], qb.x);
                a1 += (double)__fmul_rn(kf[5], qb.y);
                a0 += (double)__fmul_rn(kf[6], qb.z);
                a1 += (double)__fmul_rn(kf[7], qb.w);
                r[hh] = a0 + a1;
              }
            }
  #pragma unroll
            for (int o = LP / 2; o > 0; o >>= 1)
  #pragma unroll
              for (int hh = 0; hh < 4; ++hh) r[hh] += __shfl_xor_sync(0xffffffffu, r[hh], o);
            if ((lane % LP) == 0 && jl < nloc) {
  #pragma unroll
              for (int hh = 0; hh < 4; ++hh)
                if (h0 + hh < gqa) sc[(h0 + hh) * mc + jl] = __fmul_rn((float)r[hh], scale);
            }
          }
        }
      }
      if (i0 + pl.ns < np) {  // the group's slots are refilled: every warp must be done with them
        __syncthreads();
        if (lane == 0)
          for (int i = i0 + warp; i < i0 + ig; i += ATT_NW)
            if (i + pl.ns < np) issue(0, i + pl.ns);
      }
    }
  }
  __syncthreads();  // all scores are in
  // Exchanges between the cluster's CTAs are pushes: every CTA stores its
  // values into each CTA's receive slots with asynchronous DSMEM stores that
  // count their bytes on the receiver's exchange barrier; a CTA waits on its
  // own barrier until every byte it expects has landed.  One hop, no fence,
  // no cluster-wide barrier.
  auto push_done = [&](int x) { mbar_wait_cluster_bounded(&xbar[x], 0, p.status); };
  // local max per head
  for (int h = warp; h < gqa; h += ATT_NW) {
    float m = -INFINITY;
    for (int jl = lane; jl < nloc; jl += 32) m = fmaxf(m, sc[h * mc + jl]);
    m = warp_max(m);
    if (lane == 0) lmax[h] = m;
  }
  __syncthreads();
  cluster_wait();  // every CTA of the cluster has initialised its barriers
  if (tid < gqa * C) {
    const int h = tid / C, r = tid % C;
    dsmem_st_async_f32(dsmem_addr(&gst[h * C + rank], r), lmax[h], dsmem_addr(&xbar[0], r));
  }
  push_done(0);
  // ---- global max, exp, local sum: warp h owns head h
  for (int h = warp; h < gqa; h += ATT_NW) {
    float M = lane < C ? gst[h * C + lane] : -INFINITY;
    M = warp_max(M);
    double s = 0.0;
    for (int jl = lane; jl < nloc; jl += 32) {
      const float e = sfk_expf(__fsub_rn(sc[h * mc + jl], M));
      sc[h * mc + jl] = e;
      s += (double)e;
    }
    s = warp_sum_d(s);
    if (lane == 0) lsum[h] = s;
  }
  __syncthreads();
  if (tid < gqa * C) {
    const int h = tid / C, r = tid % C;
    dsmem_st_async_f64(dsmem_addr(&gstd[h * C + rank], r), lsum[h], dsmem_addr(&xbar[1], r));
  }
  push_done(1);
  if (tid < gqa) {
    double S = 0.0;
    for (int r = 0; r < C; ++r) S += gstd[tid * C + r];
    invs[tid] = (float)(1.0 / S);
  }
  __syncthreads();

  // ---- V pages: o_i = sum_j (double)(v_ji * p'_j); each thread owns pairs of
  // output dims (at most ATT_MAXG * HD / 2 / ATT_THREADS of them)
  constexpr int NPAIR = (ATT_MAXG * HD / 2 + ATT_THREADS - 1) / ATT_THREADS;
  const int npairs = gqa * HD / 2;
  double acc[2 * NPAIR][2];  // two chains per output dim (order-free double sums)
#pragma unroll
  for (int i = 0; i < 2 * NPAIR; ++i) acc[i][0] = acc[i][1] = 0.0;
  const int pgv = max(1, min(ATT_PG, pl.ns / 2));
  for (int i0 = 0; i0 < np; i0 += pgv) {
    const int ig = min(pgv, np - i0);
    for (int i = i0; i < i0 + ig; ++i) {
      const int slot = i % pl.ns;
      mbar_wait_bounded(&vfull[slot], (uint32_t)((i / pl.ns) & 1), p.status);
      const uint8_t* vp = vring + (int64_t)slot * pl.slot_bytes;
      const int jn = min(16, nloc - i * 16);
  #pragma unroll
      for (int q2 = 0; q2 < NPAIR; ++q2) {
        const int pi = tid + q2 * ATT_THREADS;
        if (pi < npairs) {
          const int h = (pi * 2) / HD, dd = (pi * 2) % HD;
          const float inv = invs[h];
          const float* sh = sc + h * mc + i * 16;
          auto step = [&](int jj, int c) {
            const float pj = __fmul_rn(sh[jj], inv);
            float2 v;
            if constexpr (F16)
              v = __half22float2(*reinterpret_cast<const __half2*>(vp + (jj * HD + dd) * 2));
            else
              v = *reinterpret_cast<const float2*>(vp + (jj * HD + dd) * 4);
            acc[2 * q2][c] += (double)__fmul_rn(v.x, pj);
            acc[2 * q2 + 1][c] += (double)__fmul_rn(v.y, pj);
          };
          if (jn == 16) {
  #pragma unroll
            for (int jj = 0; jj < 16; ++jj) step(jj, jj & 1);
          } else {
            for (int jj = 0; jj < jn; ++jj) step(jj, jj & 1);
          }
        }
      }
    }
    if (i0 + pl.ns < np) {  // the group's slots are refilled: every thread must be done with them
      __syncthreads();
      if (lane == 0)
        for (int i = i0 + warp; i < i0 + ig; i += ATT_NW)
          if (i + pl.ns < np) issue(1, i + pl.ns);
    }
  }
  // ---- partial outputs: output o belongs to CTA o / per, which adds the C
  // partials in rank order
#pragma unroll
  for (int q2 = 0; q2 < NPAIR; ++q2) {
    const int pi = tid + q2 * ATT_THREADS;
    if (pi < npairs) {
#pragma unroll
      for (int d2 = 0; d2 < 2; ++d2) {
        const int o = 2 * pi + d2, r = o / per;
        dsmem_st_async_f64(dsmem_addr(&ored[rank * per + (o - r * per)], r), acc[2 * q2 + d2][0] + acc[2 * q2 + d2][1],
                           dsmem_addr(&xbar[2], r));
      }
    }
  }
  push_done(2);
  {
    const int o0 = rank * per, o1 = min(nout, o0 + per);
    for (int o = o0 + tid; o < o1; o += ATT_THREADS) {
      double sum = 0.0;
      for (int r = 0; r < C; ++r) sum += ored[r * per + (o - o0)];
      p.out[((int64_t)t * p.n_head + hk * gqa) * HD + o] = (float)sum;
    }
  }
}

size_t attn_smem_bytes(int hd, int gqa, int f16, int max_chunk) {
  return (size_t)make_attn_plan(hd, gqa, f16, max_chunk).total;
}

// ---------------------------------------------------------------------------
// router kernel (used when the routing is not folded into the gate/up kernel):
// one CTA per token runs route_one; the last CTA builds the slot lists.
// ---------------------------------------------------------------------------
constexpr int RT_THREADS = 1024;
constexpr int RT_MAXE = 512;

struct BlockSync {
  __device__ void operator()() const { __syncthreads(); }
};

__global__ void __launch_bounds__(RT_THREADS) router_kernel(const RouterParams p) {
  const int t = blockIdx.x, tid = threadIdx.x;
  {
    // the router weights do not depend on the previous kernel: pull them
    // toward L2 while it drains
    const char* wb = reinterpret_cast<const char*>(p.w_r);
    const int64_t nbytes = (int64_t)p.E * p.d * 4;
    for (int64_t o = (int64_t)(t * RT_THREADS + tid) * 128; o < nbytes; o += (int64_t)gridDim.x * RT_THREADS * 128)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(wb + o));
  }
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ __align__(16) uint8_t rsm[];
  float* xn = reinterpret_cast<float*>(rsm);  // [d]
  __shared__ double red[RT_THREADS / 32 + 1];
  __shared__ float probs[RT_MAXE];
  __shared__ double seg[RT_MAXE * 4];
  __shared__ int last_flag;
  route_one<RT_THREADS / 32>(p.x + (int64_t)t * p.d, p.norm_w, p.w_r, p.d, p.E, p.k, p.eps, p.act_type,
                             p.xq + (int64_t)t * qact_bytes(p.d), xn, seg, probs, red, &p.route->ids[t * p.k],
                             &p.route->w[t * p.k], p.xn ? p.xn + (int64_t)t * p.d : nullptr, BlockSync{});
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int old = atomicAdd(p.counter, 1);
    last_flag = (old == p.b - 1);
  }
  __syncthreads();
  if (!last_flag || tid != 0) return;
  __threadfence();
  Route* r = p.route;
  const int np = p.b * p.k;
  int ids_l[MAXP];
  for (int i = 0; i < np; ++i) ids_l[i] = __ldcg(&r->ids[i]);
  build_slots(ids_l, np, r, p.ep_e0, p.ep_eloc);
  r->k = p.k;
  r->b = p.b;
  atomicExch(p.counter, 0);
}

// ---------------------------------------------------------------------------
// embedding: token id -> dequantized row (ggml_get_rows, engine.cpp:2708-2723)
// one CTA; greedy mode takes the previous step's argmax and clears it.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) embed_kernel(const EmbedParams p) {
  pdl_wait();
  pdl_launch_dependents();
  // every CTA resolves the tokens (read-only); CTA 0 records them.  The
  // argmax keys are cleared later in the step (layer 0's QKV kernel), after
  // every CTA here has read them.
  __shared__ int toks[MAXB];
  const int tid = threadIdx.x;
  if (tid < p.b) {
    int tok;
    if (p.greedy) {
      const unsigned long long key = p.argmax_key[tid];
      tok = (int)(0xFFFFFFFFu - (unsigned)(key & 0xFFFFFFFFull));
    } else {
      tok = p.tok_in[tid];
    }
    if (tok < 0 || tok >= p.V) {
      if (blockIdx.x == 0) atomicExch(p.status, ERR_BAD_ID);
      tok = 0;
    }
    toks[tid] = tok;
    if (blockIdx.x == 0) {
      const int pos = p.pos_in ? p.pos_in[tid] : p.pos_state[tid];
      p.pos_cur[tid] = pos;
      if (p.pos_state) p.pos_state[tid] = pos + 1;
      p.tok_hist[tid] = tok;
    }
  }
  if (blockIdx.x == 0 && tid == 0 && p.ep_step) *p.ep_step += 1;  // expert-parallel combine epochs
  __syncthreads();
  const int64_t rb = (int64_t)dev_gguf_row_bytes(p.type, p.d);
  const int i = blockIdx.x * 256 + tid;
  if (i < p.d) {
    for (int t = 0; t < p.b; ++t) p.x[(int64_t)t * p.d + i] = gguf_dequant_one(p.type, p.tok_embd + (int64_t)toks[t] * rb, i);
  }
}

// ---------------------------------------------------------------------------
// Expert-parallel combine (see EpParams): signal this rank's partial to every
// rank, wait for every rank's, add them in rank order.  The waits are bounded
// and report ERR_TIMEOUT; nothing traps.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(256) ep_combine_kernel(const EpParams p) {
  // the step counter was written by the embed kernel, two or more kernels back
  const unsigned epoch = ep_epoch(*p.ep_step, p.n_layer, p.layer, p.stage);
  pdl_wait();
  pdl_launch_dependents();
  if (blockIdx.x == 0 && (int)threadIdx.x < p.n_ranks) {
    __threadfence_system();  // this rank's partial (the down kernel's output) before the flag
    st_release_sys(p.peer_flags[threadIdx.x] + p.rank, epoch);
  }
  if (threadIdx.x == 0) {
    const long long t0 = clock64();
    bool ok = true;
    for (int r = 0; r < p.n_ranks && ok; ++r) {
      while (!ep_reached(ld_acquire_sys(p.flags + r), epoch)) {
        __nanosleep(32);
        if (clock64() - t0 > (1ll << 31)) {
          atomicExch(p.status, ERR_TIMEOUT);
          ok = false;
          break;
        }
      }
    }
  }
  __syncthreads();
  const int off = ((p.layer & 1) * 2 + p.stage) * p.half;
  for (int i = blockIdx.x * 256 + threadIdx.x; i < p.n; i += gridDim.x * 256) {
    float a = __ldcv(p.parts[0] + off + i);
    for (int r = 1; r < p.n_ranks; ++r) a = __fadd_rn(a, __ldcv(p.parts[r] + off + i));
    p.x[i] = a;
  }
}

__global__ void __launch_bounds__(32) ep_argmax_kernel(const EpHeadParams p) {
  pdl_wait();
  pdl_launch_dependents();
  const unsigned epoch = *p.ep_step;  // written by this step's embed kernel: one exchange per step
  const int tid = threadIdx.x;
  if (tid < p.b) {
    p.own_keys[tid] = p.key[tid];
    __threadfence_system();  // the published keys before the flag
  }
  __syncthreads();
  if (tid < p.n_ranks) {
    __threadfence_system();
    st_release_sys(p.peer_flags[tid] + p.rank, epoch);
  }
  __shared__ int ok;
  if (tid == 0) {
    ok = 1;
    const long long t0 = clock64();
    for (int r = 0; r < p.n_ranks && ok; ++r) {
      while (!ep_reached(ld_acquire_sys(p.flags + r), epoch)) {
        __nanosleep(32);
        if (clock64() - t0 > (1ll << 31)) {
          atomicExch(p.status, ERR_TIMEOUT);
          ok = 0;
          break;
        }
      }
    }
  }
  __syncthreads();
  if (ok && tid < p.b) {
    unsigned long long m = 0;
    for (int r = 0; r < p.n_ranks; ++r) {
      const unsigned long long k = __ldcv(p.peer_keys[r] + tid);
      m = k > m ? k : m;
    }
    p.key[tid] = m;
  }
}

// ---------------------------------------------------------------------------
// Route from caller-supplied ids / weights (operator-level mul_mat_id / moe_ffn)
// ---------------------------------------------------------------------------
__global__ void route_build_kernel(const int* ids, const float* w, int b, int k, int n_expert, Route* r, int* status) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const int np = b * k;
  int ns = 0, fill = 0, prev = -1;
  for (int i = 0; i < np; ++i) {
    const int e = ids[i];
    if (e < 0 || e >= n_expert) {
      atomicExch(status, ERR_BAD_ID);
      r->n_slots = 0;
      r->slot_off[0] = 0;
      return;
    }
    r->ids[i] = e;
    r->w[i] = w ? w[i] : 1.0f;
  }
  r->slot_off[0] = 0;
  while (true) {
    int nxt = 0x7fffffff;
    for (int i = 0; i < np; ++i)
      if (ids[i] > prev && ids[i] < nxt) nxt = ids[i];
    if (nxt == 0x7fffffff) break;
    r->slot_expert[ns] = nxt;
    for (int i = 0; i < np; ++i)
      if (ids[i] == nxt) r->slot_pairs[fill++] = i;
    r->slot_off[++ns] = fill;
    prev = nxt;
  }
  r->n_slots = ns;
  r->k = k;
  r->b = b;
}

cudaError_t launch_route_build(const int* ids, const float* w, int b, int k, int n_expert, Route* r, int* status,
                               cudaStream_t st) {
  if (b * k > MAXP) return cudaErrorInvalidValue;
  route_build_kernel<<<1, 32, 0, st>>>(ids, w, b, k, n_expert, r, status);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------
template <typename Kern, typename Arg>
static cudaError_t launch_pdl(Kern k, dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl, const Arg& a) {
  // every kernel of the step asks for the same L1/shared split (all shared),
  // so consecutive kernels never wait for an SM to reconfigure its carveout
  cudaError_t ce = cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  if (ce != cudaSuccess) return ce;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, a);
}

template <int WT>
static cudaError_t launch_stream_t(const StreamParams& p, int grid, cudaStream_t st, bool pdl) {
  const Plan2 pl2 = choose_plan2(p);
  if (pl2.nws) {
    StreamParams q = p;
    q.pl = pl2;
    const int smem2 = pl2.total;
    const dim3 block(pl2.nws * 32);
    cudaError_t e;
#define SFK_LAUNCH2(NM, NWV, MB)                                                                              \
  do {                                                                                                         \
    e = cudaFuncSetAttribute(stream2_kernel<WT, NM, NWV, MB>, cudaFuncAttributeMaxDynamicSharedMemorySize,     \
                             smem2);                                                                           \
    if (e != cudaSuccess) return e;                                                                            \
    return launch_pdl(stream2_kernel<WT, NM, NWV, MB>, dim3(grid), block, smem2, st, pdl, q);                  \
  } while (0)
    if (p.nmat == 1) {
      if (pl2.occ == 2) SFK_LAUNCH2(1, 8, 2);
      if (pl2.nws == 16) SFK_LAUNCH2(1, 16, 1);
      SFK_LAUNCH2(1, 8, 1);
    }
    if (pl2.occ == 2) SFK_LAUNCH2(2, 8, 2);
    if (pl2.nws == 16) SFK_LAUNCH2(2, 16, 1);
    SFK_LAUNCH2(2, 8, 1);
#undef SFK_LAUNCH2
  }
  if (p.pro == PRO_ROUTE) return cudaErrorInvalidValue;  // only the warp-tile kernel routes in its prologue
  const StreamPlan pl = make_plan(p);
  cudaError_t e = cudaFuncSetAttribute(stream_kernel<WT>, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.total);
  if (e != cudaSuccess) return e;
  return launch_pdl(stream_kernel<WT>, dim3(grid), dim3((NW + 1) * 32), pl.total, st, pdl, p);
}

cudaError_t launch_stream(const StreamParams& p, int grid, cudaStream_t st, bool pdl) {
  switch (p.wtype) {
    case T_Q4_K: return launch_stream_t<T_Q4_K>(p, grid, st, pdl);
    case T_Q6_K: return launch_stream_t<T_Q6_K>(p, grid, st, pdl);
    case T_Q8_0: return launch_stream_t<T_Q8_0>(p, grid, st, pdl);
    default: return cudaErrorInvalidValue;
  }
}

template <int HD, int F16>
static cudaError_t launch_attn_t(const AttnParams& p, cudaStream_t st, bool pdl) {
  const size_t smem = attn_smem_bytes(HD, p.n_head / p.kv.n_head_kv, F16, p.max_chunk);
  cudaError_t e = cudaFuncSetAttribute(attn_kernel<HD, F16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  if (p.cluster > 8) {
    e = cudaFuncSetAttribute(attn_kernel<HD, F16>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
  }
  e = cudaFuncSetAttribute(attn_kernel<HD, F16>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.cluster * p.kv.n_head_kv, p.b, 1);
  cfg.blockDim = dim3(ATT_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, attn_kernel<HD, F16>, p);
}

template <int HD, int F16>
static int attn_active_clusters_t(int gqa, int cluster, int max_chunk) {
  const size_t smem = attn_smem_bytes(HD, gqa, F16, max_chunk);
  if (cudaFuncSetAttribute(attn_kernel<HD, F16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return 0;
  if (cluster > 8 &&
      cudaFuncSetAttribute(attn_kernel<HD, F16>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
    return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cluster, 1, 1);
  cfg.blockDim = dim3(ATT_THREADS);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, attn_kernel<HD, F16>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

int attn_active_clusters(int head_dim, int f16, int gqa, int cluster, int max_chunk) {
  switch (head_dim) {
    case 32: return f16 ? attn_active_clusters_t<32, 1>(gqa, cluster, max_chunk) : attn_active_clusters_t<32, 0>(gqa, cluster, max_chunk);
    case 64: return f16 ? attn_active_clusters_t<64, 1>(gqa, cluster, max_chunk) : attn_active_clusters_t<64, 0>(gqa, cluster, max_chunk);
    case 128: return f16 ? attn_active_clusters_t<128, 1>(gqa, cluster, max_chunk) : attn_active_clusters_t<128, 0>(gqa, cluster, max_chunk);
    case 256: return f16 ? attn_active_clusters_t<256, 1>(gqa, cluster, max_chunk) : attn_active_clusters_t<256, 0>(gqa, cluster, max_chunk);
    default: return 0;
  }
}

cudaError_t launch_ep_argmax(const EpHeadParams& p, cudaStream_t st, bool pdl) {
  if (p.b < 1 || p.b > 32 || p.n_ranks < 1 || p.n_ranks > MAXR) return cudaErrorInvalidValue;
  return launch_pdl(ep_argmax_kernel, dim3(1), dim3(32), 0, st, pdl, p);
}

cudaError_t launch_ep_combine(const EpParams& p, cudaStream_t st, bool pdl) {
  if (p.n_ranks < 1 || p.n_ranks > MAXR || p.n < 1) return cudaErrorInvalidValue;
  const int grid = std::min(64, (p.n + 255) / 256);
  return launch_pdl(ep_combine_kernel, dim3(grid), dim3(256), 0, st, pdl, p);
}

cudaError_t launch_attn(const AttnParams& p, cudaStream_t st, bool pdl) {
  if (p.n_head % p.kv.n_head_kv || p.n_head / p.kv.n_head_kv > ATT_MAXG || p.cluster < 1 || p.cluster > ATT_MAXC)
    return cudaErrorInvalidValue;
  const bool h = p.kv.f16 != 0;
  switch (p.kv.head_dim) {
    case 32: return h ? launch_attn_t<32, 1>(p, st, pdl) : launch_attn_t<32, 0>(p, st, pdl);
    case 64: return h ? launch_attn_t<64, 1>(p, st, pdl) : launch_attn_t<64, 0>(p, st, pdl);
    case 128: return h ? launch_attn_t<128, 1>(p, st, pdl) : launch_attn_t<128, 0>(p, st, pdl);
    case 256: return h ? launch_attn_t<256, 1>(p, st, pdl) : launch_attn_t<256, 0>(p, st, pdl);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_router(const RouterParams& p, cudaStream_t st, bool pdl) {
  if (p.E > RT_MAXE || p.k > 16 || p.b * p.k > MAXP) return cudaErrorInvalidValue;
  const size_t smem = (size_t)p.d * sizeof(float);
  cudaError_t e = cudaFuncSetAttribute(router_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return launch_pdl(router_kernel, dim3(p.b), dim3(RT_THREADS), smem, st, pdl, p);
}

cudaError_t launch_embed(const EmbedParams& p, cudaStream_t st, bool pdl) {
  if (p.b > MAXB) return cudaErrorInvalidValue;
  return launch_pdl(embed_kernel, dim3((p.d + 255) / 256), dim3(256), 0, st, pdl, p);
}

}  // namespace sfk
