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
#include <cstdint>
#include <cstdio>

#include "sfk_act.cuh"
#include "sfk_device.cuh"
#include "sfk_kernels.cuh"
#include "sfk_dequant.cuh"

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

int stream_smem_bytes(const StreamParams& p, int* n_stages, int* stage_bytes, int* rows_per_warp) {
  const StreamPlan s = make_plan(p);
  if (n_stages) *n_stages = s.n_stages;
  if (stage_bytes) *stage_bytes = s.stage_bytes;
  if (rows_per_warp) *rows_per_warp = s.rows_per_warp;
  return s.total;
}

// consumer-only named barrier (the producer warp never joins it)
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"r"(NW * 32) : "memory"); }

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
__device__ void prologue_quant(const StreamParams& p, uint8_t* xq, int xq_vec_bytes, double* red) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = p.K;
  for (int t = 0; t < p.n_vec; ++t) {
    const float* x = p.x + (int64_t)t * K;
    float scale = 1.0f;
    if (p.norm_w) {
      double s = 0.0;
      for (int c = tid; c < K; c += NW * 32) {
        const float v = x[c];
        s += (double)__fmul_rn(v, v);
      }
      s = warp_sum_d(s);
      if (lane == 0) red[warp] = s;
      consumer_sync();
      if (tid == 0) {
        double tot = 0.0;
        for (int w = 0; w < NW; ++w) tot += red[w];
        red[NW] = tot;
      }
      consumer_sync();
      const float mean = (float)(red[NW] / (double)K);
      scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
      consumer_sync();
    }
    uint8_t* qa = xq + (int64_t)t * xq_vec_bytes;
    for (int blk = warp; blk < K / QK_K; blk += NW) {
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
    for (int64_t o = tid * 16; o < nbytes; o += NW * 32 * 16)
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

__device__ void epi_qkv(const StreamParams& p, const float* acc, int r0, int r1) {
  const int hd = p.kv.head_dim, Hkv = p.kv.n_head_kv;
  const int nq = p.n_head * hd, nk = Hkv * hd;
  const int npair_rows = (r1 - r0) / 2;
  for (int idx = threadIdx.x; idx < npair_rows * p.b; idx += NW * 32) {
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

__device__ void epi_gateup(const StreamParams& p, const float* acc, int r0, int r1, int* flags) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nr = r1 - r0;
  // h = silu(gate) * up  (ggml_swiglu_split(gate, up), engine.cpp:1969)
  for (int idx = tid; idx < nr * p.n_pairs; idx += NW * 32) {
    const int row = idx % nr, pr = idx / nr;
    const float g = acc[(row * p.n_pairs + pr) * 2 + 0];
    const float u = acc[(row * p.n_pairs + pr) * 2 + 1];
    const float sl = __fdiv_rn(g, __fadd_rn(1.0f, sfk_expf(-g)));
    p.h[(int64_t)pr * p.rows + r0 + row] = __fmul_rn(sl, u);
  }
  __threadfence();
  consumer_sync();
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
  consumer_sync();
  for (int q = q0; q <= q1; ++q) {
    if (!flags[q - q0]) continue;
    __threadfence();
    for (int pr = warp; pr < p.n_pairs; pr += NW) {
      const float* hp = p.h + (int64_t)pr * p.rows + q * QK_K + lane * 8;
      const float4 a = __ldcg(reinterpret_cast<const float4*>(hp));
      const float4 b = __ldcg(reinterpret_cast<const float4*>(hp + 4));
      const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
      qact_put(p.h_act_type, p.hq + (int64_t)pr * qact_bytes(p.rows), p.rows, q, v, lane);
    }
    if (tid == 0) atomicExch(&p.grp_counter[q], 0);
  }
}

__device__ void epi_down(const StreamParams& p, const float* acc, int r0, int r1) {
  const int nr = r1 - r0;
  const int k = p.k;
  for (int idx = threadIdx.x; idx < nr * p.b; idx += NW * 32) {
    const int row = idx % nr, t = idx / nr;
    // experts * weights, then moe_out = e0 + e1 + ..., then + ffn_inp
    // (engine.cpp:1973-1986)
    float a = __fmul_rn(acc[row * p.n_pairs + t * k], p.route->w[t * k]);
    for (int j = 1; j < k; ++j) a = __fadd_rn(a, __fmul_rn(acc[row * p.n_pairs + t * k + j], p.route->w[t * k + j]));
    if (p.res) a = __fadd_rn(a, p.res[(int64_t)t * p.rows + r0 + row]);
    p.y[(int64_t)t * p.y_stride + r0 + row] = a;
  }
}

__device__ void epi_lmhead(const StreamParams& p, const float* acc, int r0, int r1, unsigned long long* red) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nr = r1 - r0;
  for (int t = 0; t < p.b; ++t) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int row = tid; row < nr; row += NW * 32) {
      const float v = acc[row * p.n_pairs + t];
      if (p.store_logits) p.y[(int64_t)t * p.y_stride + r0 + row] = v;
      if (v > best) { best = v; bi = r0 + row; }
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
    consumer_sync();
    if (tid == 0) {
      unsigned long long m = 0;
      for (int w = 0; w < NW; ++w) m = red[w] > m ? red[w] : m;
      if (m) atomicMax(&p.argmax_key[t], m);
    }
    consumer_sync();
  }
}

// ---------------------------------------------------------------------------
// the streaming kernel
// ---------------------------------------------------------------------------
template <int WT>
__global__ void __launch_bounds__((NW + 1) * 32, 1) stream_kernel(const StreamParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  pdl_launch_dependents();
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
    if (p.route) {
      pdl_wait();  // routed experts are known only after the router ran
      tw.n_slots = p.route->n_slots;
    }
    uint32_t it = 0;
    for (tw.begin(); !tw.done(); tw.next(), ++it) {
      const int s = it % pl.n_stages;
      if (it >= (uint32_t)pl.n_stages) {
        if (!mbar_wait_bounded(&empty[s], ((it / pl.n_stages) - 1) & 1, p.status)) break;
      }
      const int ng = group_units(p.K, tw.g);
      const int gb = group_bytes(WT, ng);
      const int rbase = r0 + tw.rb * pl.rows_tile;
      const int nrows = min(pl.rows_tile, r1 - rbase);
      mbar_arrive_expect_tx(&full[s], (uint32_t)(nrows * p.nmat * gb));
      const int64_t eoff = (int64_t)slot_expert(p, tw.si) * p.expert_stride + group_offset(WT, p.K, tw.g);
      uint8_t* dst = ring + (int64_t)s * pl.stage_bytes;
      for (int m = 0; m < p.nmat; ++m) {
        const uint8_t* base = (m == 0 ? p.w0 : p.w1) + eoff;
        for (int r = 0; r < nrows; ++r)
          bulk_g2s(dst + (m * pl.rows_tile + r) * gb, base + (int64_t)(rbase + r) * p.rowstride, gb, &full[s]);
      }
    }
    if (!p.route) pdl_wait();
    return;
  }

  // ------------------------------ consumers ------------------------------
  pdl_wait();
  const int nacc = (r1 > r0 ? (r1 - r0) : 0) * p.n_pairs * p.nmat;
  for (int i = threadIdx.x; i < nacc; i += NW * 32) acc[i] = 0.0f;
  if (p.route) tw.n_slots = p.route->n_slots;
  if (p.xq_resident) {
    if (p.pro == PRO_QUANT)
      prologue_quant(p, xq, pl.xq_vec_bytes, red);
    else
      prologue_load(p, xq, pl.xq_vec_bytes, -1);
  }
  consumer_sync();

  uint32_t it = 0;
  int cur_g = -1;
  bool ok = true;
  for (tw.begin(); !tw.done(); tw.next(), ++it) {
    if (!p.xq_resident && tw.g != cur_g) {
      consumer_sync();
      prologue_load(p, xq, pl.xq_vec_bytes, tw.g);
      consumer_sync();
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
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  (void)ng_full;
  consumer_sync();
  if (!ok || r0 >= r1) return;

  switch (p.epi) {
    case EPI_STORE: {
      const int nr = r1 - r0;
      for (int idx = threadIdx.x; idx < nr * p.n_pairs; idx += NW * 32) {
        const int row = idx % nr, pr = idx / nr;
        p.y[(int64_t)pr * p.y_stride + r0 + row] = acc[row * p.n_pairs + pr];
      }
      break;
    }
    case EPI_RESID: {
      const int nr = r1 - r0;
      for (int idx = threadIdx.x; idx < nr * p.b; idx += NW * 32) {
        const int row = idx % nr, t = idx / nr;
        const float v = acc[row * p.n_pairs + t];
        p.y[(int64_t)t * p.y_stride + r0 + row] = p.res ? __fadd_rn(v, p.res[(int64_t)t * p.y_stride + r0 + row]) : v;
      }
      break;
    }
    case EPI_QKV: epi_qkv(p, acc, r0, r1); break;
    case EPI_GATEUP: epi_gateup(p, acc, r0, r1, reinterpret_cast<int*>(red)); break;
    case EPI_DOWN: epi_down(p, acc, r0, r1); break;
    case EPI_LMHEAD: epi_lmhead(p, acc, r0, r1, reinterpret_cast<unsigned long long*>(red)); break;
    default: break;
  }
}

// ---------------------------------------------------------------------------
// GQA decode attention over the paged KV cache, ggml's op order exactly
// (engine.cpp:1751-1761):
//   kq_j  = (float) sum_i (double)(k_ji * q_i)          ggml_mul_mat F32
//   s_j   = kq_j * (1/sqrt(hd)); M = max_j s_j          ggml_soft_max_ext
//   p_j   = exp(s_j - M); S = sum_j (double) p_j; p'_j = p_j * (float)(1/S)
//   o_i   = (float) sum_j (double)(v_ji * p'_j)         ggml_mul_mat F32
// One thread-block cluster per (token, kv head); each CTA of the cluster owns
// a contiguous slice of positions.  The cross-CTA steps (global max, global
// sum, the final o reduction) go through distributed shared memory with
// cluster barriers, so the two-pass softmax is exact without a second kernel.
// 128 threads; the GQA group's query heads share each K/V load.
// ---------------------------------------------------------------------------
constexpr int ATT_THREADS = 128;
constexpr int ATT_MAXG = 16;  // max query heads per kv head

template <int HD>
__global__ void __launch_bounds__(ATT_THREADS) attn_kernel(const AttnParams p) {
  namespace cg = cooperative_groups;
  pdl_launch_dependents();
  pdl_wait();
  cg::cluster_group cl = cg::this_cluster();
  const int C = (int)cl.num_blocks();
  const int rank = (int)cl.block_rank();
  const int hk = blockIdx.x / C, t = blockIdx.y;
  const int Hkv = p.kv.n_head_kv;
  const int gqa = p.n_head / Hkv;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int PER = HD / 32;  // output dims per lane
  constexpr int QD = HD / 4;    // dims per lane in the score pass (4 lanes per position)

  // shared layout (attn_smem_bytes): opart [gqa][HD] f64 | qs [gqa][HD] f32 |
  // lsum [gqa] f64 | wred [4][gqa] f64 | lmax [gqa] f32 | sc [gqa][max_chunk] f32
  extern __shared__ __align__(16) uint8_t asmem[];
  double* opart = reinterpret_cast<double*>(asmem);
  float* qs = reinterpret_cast<float*>(opart + gqa * HD);
  double* lsum = reinterpret_cast<double*>(qs + gqa * HD);
  double* wred = lsum + gqa;
  float* lmax = reinterpret_cast<float*>(wred + 4 * gqa);
  float* sc = lmax + ((gqa + 3) & ~3);
  int n_kv = p.pos[t] + 1;
  if (n_kv < 1 || n_kv > p.kv.max_pages * 16) {  // outside the page table: no access, report
    if (tid == 0 && rank == 0) atomicExch(p.status, ERR_BAD_POS);
    n_kv = 0;
  }
  const int chunk = (n_kv + C - 1) / C;
  const int j0 = rank * chunk;
  const int nloc = max(0, min(n_kv, j0 + chunk) - j0);
  const float scale = __fdiv_rn(1.0f, sqrtf((float)HD));
  const int* ptab = p.kv.page_table + t * p.kv.max_pages;
  const int q0 = hk * gqa;

  for (int i = tid; i < gqa * HD; i += ATT_THREADS) qs[i] = p.q[((int64_t)t * p.n_head + q0) * HD + i];
  __syncthreads();

  // ---- pass 1: scores of this CTA's positions; 8 positions per warp step
  const int n_oct = (nloc + 7) >> 3;
  for (int item = warp; item < gqa * n_oct; item += ATT_THREADS / 32) {
    const int h = item % gqa, oct = item / gqa;
    const int jl = oct * 8 + (lane >> 2);
    const int c = lane & 3;
    double acc = 0.0;
    if (jl < nloc) {
      const int j = j0 + jl;
      const int64_t off = (((int64_t)ptab[j >> 4] * Hkv + hk) * 16 + (j & 15)) * HD + c * QD;
      const float* qh = qs + h * HD + c * QD;
      if (p.kv.f16) {
        const __half* kr = reinterpret_cast<const __half*>(p.kv.k) + off;
#pragma unroll
        for (int i = 0; i < QD; i += 8) {
          const uint4 raw = *reinterpret_cast<const uint4*>(kr + i);
          const __half2* hv = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 kf = __half22float2(hv[e]);
            acc += (double)__fmul_rn(kf.x, qh[i + 2 * e]);
            acc += (double)__fmul_rn(kf.y, qh[i + 2 * e + 1]);
          }
        }
      } else {
        const float* kr = reinterpret_cast<const float*>(p.kv.k) + off;
#pragma unroll
        for (int i = 0; i < QD; i += 4) {
          const float4 kf = *reinterpret_cast<const float4*>(kr + i);
          acc += (double)__fmul_rn(kf.x, qh[i]);
          acc += (double)__fmul_rn(kf.y, qh[i + 1]);
          acc += (double)__fmul_rn(kf.z, qh[i + 2]);
          acc += (double)__fmul_rn(kf.w, qh[i + 3]);
        }
      }
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    if (c == 0 && jl < nloc) sc[h * p.max_chunk + jl] = __fmul_rn((float)acc, scale);
  }
  __syncthreads();
  // local max per head
  for (int h = warp; h < gqa; h += ATT_THREADS / 32) {
    float m = -INFINITY;
    for (int jl = lane; jl < nloc; jl += 32) m = fmaxf(m, sc[h * p.max_chunk + jl]);
    m = warp_max(m);
    if (lane == 0) lmax[h] = m;
  }
  cl.sync();
  // ---- pass 2: global max, exp, local sum
  for (int h = 0; h < gqa; ++h) {
    float M = -INFINITY;
    for (int r = 0; r < C; ++r) M = fmaxf(M, cl.map_shared_rank(lmax, r)[h]);
    double s = 0.0;
    for (int jl = tid; jl < nloc; jl += ATT_THREADS) {
      const float e = sfk_expf(__fsub_rn(sc[h * p.max_chunk + jl], M));
      sc[h * p.max_chunk + jl] = e;
      s += (double)e;
    }
    s = warp_sum_d(s);
    if (lane == 0) wred[warp * gqa + h] = s;
  }
  __syncthreads();
  if (tid < gqa) {
    double s = 0.0;
    for (int w = 0; w < ATT_THREADS / 32; ++w) s += wred[w * gqa + tid];
    lsum[tid] = s;
  }
  cl.sync();
  // ---- pass 3: p' = p * (float)(1/S); o_i = sum_j (double)(v_ji * p'_j)
  for (int h = warp; h < gqa; h += ATT_THREADS / 32) {
    double S = 0.0;
    for (int r = 0; r < C; ++r) S += cl.map_shared_rank(lsum, r)[h];
    const float inv = (float)(1.0 / S);
    double o[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) o[i] = 0.0;
    for (int jl = 0; jl < nloc; ++jl) {
      const int j = j0 + jl;
      const float pj = __fmul_rn(sc[h * p.max_chunk + jl], inv);
      const int64_t off = (((int64_t)ptab[j >> 4] * Hkv + hk) * 16 + (j & 15)) * HD + lane * PER;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const float vv = p.kv.f16 ? __half2float(reinterpret_cast<const __half*>(p.kv.v)[off + i])
                                  : reinterpret_cast<const float*>(p.kv.v)[off + i];
        o[i] += (double)__fmul_rn(vv, pj);
      }
    }
#pragma unroll
    for (int i = 0; i < PER; ++i) opart[h * HD + lane * PER + i] = o[i];
  }
  cl.sync();
  // ---- reduce the cluster's partial outputs on rank 0
  if (rank == 0) {
    for (int i = tid; i < gqa * HD; i += ATT_THREADS) {
      double o = 0.0;
      for (int r = 0; r < C; ++r) o += cl.map_shared_rank(opart, r)[i];
      p.out[((int64_t)t * p.n_head + q0) * HD + i] = (float)o;
    }
  }
  cl.sync();
}

size_t attn_smem_bytes(int hd, int gqa, int max_chunk) {
  return (size_t)gqa * hd * 8 + (size_t)gqa * hd * 4 + (size_t)gqa * 8 + 4 * (size_t)gqa * 8 +
         (size_t)((gqa + 3) & ~3) * 4 + (size_t)gqa * max_chunk * 4;
}

// ---------------------------------------------------------------------------
// router: ffn_norm -> quantized expert input; logits = W_r x (f32);
// probs = softmax; top-k (descending, lower index on ties);
// w = probs[ids] / max(sum, 6.103515625e-5)   (engine.cpp:1909-1924)
// grid b, 256 threads.  The last CTA builds the slot lists.
// ---------------------------------------------------------------------------
constexpr int RT_THREADS = 256;
constexpr int RT_MAXE = 512;

__global__ void __launch_bounds__(RT_THREADS) router_kernel(const RouterParams p) {
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ __align__(16) uint8_t rsm[];
  float* xn = reinterpret_cast<float*>(rsm);  // [d]
  __shared__ double red[RT_THREADS / 32 + 1];
  __shared__ float probs[RT_MAXE];
  __shared__ int last_flag;
  const int t = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int d = p.d;
  const float* x = p.x + (int64_t)t * d;
  double s = 0.0;
  for (int c = tid; c < d; c += RT_THREADS) s += (double)__fmul_rn(x[c], x[c]);
  s = warp_sum_d(s);
  if (lane == 0) red[warp] = s;
  __syncthreads();
  if (tid == 0) {
    double tot = 0.0;
    for (int w = 0; w < RT_THREADS / 32; ++w) tot += red[w];
    red[RT_THREADS / 32] = tot;
  }
  __syncthreads();
  const float mean = (float)(red[RT_THREADS / 32] / (double)d);
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
  for (int c = tid; c < d; c += RT_THREADS) {
    const float v = __fmul_rn(__fmul_rn(x[c], scale), p.norm_w[c]);
    xn[c] = v;
    if (p.xn) p.xn[(int64_t)t * d + c] = v;
  }
  __syncthreads();
  uint8_t* xq = p.xq + (int64_t)t * qact_bytes(d);
  for (int blk = warp; blk < d / QK_K; blk += RT_THREADS / 32) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = xn[blk * QK_K + lane * 8 + i];
    qact_put(p.act_type, xq, d, blk, v, lane);
  }
  // router logits (F32 weights)
  // ggml F32 mul_mat: float products summed in double
  for (int e = warp; e < p.E; e += RT_THREADS / 32) {
    const float* wr = p.w_r + (int64_t)e * d;
    double a = 0.0;
    for (int c = lane * 4; c < d; c += 128) {
      const float4 w4 = *reinterpret_cast<const float4*>(wr + c);
      a += (double)__fmul_rn(w4.x, xn[c]);
      a += (double)__fmul_rn(w4.y, xn[c + 1]);
      a += (double)__fmul_rn(w4.z, xn[c + 2]);
      a += (double)__fmul_rn(w4.w, xn[c + 3]);
    }
    a = warp_sum_d(a);
    if (lane == 0) probs[e] = (float)a;
  }
  __syncthreads();
  if (warp == 0) {
    // softmax (scale 1): max, e^(x-max), sum in double, * (float)(1/sum)
    float mx = -INFINITY;
    for (int e = lane; e < p.E; e += 32) mx = fmaxf(mx, probs[e]);
    mx = warp_max(mx);
    double sum = 0.0;
    for (int e = lane; e < p.E; e += 32) {
      const float ex = sfk_expf(__fsub_rn(probs[e], mx));
      probs[e] = ex;
      sum += (double)ex;
    }
    sum = warp_sum_d(sum);
    const float inv = (float)(1.0 / sum);
    for (int e = lane; e < p.E; e += 32) probs[e] = __fmul_rn(probs[e], inv);
    __syncwarp();
    // top-k by repeated warp argmax (lower index wins ties)
    int ids[16];
    float wsel[16];
    double wsum = 0.0;
    for (int j = 0; j < p.k; ++j) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int e = lane; e < p.E; e += 32) {
        bool taken = false;
        for (int jj = 0; jj < j; ++jj) taken |= (ids[jj] == e);
        if (!taken && (probs[e] > bv || (probs[e] == bv && e < bi))) { bv = probs[e]; bi = e; }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      ids[j] = bi;
      wsel[j] = bv;
      wsum += (double)bv;
    }
    float ws = (float)wsum;
    if (ws < 6.103515625e-5f) ws = 6.103515625e-5f;
    if (lane == 0) {
      for (int j = 0; j < p.k; ++j) {
        p.route->ids[t * p.k + j] = ids[j];
        p.route->w[t * p.k + j] = __fdiv_rn(wsel[j], ws);
      }
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int old = atomicAdd(p.counter, 1);
    last_flag = (old == p.b - 1);
  }
  __syncthreads();
  if (!last_flag || tid != 0) return;
  __threadfence();
  // slot lists: distinct experts ascending, each with its pairs ascending
  Route* r = p.route;
  const int np = p.b * p.k;
  int ns = 0;
  int ids_l[MAXP];
  for (int i = 0; i < np; ++i) ids_l[i] = __ldcg(&r->ids[i]);
  int prev = -1;
  r->slot_off[0] = 0;
  int fill = 0;
  while (true) {
    int nxt = 0x7fffffff;
    for (int i = 0; i < np; ++i)
      if (ids_l[i] > prev && ids_l[i] < nxt) nxt = ids_l[i];
    if (nxt == 0x7fffffff) break;
    r->slot_expert[ns] = nxt;
    for (int i = 0; i < np; ++i)
      if (ids_l[i] == nxt) r->slot_pairs[fill++] = i;
    r->slot_off[++ns] = fill;
    prev = nxt;
  }
  r->n_slots = ns;
  r->k = p.k;
  r->b = p.b;
  atomicExch(p.counter, 0);
}

// ---------------------------------------------------------------------------
// embedding: token id -> dequantized row (ggml_get_rows, engine.cpp:2708-2723)
// one CTA; greedy mode takes the previous step's argmax and clears it.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) embed_kernel(const EmbedParams p) {
  pdl_launch_dependents();
  pdl_wait();
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
      atomicExch(p.status, ERR_BAD_ID);
      tok = 0;
    }
    toks[tid] = tok;
    int pos = p.pos_in ? p.pos_in[tid] : p.pos_state[tid];
    p.pos_cur[tid] = pos;
    if (p.pos_state) p.pos_state[tid] = pos + 1;
    p.tok_hist[tid] = tok;
  }
  __syncthreads();
  if (tid < p.b) p.argmax_key[tid] = 0ull;
  const int64_t rb = (int64_t)dev_gguf_row_bytes(p.type, p.d);
  for (int t = 0; t < p.b; ++t) {
    const uint8_t* row = p.tok_embd + (int64_t)toks[t] * rb;
    for (int i = tid; i < p.d; i += blockDim.x) p.x[(int64_t)t * p.d + i] = gguf_dequant_one(p.type, row, i);
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
  const StreamPlan pl = make_plan(p);
  static bool attr_set[2] = {false, false};
  (void)attr_set;
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

template <int HD>
static cudaError_t launch_attn_t(const AttnParams& p, cudaStream_t st, bool pdl) {
  const size_t smem = attn_smem_bytes(HD, p.n_head / p.kv.n_head_kv, p.max_chunk);
  cudaError_t e = cudaFuncSetAttribute(attn_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  if (p.cluster > 8) {
    e = cudaFuncSetAttribute(attn_kernel<HD>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
  }
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
  return cudaLaunchKernelEx(&cfg, attn_kernel<HD>, p);
}

cudaError_t launch_attn(const AttnParams& p, cudaStream_t st, bool pdl) {
  if (p.n_head % p.kv.n_head_kv || p.n_head / p.kv.n_head_kv > ATT_MAXG || p.cluster < 1 || p.cluster > 16)
    return cudaErrorInvalidValue;
  switch (p.kv.head_dim) {
    case 32: return launch_attn_t<32>(p, st, pdl);
    case 64: return launch_attn_t<64>(p, st, pdl);
    case 128: return launch_attn_t<128>(p, st, pdl);
    case 256: return launch_attn_t<256>(p, st, pdl);
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
  return launch_pdl(embed_kernel, dim3(1), dim3(256), 0, st, pdl, p);
}

}  // namespace sfk
