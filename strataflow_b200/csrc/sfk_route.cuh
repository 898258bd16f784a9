// sfk_route.cuh -- the MoE router of one token, shared by the standalone
// router kernel and the gate/up kernel that routes in its own prologue.
//
// engine.cpp:1909-1924 of the reference: ffn_norm (RMSNorm * w), logits =
// W_r . x with F32 weights (float products summed in double, ggml's F32
// mul_mat), probs = soft_max (max-subtracted, exp, double sum, * (float)(1/S)),
// top-k descending (lower index on ties), weights = probs[ids] /
// max(sum, 6.103515625e-5).  The normalised input is also quantized to the
// expert weights' activation type for the gate/up dot products.
#pragma once
#include "sfk_act.cuh"
#include "sfk_device.cuh"
#include "sfk_kernels.cuh"

namespace sfk {

// Softmax over the E router logits in probs (replaced by the
// probabilities), then top-k (lower index on ties) and the renormalised
// weights probs[ids] / max(sum, 6.103515625e-5).  One warp.
__device__ inline void route_select(float* probs, int E, int k, int* ids_out, float* w_out, int lane) {
  if (E <= 32) {
    // one expert per lane; butterflies over the ceil(log2 E) low lane bits only
    int L = 0;
    while ((1 << L) < E) ++L;
    float pv = lane < E ? probs[lane] : -INFINITY;
    float mx = pv;
    for (int o = (1 << L) >> 1; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float ex = lane < E ? sfk_expf(__fsub_rn(pv, mx)) : 0.0f;
    double sum = (double)ex;
    for (int o = (1 << L) >> 1; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float inv = (float)(1.0 / sum);
    pv = lane < E ? __fmul_rn(ex, inv) : -INFINITY;
    double wsum = 0.0;
    for (int j = 0; j < k; ++j) {
      float bv = pv;
      int bi = lane < E ? lane : 0x7fffffff;
      for (int o = (1 << L) >> 1; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      if (lane == 0) {
        ids_out[j] = bi;
        w_out[j] = bv;
      }
      if (lane == bi) pv = -INFINITY;  // knocked out of the next rounds
      wsum += (double)bv;
    }
    __syncwarp();
    float ws = (float)wsum;
    if (ws < 6.103515625e-5f) ws = 6.103515625e-5f;
    if (lane < k) w_out[lane] = __fdiv_rn(w_out[lane], ws);
    __syncwarp();
    return;
  }
  float mx = -INFINITY;
  for (int e = lane; e < E; e += 32) mx = fmaxf(mx, probs[e]);
  mx = warp_max(mx);
  double sum = 0.0;
  for (int e = lane; e < E; e += 32) {
    const float ex = sfk_expf(__fsub_rn(probs[e], mx));
    probs[e] = ex;
    sum += (double)ex;
  }
  sum = warp_sum_d(sum);
  const float inv = (float)(1.0 / sum);
  for (int e = lane; e < E; e += 32) probs[e] = __fmul_rn(probs[e], inv);
  __syncwarp();
  // top-k: the winner of each round is knocked out of probs (-inf; a
  // probability is never negative); its weight waits in w_out
  double wsum = 0.0;
  for (int j = 0; j < k; ++j) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int e = lane; e < E; e += 32) {
      const float pe = probs[e];
      if (pe > bv || (pe == bv && e < bi)) { bv = pe; bi = e; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) {
      ids_out[j] = bi;
      w_out[j] = bv;
      probs[bi] = -INFINITY;
    }
    __syncwarp();
    wsum += (double)bv;
  }
  float ws = (float)wsum;
  if (ws < 6.103515625e-5f) ws = 6.103515625e-5f;
  if (lane < k) w_out[lane] = __fdiv_rn(w_out[lane], ws);
  __syncwarp();
}

// ffn_norm of one token by NWARPS warps (threads 0 .. 32*NWARPS-1 of the
// block; `sync` synchronises exactly those threads): RMSNorm (squares summed
// in double, mean = (float)(sum/d), scale = 1/sqrtf(mean+eps), y = x*scale)
// times the weight, written to xn [d] (shared) and xn_global (optional), and
// quantized to the expert weights' activation type into xq.  Scratch: red
// [NWARPS+1] doubles.
template <int NWARPS, int RB, typename Sync>
__device__ void route_norm(const float* x, const float* norm_w, int d, float eps, int act_type, uint8_t* xq, float* xn,
                           double* red, float* xn_global, Sync sync) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nblk = d / QK_K;
  if (nblk <= RB * NWARPS) {  // RB 256-column blocks per warp fit in registers
    // x and the norm weight of this warp's blocks (warp, warp + NWARPS, ...),
    // 8 columns per lane, fetched in one round trip
    float xv[RB][8], wv[RB][8];
#pragma unroll
    for (int i = 0; i < RB; ++i) {
      const int blk = warp + i * NWARPS;
      if (blk < nblk) {
        const float4* xp = reinterpret_cast<const float4*>(x + blk * QK_K + lane * 8);
        const float4* wp = reinterpret_cast<const float4*>(norm_w + blk * QK_K + lane * 8);
        const float4 x0 = xp[0], x1 = xp[1], w0 = wp[0], w1 = wp[1];
        xv[i][0] = x0.x; xv[i][1] = x0.y; xv[i][2] = x0.z; xv[i][3] = x0.w;
        xv[i][4] = x1.x; xv[i][5] = x1.y; xv[i][6] = x1.z; xv[i][7] = x1.w;
        wv[i][0] = w0.x; wv[i][1] = w0.y; wv[i][2] = w0.z; wv[i][3] = w0.w;
        wv[i][4] = w1.x; wv[i][5] = w1.y; wv[i][6] = w1.z; wv[i][7] = w1.w;
      }
    }
    double s = 0.0;
#pragma unroll
    for (int i = 0; i < RB; ++i)
      if (warp + i * NWARPS < nblk) {
#pragma unroll
        for (int j = 0; j < 8; ++j) s += (double)__fmul_rn(xv[i][j], xv[i][j]);
      }
    s = warp_sum_d(s);
    if (lane == 0) red[warp] = s;
    sync();
    double tot = 0.0;
    for (int w = 0; w < NWARPS; ++w) tot += red[w];  // every thread, same order
    const float mean = (float)(tot / (double)d);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    float vn[RB][8];
#pragma unroll
    for (int i = 0; i < RB; ++i) {
      const int blk = warp + i * NWARPS;
      if (blk < nblk) {
#pragma unroll
        for (int j = 0; j < 8; ++j) vn[i][j] = __fmul_rn(__fmul_rn(xv[i][j], scale), wv[i][j]);
        float4* xo = reinterpret_cast<float4*>(xn + blk * QK_K + lane * 8);
        xo[0] = make_float4(vn[i][0], vn[i][1], vn[i][2], vn[i][3]);
        xo[1] = make_float4(vn[i][4], vn[i][5], vn[i][6], vn[i][7]);
        if (xn_global) {
          float4* xg = reinterpret_cast<float4*>(xn_global + blk * QK_K + lane * 8);
          xg[0] = make_float4(vn[i][0], vn[i][1], vn[i][2], vn[i][3]);
          xg[1] = make_float4(vn[i][4], vn[i][5], vn[i][6], vn[i][7]);
        }
      }
    }
    const int nb = warp < nblk ? (nblk - warp + NWARPS - 1) / NWARPS : 0;
    if (act_type == T_Q8_K) {
      qact_put_q8k_blocks<RB>(xq, d, warp, NWARPS, nb < RB ? nb : RB, vn, lane);
    } else {
#pragma unroll
      for (int i = 0; i < RB; ++i)
        if (i < nb) qact_put(act_type, xq, d, warp + i * NWARPS, vn[i], lane);
    }
    sync();
  } else {
    double s = 0.0;
    for (int c = tid; c < d; c += NWARPS * 32) s += (double)__fmul_rn(x[c], x[c]);
    s = warp_sum_d(s);
    if (lane == 0) red[warp] = s;
    sync();
    if (tid == 0) {
      double tot = 0.0;
      for (int w = 0; w < NWARPS; ++w) tot += red[w];
      red[NWARPS] = tot;
    }
    sync();
    const float mean = (float)(red[NWARPS] / (double)d);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    for (int c = tid; c < d; c += NWARPS * 32) {
      const float v = __fmul_rn(__fmul_rn(x[c], scale), norm_w[c]);
      xn[c] = v;
      if (xn_global) xn_global[c] = v;
    }
    sync();
    for (int blk = warp; blk < nblk; blk += NWARPS) {
      float v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = xn[blk * QK_K + lane * 8 + i];
      qact_put(act_type, xq, d, blk, v, lane);
    }
  }
}

// Routing of one token by NWARPS warps: route_norm, then logits = W_r . xn
// (F32 weights, float products summed in double), softmax, top-k.  Shared
// scratch: xn [d], seg [E*4] doubles, probs [E], red [NWARPS+1] doubles.
// Writes the qact of ffn_norm(x) to xq and the k ids / weights to ids_out /
// w_out.
template <int NWARPS, typename Sync>
__device__ void route_one(const float* x, const float* norm_w, const float* w_r, int d, int E, int k, float eps,
                          int act_type, uint8_t* xq, float* xn, double* seg, float* probs, double* red, int* ids_out,
                          float* w_out, float* xn_global, Sync sync) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  route_norm<NWARPS, (NWARPS >= 16 ? 1 : 4)>(x, norm_w, d, eps, act_type, xq, xn, red, xn_global, sync);
  // router logits; each expert row is cut into nseg segments of a multiple of
  // 128 columns when there are fewer experts than warps; segment partials are
  // added in order
  int nseg = 1;
  while (nseg < 4 && E * nseg * 2 <= NWARPS && d % (nseg * 2 * 128) == 0) nseg *= 2;
  const int seglen = d / nseg;
  for (int item = warp; item < E * nseg; item += NWARPS) {
    const int e = item / nseg, sg = item % nseg;
    const float* wr = w_r + (int64_t)e * d + sg * seglen;
    const float* xs = xn + sg * seglen;
    double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;  // four chains (double sums are order-free here)
    int c = lane * 4;
    for (; c + 7 * 128 < seglen; c += 8 * 128) {
      float4 w4[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) w4[u] = *reinterpret_cast<const float4*>(wr + c + u * 128);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float4 x4 = *reinterpret_cast<const float4*>(xs + c + u * 128);
        a0 += (double)__fmul_rn(w4[u].x, x4.x);
        a1 += (double)__fmul_rn(w4[u].y, x4.y);
        a2 += (double)__fmul_rn(w4[u].z, x4.z);
        a3 += (double)__fmul_rn(w4[u].w, x4.w);
      }
    }
    for (; c < seglen; c += 128) {
      const float4 w4 = *reinterpret_cast<const float4*>(wr + c);
      const float4 x4 = *reinterpret_cast<const float4*>(xs + c);
      a0 += (double)__fmul_rn(w4.x, x4.x);
      a1 += (double)__fmul_rn(w4.y, x4.y);
      a2 += (double)__fmul_rn(w4.z, x4.z);
      a3 += (double)__fmul_rn(w4.w, x4.w);
    }
    double a = (a0 + a1) + (a2 + a3);
    a = warp_sum_d(a);
    if (lane == 0) seg[e * nseg + sg] = a;
  }
  sync();
  for (int e = tid; e < E; e += NWARPS * 32) {
    double a = 0.0;
    for (int sg = 0; sg < nseg; ++sg) a += seg[e * nseg + sg];
    probs[e] = (float)a;
  }
  sync();
  if (warp == 0) route_select(probs, E, k, ids_out, w_out, lane);
  sync();
}

// The same slot lists built by one warp when np <= 32 and every local id <
// 64: lane i holds pair i; the slot of an expert is the number of distinct
// smaller experts in use, a pair's place in its slot the number of earlier
// pairs of the same expert.  Only experts [e0, e0 + eloc) get slots (eloc = 0:
// all), numbered from e0.
__device__ inline void build_slots_warp(const int* ids, int np, Route* r, int lane, int e0 = 0, int eloc = 0) {
  int id = lane < np ? ids[lane] : -1;
  if (eloc > 0 && id >= 0) id = (id >= e0 && id < e0 + eloc) ? id - e0 : -1;
  const unsigned act = __ballot_sync(0xffffffffu, id >= 0);
  unsigned lo = 0, hi = 0;
  if (id >= 0 && id < 32) lo = 1u << id;
  if (id >= 32) hi = 1u << (id - 32);
  lo = __reduce_or_sync(0xffffffffu, lo);
  hi = __reduce_or_sync(0xffffffffu, hi);
  const int n_lo = __popc(lo), ns = n_lo + __popc(hi);
  // expert b in use (bit b) sits in slot popc(bits below b)
  if (lo & (1u << lane)) r->slot_expert[__popc(lo & ((1u << lane) - 1u))] = lane;
  if (hi & (1u << lane)) r->slot_expert[n_lo + __popc(hi & ((1u << lane) - 1u))] = 32 + lane;
  // pairs of each expert, and the pairs of all smaller experts before them
  const unsigned same = __match_any_sync(0xffffffffu, id) & act;
  const int slot = id < 0 ? 0 : (id < 32 ? __popc(lo & ((1u << id) - 1u)) : n_lo + __popc(hi & ((1u << (id - 32)) - 1u)));
  int before = 0;  // local pairs whose expert is smaller than mine
  for (int j = 0; j < np; ++j) {
    const int oj = __shfl_sync(0xffffffffu, id, j);
    before += (oj >= 0 && oj < id) ? 1 : 0;
  }
  const int place = __popc(same & ((1u << lane) - 1u));
  if (id >= 0) r->slot_pairs[before + place] = lane;
  // slot_off[s] = local pairs of the s smallest experts: the first pair of
  // slot s knows it, and the total closes the list
  if (id >= 0 && place == 0) r->slot_off[slot] = before;
  if (lane == 0) {
    r->slot_off[ns] = __popc(act);
    r->n_slots = ns;
  }
  __syncwarp();
}

// Slot lists from the pairs' expert ids: distinct experts ascending, each with
// its pairs ascending.  Only experts [e0, e0 + eloc) get slots (eloc = 0: all),
// numbered from e0.  One thread.
__device__ inline void build_slots(const int* ids, int np, Route* r, int e0 = 0, int eloc = 0) {
  const int lo = eloc > 0 ? e0 : 0, hi = eloc > 0 ? e0 + eloc : 0x7fffffff;
  int ns = 0, fill = 0, prev = lo - 1;
  r->slot_off[0] = 0;
  while (true) {
    int nxt = 0x7fffffff;
    for (int i = 0; i < np; ++i)
      if (ids[i] > prev && ids[i] < nxt) nxt = ids[i];
    if (nxt == 0x7fffffff || nxt >= hi) break;
    r->slot_expert[ns] = nxt - lo;
    for (int i = 0; i < np; ++i)
      if (ids[i] == nxt) r->slot_pairs[fill++] = i;
    r->slot_off[++ns] = fill;
    prev = nxt;
  }
  r->n_slots = ns;
}

}  // namespace sfk
