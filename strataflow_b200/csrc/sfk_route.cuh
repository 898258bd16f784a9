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

// Routing of one token by NWARPS warps (threads 0 .. 32*NWARPS-1 of the
// block); `sync` synchronises exactly those threads.  Shared scratch: xn [d],
// seg [E*4] doubles, probs [E], red [NWARPS+1] doubles.  Writes the qact of
// ffn_norm(x) to xq and the k ids / weights to ids_out / w_out.
template <int NWARPS, typename Sync>
__device__ void route_one(const float* x, const float* norm_w, const float* w_r, int d, int E, int k, float eps,
                          int act_type, uint8_t* xq, float* xn, double* seg, float* probs, double* red, int* ids_out,
                          float* w_out, float* xn_global, Sync sync) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
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
  for (int blk = warp; blk < d / QK_K; blk += NWARPS) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = xn[blk * QK_K + lane * 8 + i];
    qact_put(act_type, xq, d, blk, v, lane);
  }
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
    double a = 0.0;
    int c = lane * 4;
    for (; c + 7 * 128 < seglen; c += 8 * 128) {
      float4 w4[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) w4[u] = *reinterpret_cast<const float4*>(wr + c + u * 128);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int cc = c + u * 128;
        a += (double)__fmul_rn(w4[u].x, xs[cc]);
        a += (double)__fmul_rn(w4[u].y, xs[cc + 1]);
        a += (double)__fmul_rn(w4[u].z, xs[cc + 2]);
        a += (double)__fmul_rn(w4[u].w, xs[cc + 3]);
      }
    }
    for (; c < seglen; c += 128) {
      const float4 w4 = *reinterpret_cast<const float4*>(wr + c);
      a += (double)__fmul_rn(w4.x, xs[c]);
      a += (double)__fmul_rn(w4.y, xs[c + 1]);
      a += (double)__fmul_rn(w4.z, xs[c + 2]);
      a += (double)__fmul_rn(w4.w, xs[c + 3]);
    }
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
  if (warp == 0) {
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
    int ids[16];
    float wsel[16];
    double wsum = 0.0;
    for (int j = 0; j < k; ++j) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int e = lane; e < E; e += 32) {
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
      for (int j = 0; j < k; ++j) {
        ids_out[j] = ids[j];
        w_out[j] = __fdiv_rn(wsel[j], ws);
      }
    }
  }
  sync();
}

// Slot lists from the pairs' expert ids: distinct experts ascending, each with
// its pairs ascending.  One thread.
__device__ inline void build_slots(const int* ids, int np, Route* r) {
  int ns = 0, fill = 0, prev = -1;
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
}

}  // namespace sfk
