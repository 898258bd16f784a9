// sfk_sample.cu -- token sampling on the device for the generate loop.
//
// The reference declares sf_sampling_params (temperature, top_p, top_k, seed,
// max_tokens: include/strataflow/strataflow.h:193-199) but its generate loop
// never reads them and always takes the argmax (src/api/strataflow_api.cpp:
// 308-335).  The sampling defined here, restated in the CPU oracle
// (sfo_sample), is:
//   * temperature <= 0: greedy -- the argmax, first maximum winning (the
//     lm_head kernel's key; this kernel is not launched);
//   * p_i = exp((l_i - max l) * (1 / T)) with the shared exp (sfk_expf);
//   * top_k > 0: keep the k largest p, ties broken by the lower index;
//   * top_p < 1: of those, keep the shortest prefix in (p descending, index
//     ascending) order whose mass reaches top_p times the kept mass;
//   * draw u in [0, 1) from splitmix64(seed, step) and return the first kept
//     index, in index order, whose running mass exceeds u times the kept mass.
// The cut-offs are found without sorting: the kept sets are {p > t} plus the
// lowest-index ties at t, and t is found by bisection on the float bit pattern
// (p >= 0, so the bit patterns are ordered like the values).  Sums are in
// double.  One CTA of 1024 threads; V up to a few hundred thousand.
#include <cuda_runtime.h>

#include <cstdint>

#include "sfk_device.cuh"
#include "sfk_sample.cuh"

namespace sfk {
namespace {

constexpr int SM_THREADS = 1024;
constexpr int SM_WARPS = SM_THREADS / 32;

struct Red {
  double d[SM_WARPS];
  float f[SM_WARPS];
  int i[SM_WARPS];
};

__device__ double block_sum_d(double v, Red& r) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  v = warp_sum_d(v);
  __syncthreads();
  if (lane == 0) r.d[warp] = v;
  __syncthreads();
  double t = 0.0;
  for (int w = 0; w < SM_WARPS; ++w) t += r.d[w];  // every thread, the same order
  return t;
}
__device__ int block_sum_i(int v, Red& r) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) r.i[warp] = v;
  __syncthreads();
  int t = 0;
  for (int w = 0; w < SM_WARPS; ++w) t += r.i[w];
  return t;
}
__device__ float block_max_f(float v, Red& r) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) r.f[warp] = v;
  __syncthreads();
  float t = r.f[0];
  for (int w = 1; w < SM_WARPS; ++w) t = fmaxf(t, r.f[w]);
  return t;
}

__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Threads own contiguous index ranges [lo, hi) (V split into SM_THREADS runs),
// so per-thread partial sums in index order followed by an ordered scan give
// the running mass in index order.
__global__ void __launch_bounds__(SM_THREADS) sample_kernel(const float* logits, int V, float temperature, int top_k,
                                                            float top_p, uint64_t seed, int step, float* p,
                                                            unsigned long long* key_out, int* tok_out) {
  __shared__ Red red;
  __shared__ double scan[SM_THREADS];
  const int tid = threadIdx.x;
  const int per = (V + SM_THREADS - 1) / SM_THREADS;
  const int lo = min(V, tid * per), hi = min(V, lo + per);

  // p_i = exp((l_i - max) / T)
  float mx = -INFINITY;
  for (int i = lo; i < hi; ++i) mx = fmaxf(mx, logits[i]);
  mx = block_max_f(mx, red);
  const float invT = __fdiv_rn(1.0f, temperature);
  for (int i = lo; i < hi; ++i) p[i] = sfk_expf(__fmul_rn(__fsub_rn(logits[i], mx), invT));
  __syncthreads();

  // keep[i] is p_i > t, or p_i == t and i among the first `ties` indices with
  // p == t; t and ties come from the two filters below.
  uint32_t t_bits = 0;   // keep everything with p >= 0 (all)
  int ties = 0x7fffffff;
  if (top_k > 0 && top_k < V) {
    // largest t with count(p >= t) >= k
    uint32_t lo_b = 0, hi_b = 0x3F800000u;  // p in [0, 1]
    while (lo_b < hi_b) {
      const uint32_t mid = lo_b + (hi_b - lo_b + 1) / 2;
      const float t = __uint_as_float(mid);
      int c = 0;
      for (int i = lo; i < hi; ++i) c += p[i] >= t ? 1 : 0;
      c = block_sum_i(c, red);
      if (c >= top_k) lo_b = mid; else hi_b = mid - 1;
    }
    t_bits = lo_b;
    const float t = __uint_as_float(t_bits);
    int gt = 0;
    for (int i = lo; i < hi; ++i) gt += p[i] > t ? 1 : 0;
    gt = block_sum_i(gt, red);
    ties = top_k - gt;  // the lowest-index ties at t fill the k
  }
  // the kept set as a predicate over (i, p_i)
  auto kept_k = [&](int i, float v, int tie_rank) {
    const float t = __uint_as_float(t_bits);
    return v > t || (v == t && tie_rank < ties);
  };
  // rank of index i among the ties at t (in index order): prefix counts
  auto tie_ranks_base = [&](float t) {
    int c = 0;
    for (int i = lo; i < hi; ++i) c += p[i] == t ? 1 : 0;
    scan[tid] = (double)c;
    __syncthreads();
    if (tid == 0) {
      double a = 0.0;
      for (int w = 0; w < SM_THREADS; ++w) {
        const double x = scan[w];
        scan[w] = a;
        a += x;
      }
    }
    __syncthreads();
    const int base = (int)scan[tid];
    __syncthreads();
    return base;
  };
  const int kbase = tie_ranks_base(__uint_as_float(t_bits));
  // mass of the top-k set
  double mk = 0.0;
  {
    int r = kbase;
    const float t = __uint_as_float(t_bits);
    for (int i = lo; i < hi; ++i) {
      const float v = p[i];
      const bool tie = v == t;
      if (kept_k(i, v, r)) mk += (double)v;
      r += tie ? 1 : 0;
    }
  }
  mk = block_sum_d(mk, red);

  uint32_t u_bits = t_bits;  // nucleus threshold (>= the top-k one)
  int u_ties = ties;
  if (top_p < 1.0f) {
    const double target = (double)top_p * mk;
    // largest t2 >= t with mass(top-k set, p >= t2) >= target
    uint32_t lo_b = t_bits, hi_b = 0x3F800000u;
    while (lo_b < hi_b) {
      const uint32_t mid = lo_b + (hi_b - lo_b + 1) / 2;
      const float t2 = __uint_as_float(mid);
      double m = 0.0;
      int r = kbase;
      const float t = __uint_as_float(t_bits);
      for (int i = lo; i < hi; ++i) {
        const float v = p[i];
        if (v >= t2 && kept_k(i, v, r)) m += (double)v;
        r += v == t ? 1 : 0;
      }
      m = block_sum_d(m, red);
      if (m >= target) lo_b = mid; else hi_b = mid - 1;
    }
    u_bits = lo_b;
    if (u_bits != t_bits) {
      // ties at t2 (all inside the top-k set, as t2 > t) enter in index order
      // until the mass reaches the target
      const float t2 = __uint_as_float(u_bits);
      double above = 0.0;
      int c2 = 0;
      for (int i = lo; i < hi; ++i) {
        above += p[i] > t2 ? (double)p[i] : 0.0;
        c2 += p[i] == t2 ? 1 : 0;
      }
      above = block_sum_d(above, red);
      c2 = block_sum_i(c2, red);
      int n = 0;
      double a = above;
      while (a < target && n < c2) {  // (the mass of all c2 ties reaches the target)
        a += (double)t2;
        ++n;
      }
      u_ties = n > 0 ? n : 1;
    } else {
      // the nucleus threshold is the top-k one: ties at t enter in index order
      // (within the k) until the mass reaches the target
      const float t = __uint_as_float(t_bits);
      double above = 0.0;
      for (int i = lo; i < hi; ++i) above += p[i] > t ? (double)p[i] : 0.0;
      above = block_sum_d(above, red);
      int n = 0;
      double a = above;
      while (a < target && n < ties) {
        a += (double)t;
        ++n;
      }
      u_ties = n;
    }
  }
  // final kept set: p > u or (p == u and rank among the ties at u < u_ties)
  const float uth = __uint_as_float(u_bits);
  const int ubase = tie_ranks_base(uth);
  double part = 0.0;
  {
    int r = ubase;
    for (int i = lo; i < hi; ++i) {
      const float v = p[i];
      if (v > uth || (v == uth && r < u_ties)) part += (double)v;
      r += v == uth ? 1 : 0;
    }
  }
  // running mass in index order: exclusive scan of the threads' sums
  scan[tid] = part;
  __syncthreads();
  if (tid == 0) {
    double a = 0.0;
    for (int w = 0; w < SM_THREADS; ++w) {
      const double x = scan[w];
      scan[w] = a;
      a += x;
    }
    red.d[0] = a;  // total kept mass
  }
  __syncthreads();
  const double total = red.d[0];
  const uint64_t z = splitmix64(seed + (uint64_t)(step + 1) * 0x9E3779B97F4A7C15ull);
  const double u = (double)(z >> 11) * (1.0 / 9007199254740992.0);
  const double target = u * total;
  const double base = scan[tid];
  if (base <= target && target < base + part) {
    double a = base;
    int r = ubase, pick = -1, last = -1;
    for (int i = lo; i < hi && pick < 0; ++i) {
      const float v = p[i];
      const bool keep = v > uth || (v == uth && r < u_ties);
      r += v == uth ? 1 : 0;
      if (!keep) continue;
      last = i;
      a += (double)v;
      if (a > target) pick = i;
    }
    if (pick < 0) pick = last;  // rounding left the target past the run's last kept index
    *tok_out = pick;
    *key_out = (1ull << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)pick);
  }
}

}  // namespace

cudaError_t launch_sample(const float* logits, int V, const SampleArgs& a, int step, float* scratch,
                          unsigned long long* key_out, int* tok_out, cudaStream_t st) {
  if (V < 1 || !(a.temperature > 0.0f)) return cudaErrorInvalidValue;
  sample_kernel<<<1, SM_THREADS, 0, st>>>(logits, V, a.temperature, a.top_k, a.top_p, a.seed, step, scratch, key_out,
                                          tok_out);
  return cudaGetLastError();
}

}  // namespace sfk
