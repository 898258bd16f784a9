// sfk_device.cuh -- device-side building blocks for the sm_100a decode path.
//
// * block formats and the HBM weight layout ("lane-interleaved groups")
// * mbarrier / cp.async.bulk (TMA bulk copy) / griddepcontrol (PDL) wrappers
// * the per-unit integer dot products (dp4a) for Q4_K, Q6_K and Q8_0 weights
//   against Q8_K / Q8_0 activations, following ggml's vec_dot_*_q8_K / q8_0
//   reference kernels (ggml b11379, reached from
//   src/model/engine/engine.cpp:1882-1889,1905,1967-1970,2994 of the reference)
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

namespace sfk {

// ggml_type ids (ggml.h)
enum : int { T_F32 = 0, T_F16 = 1, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14, T_Q8_K = 15 };

constexpr int QK_K = 256;
constexpr int UNIT = 128;        // columns per lane work unit
constexpr int GROUP_UNITS = 32;  // units per group (one per lane)

// ---------------------------------------------------------------------------
// HBM weight layout.  A quantized row of K columns (K % 256 == 0) is U = K/128
// units; units are grouped 32 at a time (group g has n_g = min(32, U-32g)
// units, always even).  Each group is self-contained and 16-byte aligned:
//   Q4_K : [codes: 4 chunks x n_g x 16 B][hdr: n_g/2 blocks x 16 B (d,dmin,scales)]
//   Q6_K : [codes: 6 chunks x n_g x 16 B][scales: n_g/2 x 16 B][d: n_g/2 x 2 B, pad16]
//   Q8_0 : [codes: 8 chunks x n_g x 16 B][d: n_g x 4 f16 = 8 B]
// Chunk i of unit u lives at ((i * n_g) + lane) * 16 inside the group, so the
// 32 lanes of a warp read 512 contiguous bytes per 16-byte load: conflict-free
// in shared memory and fully coalesced in HBM.  Byte count per row equals the
// GGUF row (only Q6_K groups with n_g % 16 != 0 pad their d array), so the
// streamed bytes are exactly the algorithmic bytes.
// ---------------------------------------------------------------------------
__host__ __device__ inline int wt_chunks(int t) { return t == T_Q4_K ? 4 : (t == T_Q6_K ? 6 : 8); }
__host__ __device__ inline int group_units(int K, int g) {
  const int U = K / UNIT;
  const int r = U - g * GROUP_UNITS;
  return r < GROUP_UNITS ? r : GROUP_UNITS;
}
__host__ __device__ inline int n_groups(int K) { return (K / UNIT + GROUP_UNITS - 1) / GROUP_UNITS; }
__host__ __device__ inline int group_bytes(int t, int ng) {
  switch (t) {
    case T_Q4_K: return ng * 64 + (ng / 2) * 16;
    case T_Q6_K: return ng * 96 + (ng / 2) * 16 + (((ng / 2) * 2 + 15) & ~15);
    case T_Q8_0: return ng * 128 + ng * 8;
    default: return 0;
  }
}
__host__ __device__ inline int64_t group_offset(int t, int K, int g) {
  // all groups but the last are full
  return (int64_t)g * group_bytes(t, GROUP_UNITS);
}
__host__ __device__ inline int64_t dev_row_bytes(int t, int K) {
  if (t == T_F32) return (int64_t)K * 4;
  const int G = n_groups(K);
  return group_offset(t, K, G - 1) + group_bytes(t, group_units(K, G - 1));
}

// Quantized activation ("qact") layout, one vector of K columns, same grouping:
//   [codes: 8 chunks x n_g x 16 B int8][sums: n_g x 16 B][d: n_g x 4 B]
// Q8_K: sums = the eight 16-column int16 sums of the unit (ggml bsums), d = the
//       block scale (both halves of a 256-block carry the same d).
// Q8_0: sums = the four f32 block scales of the unit (f16-rounded, as ggml
//       stores them), d unused.
constexpr int QACT_UNIT_BYTES = 128 + 16 + 4;
__host__ __device__ inline int qact_group_bytes(int ng) { return ng * QACT_UNIT_BYTES; }
// vectors are padded to 128 B so consecutive vectors stay 16-byte aligned
__host__ __device__ inline int64_t qact_bytes(int K) { return ((int64_t)(K / UNIT) * QACT_UNIT_BYTES + 127) & ~(int64_t)127; }
__host__ __device__ inline int64_t qact_group_offset(int g) { return (int64_t)g * GROUP_UNITS * QACT_UNIT_BYTES; }

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// try_wait suspends the thread until the phase completes or the time hint
// (ns) runs out, so a waiting warp does not spin through issue slots the
// working warps need.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(20000u)
      : "memory");
  return ok != 0;
}
// 1-D TMA bulk copy global -> shared, completion counted on `bar` (bytes).
// src, dst 16-byte aligned, bytes a multiple of 16.  No multicast.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Same, with an L2 cache policy (createpolicy): weight streams are read once
// per step and marked evict-first so they do not push activations, routing
// weights, KV pages and kernel code out of L2.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}
// Programmatic dependent launch: wait for the previous grid / let the next start.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ uint4 lds128(const void* p) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(smem_u32(p)));
  return v;
}
__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

// Distributed shared memory: the address of the same shared variable in
// cluster CTA `rank`, stores into it, and arrivals on its mbarriers.
__device__ __forceinline__ uint32_t dsmem_addr(const void* local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
  return r;
}
__device__ __forceinline__ void dsmem_st_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void dsmem_st_f64(uint32_t addr, double v) {
  asm volatile("st.shared::cluster.f64 [%0], %1;" ::"r"(addr), "d"(v) : "memory");
}
// Asynchronous stores into another cluster CTA's shared memory that count
// their bytes on that CTA's mbarrier (complete_tx): no fence, no arrival.
__device__ __forceinline__ void dsmem_st_async_f32(uint32_t addr, float v, uint32_t remote_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(addr),
               "r"(__float_as_uint(v)), "r"(remote_bar)
               : "memory");
}
__device__ __forceinline__ void dsmem_st_async_f64(uint32_t addr, double v, uint32_t remote_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b64 [%0], %1, [%2];" ::"r"(addr),
               "l"(__double_as_longlong(v)), "r"(remote_bar)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t remote_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote_bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, "
      "p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void fence_cluster() { asm volatile("fence.acq_rel.cluster;" ::: "memory"); }
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// error codes written to the device status word
enum : int { ERR_NONE = 0, ERR_TIMEOUT = 1, ERR_BAD_ID = 2, ERR_BAD_POS = 3, ERR_BAD_PAGE = 4 };

// Bounded mbarrier wait: ~ 2^31 cycles (~1 s at 2 GHz) then records
// ERR_TIMEOUT in *status and returns false.  The clock and the status word
// (another warp's timeout ends this wait too) are looked at only every 64th
// poll: a global load in every poll would add its latency to every wake-up.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 0) {
      if (clock64() - t0 > (1ll << 31)) {
        atomicExch(status, ERR_TIMEOUT);
        return false;
      }
      if (*(volatile int*)status == ERR_TIMEOUT) return false;
    }
  }
}


// The same bounded wait on an mbarrier that other CTAs of the cluster arrive on.
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint64_t* bar, uint32_t parity, int* status) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const long long t0 = clock64();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((i & 63) == 0) {
      if (clock64() - t0 > (1ll << 31)) {
        atomicExch(status, ERR_TIMEOUT);
        return false;
      }
      if (*(volatile int*)status == ERR_TIMEOUT) return false;
    }
  }
}

// ---------------------------------------------------------------------------
// numerics shared with the CPU oracle
// ---------------------------------------------------------------------------
// ggml nearest_int: round half to even; valid for |x| <= 4194303
__device__ __forceinline__ int nearest_int(float x) { return __float2int_rn(x); }

// exp(x): Cody & Waite argument reduction (x = n ln2 + r, ln2 split into a
// 16-bit head and a tail) and the degree-7 Taylor polynomial of e^r, scaled by
// 2^n through two exact power-of-two factors.  Each step is one round-to-
// nearest operation, so the CPU oracle (sfo_expf, -ffp-contract=off) produces
// the same bits.  Max error 1.15 ulp against exp in float64.
__device__ __forceinline__ float sfk_expf(float x) {
  if (x != x) return x;
  if (x > 88.72283935546875f) return __int_as_float(0x7f800000);
  if (x < -103.97208404541015625f) return 0.0f;
  const float t = __fmul_rn(x, 1.44269502162933349609375f);
  const int n = __float2int_rn(t);
  const float fn = (float)n;
  float r = __fsub_rn(x, __fmul_rn(fn, 0.693145751953125f));
  r = __fsub_rn(r, __fmul_rn(fn, 1.428606765330187045037746429443359375e-06f));
  float p = 1.98412701138295233249664306640625e-04f;
  p = __fadd_rn(__fmul_rn(p, r), 1.38888892251998186111450195312500e-03f);
  p = __fadd_rn(__fmul_rn(p, r), 8.33333376795053482055664062500000e-03f);
  p = __fadd_rn(__fmul_rn(p, r), 4.16666679084300994873046875000000e-02f);
  p = __fadd_rn(__fmul_rn(p, r), 1.66666671633720397949218750000000e-01f);
  p = __fadd_rn(__fmul_rn(p, r), 0.5f);
  p = __fadd_rn(__fmul_rn(p, r), 1.0f);
  p = __fadd_rn(__fmul_rn(p, r), 1.0f);
  const int n1 = n / 2, n2 = n - n / 2;
  return __fmul_rn(__fmul_rn(p, __int_as_float((n1 + 127) << 23)), __int_as_float((n2 + 127) << 23));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---------------------------------------------------------------------------
// Per-unit dot products.  `w` points at the group base in shared memory, `x`
// at the qact group base for one activation vector; `ng` units in the group;
// `lane` selects the unit.  Return the lane's fp32 partial for this unit.
// ---------------------------------------------------------------------------
// Q4_K x Q8_K  (ggml vec_dot_q4_K_q8_K): per 32-column sub-block j
//   isum += sc_j * sum(q4 * q8),  imin += m_j * (bsum_2j + bsum_2j+1)
//   result = (d_w*d_x) * isum - (dmin_w*d_x) * imin
struct WQ4K {
  uint4 c[4];
  uint32_t h0, h1, h2, h3;  // d|dmin, scales[0..3], scales[4..7], scales[8..11]
  __device__ __forceinline__ void load(const uint8_t* w, int ng, int lane) {
#pragma unroll
    for (int i = 0; i < 4; ++i) c[i] = lds128(w + ((i * ng) + lane) * 16);
    const uint4 hd = lds128(w + 4 * ng * 16 + (lane >> 1) * 16);
    h0 = hd.x; h1 = hd.y; h2 = hd.z; h3 = hd.w;
  }
};
struct XQ8 {
  uint4 c[8];
  uint4 s;  // 8 x int16 16-col sums (Q8_K) or 4 x f32 block scales (Q8_0)
  float d;
  __device__ __forceinline__ void load(const uint8_t* x, int ng, int lane) {
#pragma unroll
    for (int i = 0; i < 8; ++i) c[i] = lds128(x + ((i * ng) + lane) * 16);
    s = lds128(x + 8 * ng * 16 + lane * 16);
    d = *reinterpret_cast<const float*>(x + 8 * ng * 16 + ng * 16 + lane * 4);
  }
  // same, from a generic address (shared memory or global / L2)
  __device__ __forceinline__ void load_any(const uint8_t* x, int ng, int lane) {
#pragma unroll
    for (int i = 0; i < 8; ++i) c[i] = *reinterpret_cast<const uint4*>(x + ((i * ng) + lane) * 16);
    s = *reinterpret_cast<const uint4*>(x + 8 * ng * 16 + lane * 16);
    d = *reinterpret_cast<const float*>(x + 8 * ng * 16 + ng * 16 + lane * 4);
  }
};

__device__ __forceinline__ int dot4(const uint4 w, const uint4 x, int acc) {
  acc = dp4a((int)w.x, (int)x.x, acc);
  acc = dp4a((int)w.y, (int)x.y, acc);
  acc = dp4a((int)w.z, (int)x.z, acc);
  acc = dp4a((int)w.w, (int)x.w, acc);
  return acc;
}
__device__ __forceinline__ uint4 and4(const uint4 a, uint32_t m) { return make_uint4(a.x & m, a.y & m, a.z & m, a.w & m); }
__device__ __forceinline__ uint4 shr4_and(const uint4 a, int s, uint32_t m) {
  return make_uint4((a.x >> s) & m, (a.y >> s) & m, (a.z >> s) & m, (a.w >> s) & m);
}

// unsigned weight bytes x signed activation bytes
__device__ __forceinline__ int dot4u(const uint4 w, const uint4 x, int acc) {
  asm("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(acc) : "r"(w.x), "r"(x.x));
  asm("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(acc) : "r"(w.y), "r"(x.y));
  asm("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(acc) : "r"(w.z), "r"(x.z));
  asm("dp4a.u32.s32 %0, %1, %2, %0;" : "+r"(acc) : "r"(w.w), "r"(x.w));
  return acc;
}
__device__ __forceinline__ float dot_unit_q4k(const WQ4K& w, const XQ8& x, int lane) {
  // unit parity: half h of the 256-block
  const int h = lane & 1;
  // chunks: i=0,1 -> qs chunk c=2h bytes [0..31]; i=2,3 -> chunk 2h+1.  High
  // nibbles stay in place (16 x the code) and the sum is shifted back: it is
  // a multiple of 16, so the shift is exact.
  int s0 = dot4u(and4(w.c[0], 0x0F0F0F0Fu), x.c[0], 0);
  s0 = dot4u(and4(w.c[1], 0x0F0F0F0Fu), x.c[1], s0);
  int s1 = dot4u(and4(w.c[0], 0xF0F0F0F0u), x.c[2], 0);
  s1 = dot4u(and4(w.c[1], 0xF0F0F0F0u), x.c[3], s1) >> 4;
  int s2 = dot4u(and4(w.c[2], 0x0F0F0F0Fu), x.c[4], 0);
  s2 = dot4u(and4(w.c[3], 0x0F0F0F0Fu), x.c[5], s2);
  int s3 = dot4u(and4(w.c[2], 0xF0F0F0F0u), x.c[6], 0);
  s3 = dot4u(and4(w.c[3], 0xF0F0F0F0u), x.c[7], s3) >> 4;
  // 6-bit scales / mins of sub-blocks 4h..4h+3 (ggml get_scale_min_k4)
  uint32_t sc, mn;
  if (h == 0) {
    sc = w.h1 & 0x3F3F3F3Fu;
    mn = w.h2 & 0x3F3F3F3Fu;
  } else {
    sc = (w.h3 & 0x0F0F0F0Fu) | ((w.h1 >> 2) & 0x30303030u);
    mn = ((w.h3 >> 4) & 0x0F0F0F0Fu) | ((w.h2 >> 2) & 0x30303030u);
  }
  const int isum = (int)(sc & 0xFF) * s0 + (int)((sc >> 8) & 0xFF) * s1 + (int)((sc >> 16) & 0xFF) * s2 +
                   (int)(sc >> 24) * s3;
  // imin = sum_j m_j * (bsum16_2j + bsum16_2j+1): one 2-way dot per
  // sub-block with m_j in both low bytes
  int imin = __dp2a_lo((int)x.s.x, (int)__byte_perm(mn, 0, 0x0000), 0);
  imin = __dp2a_lo((int)x.s.y, (int)__byte_perm(mn, 0, 0x1111), imin);
  imin = __dp2a_lo((int)x.s.z, (int)__byte_perm(mn, 0, 0x2222), imin);
  imin = __dp2a_lo((int)x.s.w, (int)__byte_perm(mn, 0, 0x3333), imin);
  const __half2 dd = *reinterpret_cast<const __half2*>(&w.h0);
  const float d = __fmul_rn(__low2float(dd), x.d);
  const float dmin = __fmul_rn(__high2float(dd), x.d);
  return __fsub_rn(__fmul_rn(d, (float)isum), __fmul_rn(dmin, (float)imin));
}

// Q6_K x Q8_K  (ggml vec_dot_q6_K_q8_K): per 16-column sub-block m of the half,
//   isum += sc_m * sum((q6 - 32) * q8) = sc_m * (sum(q6u * q8) - 32 * bsum_m)
struct WQ6K {
  uint4 c[6];
  uint2 sc;  // 8 int8 scales of this half
  float d;
  __device__ __forceinline__ void load(const uint8_t* w, int ng, int lane) {
#pragma unroll
    for (int i = 0; i < 6; ++i) c[i] = lds128(w + ((i * ng) + lane) * 16);
    sc = *reinterpret_cast<const uint2*>(w + 6 * ng * 16 + lane * 8);
    const __half hd = *reinterpret_cast<const __half*>(w + 6 * ng * 16 + (ng / 2) * 16 + (lane >> 1) * 2);
    d = __half2float(hd);
  }
};
__device__ __forceinline__ float dot_unit_q6k(const WQ6K& w, const XQ8& x) {
  int s[8];
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const uint4 A = w.c[q], B = w.c[2 + q], H = w.c[4 + q];
    const uint32_t m4 = 0x0F0F0F0Fu, m2 = 0x30303030u;
    uint4 v;
    v = make_uint4((A.x & m4) | ((H.x << 4) & m2), (A.y & m4) | ((H.y << 4) & m2), (A.z & m4) | ((H.z << 4) & m2),
                   (A.w & m4) | ((H.w << 4) & m2));
    s[0 + q] = dot4(v, x.c[0 + q], 0);
    v = make_uint4((B.x & m4) | ((H.x << 2) & m2), (B.y & m4) | ((H.y << 2) & m2), (B.z & m4) | ((H.z << 2) & m2),
                   (B.w & m4) | ((H.w << 2) & m2));
    s[2 + q] = dot4(v, x.c[2 + q], 0);
    v = make_uint4(((A.x >> 4) & m4) | (H.x & m2), ((A.y >> 4) & m4) | (H.y & m2), ((A.z >> 4) & m4) | (H.z & m2),
                   ((A.w >> 4) & m4) | (H.w & m2));
    s[4 + q] = dot4(v, x.c[4 + q], 0);
    v = make_uint4(((B.x >> 4) & m4) | ((H.x >> 2) & m2), ((B.y >> 4) & m4) | ((H.y >> 2) & m2),
                   ((B.z >> 4) & m4) | ((H.z >> 2) & m2), ((B.w >> 4) & m4) | ((H.w >> 2) & m2));
    s[6 + q] = dot4(v, x.c[6 + q], 0);
  }
  // isum = sum_m sc_m * (s_m - 32 * bsum_m); the bsum part is four 2-way
  // dots of (bsum_2j, bsum_2j+1) with (sc_2j, sc_2j+1)
  int isum = 0;
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const int scm = (int)(int8_t)((m < 4 ? w.sc.x : w.sc.y) >> (8 * (m & 3)));
    isum += scm * s[m];
  }
  int sb = __dp2a_lo((int)x.s.x, (int)w.sc.x, 0);
  sb = __dp2a_hi((int)x.s.y, (int)w.sc.x, sb);
  sb = __dp2a_lo((int)x.s.z, (int)w.sc.y, sb);
  sb = __dp2a_hi((int)x.s.w, (int)w.sc.y, sb);
  isum -= 32 * sb;
  return __fmul_rn(__fmul_rn(w.d, x.d), (float)isum);
}

// Q8_0 x Q8_0 (ggml vec_dot_q8_0_q8_0): per 32-block, sumi * (d_w * d_x)
struct WQ80 {
  uint4 c[8];
  uint2 dh;  // 4 f16 block scales
  __device__ __forceinline__ void load(const uint8_t* w, int ng, int lane) {
#pragma unroll
    for (int i = 0; i < 8; ++i) c[i] = lds128(w + ((i * ng) + lane) * 16);
    dh = *reinterpret_cast<const uint2*>(w + 8 * ng * 16 + lane * 8);
  }
};
__device__ __forceinline__ float dot_unit_q80(const WQ80& w, const XQ8& x) {
  const float xd[4] = {__uint_as_float(x.s.x), __uint_as_float(x.s.y), __uint_as_float(x.s.z),
                       __uint_as_float(x.s.w)};
  const __half2 d01 = *reinterpret_cast<const __half2*>(&w.dh.x);
  const __half2 d23 = *reinterpret_cast<const __half2*>(&w.dh.y);
  const float wd[4] = {__low2float(d01), __high2float(d01), __low2float(d23), __high2float(d23)};
  float acc = 0.0f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    int s = dot4(w.c[2 * j], x.c[2 * j], 0);
    s = dot4(w.c[2 * j + 1], x.c[2 * j + 1], s);
    acc = __fadd_rn(acc, __fmul_rn((float)s, __fmul_rn(wd[j], xd[j])));
  }
  return acc;
}

}  // namespace sfk
