// sfk_tc.cu -- tensor-core (tcgen05, kind::i8) quantized GEMM for many tokens
// at once: prefill and large batches.
//
// Y[t][r] = W[r,:] . x[t] for a Q4_K / Q6_K / Q8_0 weight matrix in the HBM
// layout and activations quantized the ggml way (Q8_K for the K-quants, Q8_0
// for Q8_0): the arithmetic of ggml's vec_dot_*_q8_K / q8_0 reached from
// src/model/engine/engine.cpp:1882-1889,1905,1967-1970 of the reference, with
// the integer sub-block dot products on the tensor cores.
//
//  * A operand (weights): one CTA takes 128 rows (the 128 TMEM lanes); for each
//    256-column block its threads unpack their row's codes into shared memory
//    as signed bytes (Q4_K q in 0..15, Q6_K q - 32, Q8_0 q), in the canonical
//    K-major no-swizzle layout (8-row x 16-byte core matrices, the two 16-byte
//    halves of a 32-column chunk 128 bytes apart, row groups 256 bytes apart).
//  * B operand (activations): the codes of 64 tokens, written by tc_quant in
//    the same core-matrix layout, so a (token tile, 256-block) slab is one
//    contiguous 16 KB bulk copy.
//  * One MMA (M=128, K=32) per scale sub-block writes that sub-block's exact
//    int32 dot products into its own TMEM columns (Q6_K's 16-column
//    sub-blocks use two MMAs on half-masked copies of the chunk).
//  * The epilogue reads the sub-block sums with tcgen05.ld and applies the
//    ggml scale arithmetic: Q4_K d*dx*sum_j sc_j*D_j - dmin*dx*sum_j m_j*bsums,
//    Q6_K d*dx*sum_m sc_m*D_m, Q8_0 sum_j (d_j*dx_j)*D_j, accumulated in fp32.
// The integer parts are exact; only the fp32 order of adding blocks differs
// from the decode kernels.  Every wait is bounded; the TMEM columns are freed
// on every exit path.
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "sfk_act.cuh"
#include "sfk_device.cuh"
#include "sfk_kernels.cuh"
#include "sfk_tc.cuh"

namespace sfk {
namespace {

constexpr int TC_M = 128;       // weight rows per CTA
constexpr int TC_THREADS = 128; // one warpgroup: thread r owns row r (TMEM lane r)

// ---- tcgen05 wrappers --------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// D[tmem] = A x B (accumulate = 0) or D += A x B, s8 x s8 -> s32
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on `bar` once every MMA this thread issued has completed
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, int (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// shared-memory matrix descriptor, K-major, no swizzle: start, leading byte
// offset (between the two 16-byte K halves of a core matrix pair), stride byte
// offset (between 8-row core matrix groups), descriptor version 1
__device__ __forceinline__ uint64_t smem_desc(const void* p, uint32_t lbo, uint32_t sbo) {
  uint64_t d = (uint64_t)((smem_u32(p) >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}
// instruction descriptor, kind::i8: D s32, A s8, B s8, both K-major, M x N
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ bool mbar_wait_tc(uint64_t* bar, uint32_t parity, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 0 && clock64() - t0 > (1ll << 31)) {
      atomicExch(status, ERR_TIMEOUT);
      return false;
    }
  }
}

// ---- the 256-column block of one weight row, back in GGUF byte order ---------
// (the inverse of the HBM layout's lane-interleaved groups, sfk_synth.cu)
__device__ __forceinline__ void load16(uint8_t* dst, const uint8_t* src) {
  *reinterpret_cast<uint4*>(dst) = __ldg(reinterpret_cast<const uint4*>(src));
}
__device__ void gguf_block(int type, const uint8_t* row, int K, int b, uint8_t* out) {
  const int u0 = 2 * b;
  const int g = u0 / GROUP_UNITS, l0 = u0 % GROUP_UNITS, ng = group_units(K, g);
  const uint8_t* base = row + group_offset(type, K, g);
  if (type == T_Q4_K) {  // d | dmin | scales[12] | qs[128]
    load16(out, base + 4 * ng * 16 + (l0 >> 1) * 16);
    for (int h = 0; h < 2; ++h)
      for (int i = 0; i < 4; ++i) load16(out + 16 + 64 * h + 16 * i, base + (i * ng + l0 + h) * 16);
  } else if (type == T_Q6_K) {  // ql[128] | qh[64] | scales[16] | d
    for (int h = 0; h < 2; ++h) {
      for (int i = 0; i < 4; ++i) load16(out + 64 * h + 16 * i, base + (i * ng + l0 + h) * 16);
      for (int i = 4; i < 6; ++i) load16(out + 128 + 32 * h + 16 * (i - 4), base + (i * ng + l0 + h) * 16);
      *reinterpret_cast<uint2*>(out + 192 + 8 * h) = __ldg(reinterpret_cast<const uint2*>(base + 6 * ng * 16 + (l0 + h) * 8));
    }
    const uint16_t dv = __ldg(reinterpret_cast<const unsigned short*>(base + 6 * ng * 16 + (ng / 2) * 16 + (l0 >> 1) * 2));
    out[208] = (uint8_t)(dv & 0xFF);
    out[209] = (uint8_t)(dv >> 8);
  }
}

__device__ __forceinline__ float half_bits(const uint8_t* p) {
  return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}

// ggml get_scale_min_k4: 6-bit scale and min of Q4_K sub-block j
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t* q, int* sc, int* m) {
  if (j < 4) {
    *sc = q[j] & 63;
    *m = q[j + 4] & 63;
  } else {
    *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
    *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

// Row scales of one block (per sub-block), in shared memory per row:
//   Q4_K: f[0] = d, f[1] = dmin, i8 sc[8], m[8]
//   Q6_K: f[0] = d, i8 sc[16]
//   Q8_0: f[0..7] = d_j
struct RowScales {
  float f[8];
  int8_t s[16];
  uint8_t m[8];
};

// Q8_0 rows go straight from the HBM layout into the A tile: unit h of the
// block holds 32-column blocks 4h..4h+3, chunk i of a unit is the 16-byte
// half (i & 1) of block 4h + i / 2, and the unit's four f16 scales follow.
__device__ void unpack_row_q80(const uint8_t* row, int K, int b, int r, uint8_t* A, RowScales* rs) {
  const int u0 = 2 * b;
  const int g = u0 / GROUP_UNITS, l0 = u0 % GROUP_UNITS, ng = group_units(K, g);
  const uint8_t* base = row + group_offset(T_Q8_0, K, g);
  uint8_t* rowbase = A + (r >> 3) * 256 + (r & 7) * 16;
  for (int h = 0; h < 2; ++h) {
    const int lu = l0 + h;
    for (int i = 0; i < 8; ++i)
      *reinterpret_cast<uint4*>(rowbase + (4 * h + i / 2) * 4096 + (i & 1) * 128) =
          __ldg(reinterpret_cast<const uint4*>(base + (i * ng + lu) * 16));
    const uint2 dh = __ldg(reinterpret_cast<const uint2*>(base + 8 * ng * 16 + lu * 8));
    rs->f[4 * h + 0] = __half2float(__ushort_as_half((unsigned short)(dh.x & 0xFFFF)));
    rs->f[4 * h + 1] = __half2float(__ushort_as_half((unsigned short)(dh.x >> 16)));
    rs->f[4 * h + 2] = __half2float(__ushort_as_half((unsigned short)(dh.y & 0xFFFF)));
    rs->f[4 * h + 3] = __half2float(__ushort_as_half((unsigned short)(dh.y >> 16)));
  }
}

// unpack one row's Q4_K / Q6_K block (GGUF bytes in `blk`) into the A tile
// (chunk-major core-matrix layout) and its scales
__device__ void unpack_row(int type, const uint8_t* blk, int r, uint8_t* A, RowScales* rs) {
  uint8_t* rowbase = A + (r >> 3) * 256 + (r & 7) * 16;  // + chunk * 4096 (Q6_K: masked chunk * 4096) + half * 128
  if (type == T_Q4_K) {
    rs->f[0] = half_bits(blk);
    rs->f[1] = half_bits(blk + 2);
    for (int j = 0; j < 8; ++j) {
      int sc, m;
      scale_min_k4(j, blk + 4, &sc, &m);
      rs->s[j] = (int8_t)sc;
      rs->m[j] = (uint8_t)m;
    }
    const uint8_t* qs = blk + 16;
    // sub-block j = 2c (low nibbles of qs chunk c) and 2c + 1 (high nibbles)
    for (int c = 0; c < 4; ++c)
      for (int hi = 0; hi < 2; ++hi) {
        const int j = 2 * c + hi;
        for (int kh = 0; kh < 2; ++kh) {
          uint32_t w[4];
          for (int q = 0; q < 4; ++q) {
            const uint32_t v = *reinterpret_cast<const uint32_t*>(qs + 32 * c + 16 * kh + 4 * q);
            w[q] = hi ? ((v >> 4) & 0x0F0F0F0Fu) : (v & 0x0F0F0F0Fu);
          }
          *reinterpret_cast<uint4*>(rowbase + j * 4096 + kh * 128) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
  } else if (type == T_Q6_K) {
    rs->f[0] = half_bits(blk + 208);
    for (int m = 0; m < 16; ++m) rs->s[m] = (int8_t)blk[192 + m];
    const uint8_t* ql = blk;
    const uint8_t* qh = blk + 128;
    // ggml dequantize_row_q6_K: two halves of 128; in half n, l in 0..31:
    // y[l] = q1, y[l+32] = q2, y[l+64] = q3, y[l+96] = q4 (each q - 32)
    __align__(16) uint8_t codes[256];
    for (int n = 0; n < 2; ++n)
      for (int l = 0; l < 32; ++l) {
        const uint8_t a = ql[64 * n + l], b = ql[64 * n + l + 32], h = qh[32 * n + l];
        codes[128 * n + l] = (uint8_t)(int8_t)(((a & 0xF) | ((h & 3) << 4)) - 32);
        codes[128 * n + l + 32] = (uint8_t)(int8_t)(((b & 0xF) | (((h >> 2) & 3) << 4)) - 32);
        codes[128 * n + l + 64] = (uint8_t)(int8_t)(((a >> 4) | (((h >> 4) & 3) << 4)) - 32);
        codes[128 * n + l + 96] = (uint8_t)(int8_t)(((b >> 4) | (((h >> 6) & 3) << 4)) - 32);
      }
    // 16-column sub-block m = e / 16 sits in masked chunk m: its codes in the
    // K half (m & 1) of 32-column chunk m / 2, zeros in the other half
    const uint4 z = make_uint4(0, 0, 0, 0);
    for (int m = 0; m < 16; ++m) {
      const uint4 v = *reinterpret_cast<const uint4*>(codes + 16 * m);
      *reinterpret_cast<uint4*>(rowbase + m * 4096 + (m & 1) * 128) = v;
      *reinterpret_cast<uint4*>(rowbase + m * 4096 + ((m & 1) ^ 1) * 128) = z;
    }
  }
}

__device__ __forceinline__ void zero_row(int type, int r, uint8_t* A, RowScales* rs) {
  uint8_t* rowbase = A + (r >> 3) * 256 + (r & 7) * 16;
  const int nch = type == T_Q6_K ? 16 : 8;
  const uint4 z = make_uint4(0, 0, 0, 0);
  for (int c = 0; c < nch; ++c)
    for (int kh = 0; kh < 2; ++kh) *reinterpret_cast<uint4*>(rowbase + c * 4096 + kh * 128) = z;
  for (int i = 0; i < 8; ++i) rs->f[i] = 0.0f;
  for (int i = 0; i < 16; ++i) rs->s[i] = 0;
  for (int i = 0; i < 8; ++i) rs->m[i] = 0;
}

// ---- activations -------------------------------------------------------------
// Codes of token t, column k in the tile layout: tile t / 64, 32-column chunk
// k / 32, token group (t % 64) / 8, K half, token row, byte.
__device__ __forceinline__ int64_t xq_off(int t, int k, int KC) {
  const int64_t tile = t / TC_TT, tg = (t % TC_TT) >> 3;
  return ((tile * KC + k / 32) * 8 + tg) * 256 + ((k % 32) / 16) * 128 + (t & 7) * 16 + (k % 16);
}

// One warp per (token, 256-column block): ggml quantize_row_q8_K_ref (or
// quantize_row_q8_0_ref) of x[t][256 blk .. +256), codes into the tile layout,
// the block scale (Q8_K d, or the eight f16-rounded Q8_0 scales) and the
// 16-column sums (Q8_K).  Tokens n..npad-1 get zeros.
__global__ void __launch_bounds__(256) tc_quant_kernel(int act_type, const float* x, int n, int npad, int K,
                                                       int8_t* xq, float* dx, int16_t* bs) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = K / 256, KC = K / 32;
  for (int w = blockIdx.x * 8 + warp; w < npad * nb; w += gridDim.x * 8) {
    const int t = w / nb, blk = w % nb;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = t < n ? x[(int64_t)t * K + blk * 256 + lane * 8 + i] : 0.0f;
    int q[8];
    if (act_type == T_Q8_K) {
      float d;
      int s;
      q8k_block(v, lane, q, &d, &s);
      if (lane == 0) dx[(int64_t)t * nb + blk] = d;
      if ((lane & 1) == 0) bs[(int64_t)t * (K / 16) + blk * 16 + (lane >> 1)] = (int16_t)s;
    } else {
      float amax = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      const float d = __fdiv_rn(amax, 127.0f);
      const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) q[i] = (int)roundf(__fmul_rn(v[i], id));
      if ((lane & 3) == 0) dx[(int64_t)t * (K / 32) + blk * 8 + (lane >> 2)] = __half2float(__float2half_rn(d));
    }
    const int k0 = blk * 256 + lane * 8;
    const uint32_t lo = (uint32_t)(q[0] & 0xFF) | ((uint32_t)(q[1] & 0xFF) << 8) | ((uint32_t)(q[2] & 0xFF) << 16) |
                        ((uint32_t)(q[3] & 0xFF) << 24);
    const uint32_t hi = (uint32_t)(q[4] & 0xFF) | ((uint32_t)(q[5] & 0xFF) << 8) | ((uint32_t)(q[6] & 0xFF) << 16) |
                        ((uint32_t)(q[7] & 0xFF) << 24);
    *reinterpret_cast<uint2*>(xq + xq_off(t, k0, KC)) = make_uint2(lo, hi);
  }
}

// ---- the GEMM ----------------------------------------------------------------
// grid.x: 128-row weight tiles; grid.y: token tiles of N tokens (N = 64, or 32
// for Q6_K whose 16 sub-block accumulators per block need twice the columns).
template <int TYPE, int N>
__global__ void __launch_bounds__(TC_THREADS, 1) tc_gemm_kernel(TcGemmParams p) {
  constexpr int NCH = TYPE == T_Q6_K ? 16 : 8;       // accumulators (sub-blocks) per 256-block
  constexpr uint32_t NCOL = (uint32_t)(NCH * N);     // TMEM columns: 512
  static_assert(NCOL <= 512, "TMEM holds 512 columns");
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* A = smem;                                 // NCH x 4 KB
  uint8_t* B = smem + NCH * 4096;                    // 16 KB: one (64-token tile, 256-block) slab
  RowScales* rsc = reinterpret_cast<RowScales*>(B + 16384);
  float* dxs = reinterpret_cast<float*>(rsc + TC_M);        // [N] (Q8_K) or [N][8] (Q8_0)
  int16_t* bss = reinterpret_cast<int16_t*>(dxs + N * 8);  // [N][16]
  uint64_t* bars = reinterpret_cast<uint64_t*>(bss + N * 16);  // [0] B copy, [1] MMA done
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 2);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int r = tid;
  const int row = blockIdx.x * TC_M + r;
  const int tt = blockIdx.y;                 // token tile of N tokens
  const int t64 = (tt * N) / TC_TT;          // 64-token activation tile
  const int half = ((tt * N) % TC_TT) / 32;  // Q6_K: which 32 tokens of it
  const int KC = p.K / 32, nb = p.K / 256;

  if (warp == 0) {
    tmem_alloc(tslot, NCOL);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  float acc[N];
#pragma unroll
  for (int i = 0; i < N; ++i) acc[i] = 0.0f;
  const uint32_t idesc = idesc_i8(TC_M, N);
  bool ok = true;
  __align__(16) uint8_t blk[224];
  for (int b = 0; b < nb && ok; ++b) {
    // activations of this (token tile, block): one bulk copy + scales
    if (tid == 0) {
      mbar_arrive_expect_tx(&bars[0], 16384u);
      bulk_g2s(B, p.xq + ((int64_t)t64 * KC + b * 8) * 2048, 16384u, &bars[0]);
    }
    for (int i = tid; i < N; i += TC_THREADS) {
      const int t = tt * N + i;
      if (p.act_type == T_Q8_K) {
        dxs[i] = p.dx[(int64_t)t * nb + b];
      } else {
        for (int j = 0; j < 8; ++j) dxs[i * 8 + j] = p.dx[(int64_t)t * (p.K / 32) + b * 8 + j];
      }
    }
    if (p.act_type == T_Q8_K)
      for (int i = tid; i < N * 16; i += TC_THREADS)
        bss[i] = p.bs[(int64_t)(tt * N + i / 16) * (p.K / 16) + b * 16 + (i % 16)];
    // this thread's weight row: GGUF block bytes -> A codes + scales
    if (row < p.rows) {
      if (TYPE == T_Q8_0) {
        unpack_row_q80(p.w + (int64_t)row * p.rowstride, p.K, b, r, A, &rsc[r]);
      } else {
        gguf_block(TYPE, p.w + (int64_t)row * p.rowstride, p.K, b, blk);
        unpack_row(TYPE, blk, r, A, &rsc[r]);
      }
    } else {
      zero_row(TYPE, r, A, &rsc[r]);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the generic stores -> the tensor core's reads
    __syncthreads();
    ok = mbar_wait_tc(&bars[0], b & 1, p.status);
    ok = __syncthreads_and(ok) != 0;  // every thread leaves together
    tc_fence_after();
    if (ok && tid == 0) {
      // one K = 32 MMA per accumulator: sub-block c's dots -> columns [c*N, c*N + N)
#pragma unroll 1
      for (int c = 0; c < NCH; ++c) {
        const int chunk = TYPE == T_Q6_K ? (c >> 1) : c;  // the 32-column chunk of the activations
        const uint64_t ad = smem_desc(A + c * 4096, 128, 256);
        const uint64_t bd = smem_desc(B + chunk * 2048 + half * 1024, 128, 256);
        mma_i8(tmem + (uint32_t)(c * N), ad, bd, idesc, 0u);
      }
      mma_commit(&bars[1]);
    }
    if (ok) ok = mbar_wait_tc(&bars[1], b & 1, p.status);
    ok = __syncthreads_and(ok) != 0;
    tc_fence_after();
    if (ok) {
      // epilogue: the sub-block sums of row r (TMEM lane r) for 8 tokens at a time
      const RowScales& s = rsc[r];
      const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll
      for (int t0 = 0; t0 < N; t0 += 8) {
        int isum[8], D[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) isum[i] = 0;
#pragma unroll 1
        for (int c = 0; c < NCH; ++c) {
          tmem_ld8(lane_base + (uint32_t)(c * N + t0), D);
          tmem_wait_ld();
          if (TYPE == T_Q8_0) {  // ggml vec_dot_q8_0_q8_0: each 32-block added in order
#pragma unroll
            for (int i = 0; i < 8; ++i)
              acc[t0 + i] = __fadd_rn(acc[t0 + i], __fmul_rn((float)D[i], __fmul_rn(s.f[c], dxs[(t0 + i) * 8 + c])));
          } else {
            const int sc = s.s[c];
#pragma unroll
            for (int i = 0; i < 8; ++i) isum[i] += sc * D[i];
          }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int t = t0 + i;
          float v = 0.0f;
          if (TYPE == T_Q4_K) {
            int imin = 0;
            for (int j = 0; j < 8; ++j) imin += (int)s.m[j] * ((int)bss[t * 16 + 2 * j] + (int)bss[t * 16 + 2 * j + 1]);
            const float d = __fmul_rn(s.f[0], dxs[t]), dmin = __fmul_rn(s.f[1], dxs[t]);
            v = __fsub_rn(__fmul_rn(d, (float)isum[i]), __fmul_rn(dmin, (float)imin));
          } else if (TYPE == T_Q6_K) {
            v = __fmul_rn(__fmul_rn(s.f[0], dxs[t]), (float)isum[i]);
          }
          if (TYPE != T_Q8_0) acc[t] = __fadd_rn(acc[t], v);
        }
      }
    }
    tc_fence_before();
    __syncthreads();  // A, B, the scales and TMEM are rewritten by the next block
  }
  if (ok && row < p.rows) {
#pragma unroll
    for (int i = 0; i < N; ++i) {
      const int t = tt * N + i;
      if (t < p.n) p.y[(int64_t)t * p.ldy + row] = acc[i];
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, NCOL);
}

template <int TYPE, int N>
cudaError_t launch_gemm_t(const TcGemmParams& p, cudaStream_t st) {
  constexpr int NCH = TYPE == T_Q6_K ? 16 : 8;
  const size_t smem = (size_t)NCH * 4096 + 16384 + sizeof(RowScales) * TC_M + (size_t)N * 8 * 4 + (size_t)N * 16 * 2 +
                      2 * 8 + 16;
  auto kern = tc_gemm_kernel<TYPE, N>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int tiles = (p.npad + N - 1) / N;
  kern<<<dim3((unsigned)((p.rows + TC_M - 1) / TC_M), (unsigned)tiles), TC_THREADS, smem, st>>>(p);
  return cudaGetLastError();
}

}  // namespace

size_t tc_act_bytes(int act_type, int n, int K, size_t* off_dx, size_t* off_bs) {
  const int npad = (n + TC_TT - 1) / TC_TT * TC_TT;
  const size_t codes = (size_t)npad * K;
  const size_t dxn = act_type == T_Q8_K ? (size_t)npad * (K / 256) : (size_t)npad * (K / 32);
  const size_t a = (codes + 255) & ~(size_t)255;
  const size_t b = (a + dxn * 4 + 255) & ~(size_t)255;
  if (off_dx) *off_dx = a;
  if (off_bs) *off_bs = b;
  return b + (size_t)npad * (K / 16) * 2;
}

cudaError_t launch_tc_quant(int act_type, const float* x, int n, int K, uint8_t* buf, cudaStream_t st) {
  size_t odx = 0, obs = 0;
  tc_act_bytes(act_type, n, K, &odx, &obs);
  const int npad = (n + TC_TT - 1) / TC_TT * TC_TT;
  const int items = npad * (K / 256);
  tc_quant_kernel<<<(items + 7) / 8 < 4096 ? (items + 7) / 8 : 4096, 256, 0, st>>>(
      act_type, x, n, npad, K, reinterpret_cast<int8_t*>(buf), reinterpret_cast<float*>(buf + odx),
      reinterpret_cast<int16_t*>(buf + obs));
  return cudaGetLastError();
}

cudaError_t launch_tc_gemm(const TcGemmParams& p, cudaStream_t st) {
  switch (p.wtype) {
    case T_Q4_K: return launch_gemm_t<T_Q4_K, 64>(p, st);
    case T_Q6_K: return launch_gemm_t<T_Q6_K, 32>(p, st);
    case T_Q8_0: return launch_gemm_t<T_Q8_0, 64>(p, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace sfk
