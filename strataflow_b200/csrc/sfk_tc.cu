// sfk_tc.cu -- tensor-core (tcgen05, kind::i8) quantized GEMM for many
// activation rows at once: prompt prefill, and the routed pairs of a prefill
// chunk grouped by expert.
//
// Y[i][r] = W[r,:] . x[i] for a Q4_K / Q6_K / Q8_0 weight matrix in the HBM
// layout and activations quantized the ggml way (Q8_K for the K-quants, Q8_0
// for Q8_0): the arithmetic of ggml's vec_dot_*_q8_K / q8_0 reached from
// src/model/engine/engine.cpp:1882-1889,1905,1967-1970 of the reference, with
// the integer dot products on the tensor cores.
//
//  * A operand (weights): one CTA takes 128 rows (the 128 TMEM lanes); for each
//    256-column block its thread r unpacks row r's codes into shared memory as
//    signed bytes in the canonical K-major no-swizzle layout (8-row x 16-byte
//    core matrices, the two 16-byte halves of a 32-column chunk 128 bytes
//    apart, row groups 256 bytes apart).  The raw bytes of the next block are
//    loaded into registers while the current block is on the tensor core.
//  * B operand (activations): a (64-row tile, 256-column block) slab -- codes
//    in the same core-matrix layout followed by the block's scales -- is one
//    contiguous bulk copy; two slab buffers, the next copy in flight.
//  * Q4_K: the 6-bit sub-block scale sc_j is split into two 3-bit digits,
//    sc_j = 8 h_j + l_j, and the A tile holds h_j q and l_j q (each <= 105, a
//    signed byte).  Two K = 256 accumulations then give sum_j sc_j D_j =
//    8 D_hi + D_lo exactly: two TMEM accumulators per block instead of eight.
//    The min term sum_j m_j S_j is two more K = 32 MMAs: a tile holding the
//    row's eight mins against the activation's 32-column code sums split as
//    S_j = 128 hi_j + lo_j.  Two threads per row (256 threads), each
//    unpacking half the sub-blocks and finishing half the tokens.
//    Q6_K keeps one accumulator per 16-column sub-block (two MMAs per
//    32-column chunk on half-masked copies), Q8_0 one per 32-column block (its
//    scales are f16 per block on both sides).
//  * The epilogue reads the accumulators with tcgen05.ld and applies ggml's
//    scale arithmetic block by block, summing the blocks in order in fp32:
//    Q4_K d*dx*sum_j sc_j D_j - dmin*dx*sum_j m_j S_j, Q6_K d*dx*sum_m sc_m D_m,
//    Q8_0 sum_j (d_j*dx_j)*D_j.  The integer parts are exact.
// Every wait is bounded; on a timeout the CTA records ERR_TIMEOUT, waits
// (bounded) for its copies and MMAs in flight, frees its TMEM and returns.
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "sfk_act.cuh"
#include "sfk_device.cuh"
#include "sfk_kernels.cuh"
#include "sfk_tc.cuh"

namespace sfk {
namespace {

constexpr int TC_M = 128;        // weight rows per CTA
constexpr int TC_THREADS = 128;  // one warpgroup: thread r owns row r (TMEM lane r)

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
// TMEM loads and their wait: the destination registers of tcgen05.ld are
// written asynchronously, and an arithmetic use of them does not depend on a
// separate wait statement, so the compiler could move the use above it.  The
// helpers below either issue the loads and the wait in one asm statement, or
// make the wait take the loaded registers as operands.
// Two 16-column loads, then the wait.
__device__ __forceinline__ void tmem_ld16x2(uint32_t a0, uint32_t a1, int (&v0)[16], int (&v1)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%32];\n"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, "
      "[%33];\n"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(v0[0]), "=r"(v0[1]), "=r"(v0[2]), "=r"(v0[3]), "=r"(v0[4]), "=r"(v0[5]), "=r"(v0[6]), "=r"(v0[7]),
        "=r"(v0[8]), "=r"(v0[9]), "=r"(v0[10]), "=r"(v0[11]), "=r"(v0[12]), "=r"(v0[13]), "=r"(v0[14]), "=r"(v0[15]),
        "=r"(v1[0]), "=r"(v1[1]), "=r"(v1[2]), "=r"(v1[3]), "=r"(v1[4]), "=r"(v1[5]), "=r"(v1[6]), "=r"(v1[7]),
        "=r"(v1[8]), "=r"(v1[9]), "=r"(v1[10]), "=r"(v1[11]), "=r"(v1[12]), "=r"(v1[13]), "=r"(v1[14]), "=r"(v1[15])
      : "r"(a0), "r"(a1)
      : "memory");
}
// Four 8-column loads without the wait; tmem_wait8x4 (which takes the
// same registers as operands, so their uses cannot move above it) completes
// them.  Lets the next group's loads overlap this group's arithmetic.
__device__ __forceinline__ void tmem_issue8x4(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, int (&v0)[8],
                                              int (&v1)[8], int (&v2)[8], int (&v3)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%32];\n"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%8,%9,%10,%11,%12,%13,%14,%15}, [%33];\n"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%16,%17,%18,%19,%20,%21,%22,%23}, [%34];\n"
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%24,%25,%26,%27,%28,%29,%30,%31}, [%35];\n"
      : "=r"(v0[0]), "=r"(v0[1]), "=r"(v0[2]), "=r"(v0[3]), "=r"(v0[4]), "=r"(v0[5]), "=r"(v0[6]), "=r"(v0[7]),
        "=r"(v1[0]), "=r"(v1[1]), "=r"(v1[2]), "=r"(v1[3]), "=r"(v1[4]), "=r"(v1[5]), "=r"(v1[6]), "=r"(v1[7]),
        "=r"(v2[0]), "=r"(v2[1]), "=r"(v2[2]), "=r"(v2[3]), "=r"(v2[4]), "=r"(v2[5]), "=r"(v2[6]), "=r"(v2[7]),
        "=r"(v3[0]), "=r"(v3[1]), "=r"(v3[2]), "=r"(v3[3]), "=r"(v3[4]), "=r"(v3[5]), "=r"(v3[6]), "=r"(v3[7])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3)
      : "memory");
}
__device__ __forceinline__ void tmem_wait8x4(int (&v0)[8], int (&v1)[8], int (&v2)[8], int (&v3)[8]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n"
               : "+r"(v0[0]), "+r"(v0[1]), "+r"(v0[2]), "+r"(v0[3]), "+r"(v0[4]), "+r"(v0[5]), "+r"(v0[6]),
                 "+r"(v0[7]), "+r"(v1[0]), "+r"(v1[1]), "+r"(v1[2]), "+r"(v1[3]), "+r"(v1[4]), "+r"(v1[5]),
                 "+r"(v1[6]), "+r"(v1[7]), "+r"(v2[0]), "+r"(v2[1]), "+r"(v2[2]), "+r"(v2[3]), "+r"(v2[4]),
                 "+r"(v2[5]), "+r"(v2[6]), "+r"(v2[7]), "+r"(v3[0]), "+r"(v3[1]), "+r"(v3[2]), "+r"(v3[3]),
                 "+r"(v3[4]), "+r"(v3[5]), "+r"(v3[6]), "+r"(v3[7])
               :
               : "memory");
}
// One 16-column load, then the wait.
__device__ __forceinline__ void tmem_ld16w(uint32_t taddr, int (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      "tcgen05.wait::ld.sync.aligned;\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}

// A compiler-level use of 32 values: the loads producing them are complete
// before whatever follows is issued.
__device__ __forceinline__ void use32(const float (&v)[32]) {
  asm volatile(
      "" ::"f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]),
      "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]), "f"(v[16]), "f"(v[17]),
      "f"(v[18]), "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]), "f"(v[24]), "f"(v[25]), "f"(v[26]),
      "f"(v[27]), "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
      : "memory");
}

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

__device__ __forceinline__ uint4 ldg16(const uint8_t* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ float half_lo(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w & 0xFFFF))); }
__device__ __forceinline__ float half_hi(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w >> 16))); }
__device__ __forceinline__ uint32_t byte_of(const uint4& v, int i) {
  const uint32_t w = i < 4 ? v.x : (i < 8 ? v.y : (i < 12 ? v.z : v.w));
  return (w >> (8 * (i & 3))) & 0xFF;
}
__device__ __forceinline__ void sts16(uint8_t* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  *reinterpret_cast<uint4*>(p) = make_uint4(a, b, c, d);
}

// ---- one 256-column block of a weight row: raw bytes (registers) ------------
// The HBM layout keeps a row as lane-interleaved groups of 32 units of 128
// columns (sfk_synth.cu); block b is units 2b and 2b + 1.
struct BlockAddr {
  const uint8_t* base;
  int ng, l0;
};
__device__ __forceinline__ BlockAddr block_addr(int type, const uint8_t* row, int K, int b) {
  const int u0 = 2 * b;
  const int g = u0 / GROUP_UNITS;
  BlockAddr a;
  a.l0 = u0 % GROUP_UNITS;
  a.ng = group_units(K, g);
  a.base = row + group_offset(type, K, g);
  return a;
}

template <int TYPE>
struct RawBlock;

// Q4_K, one half of the block for one of the row's two threads: the header
// (d, dmin, 12 scale bytes) and the 128-column unit h of qs (qs bytes
// 64 h + 16 i .. + 15 in q[i]).
struct RawQ4Half {
  uint4 hdr, q[4];
  __device__ __forceinline__ void load(const uint8_t* row, int K, int b, int h) {
    const BlockAddr a = block_addr(T_Q4_K, row, K, b);
    hdr = ldg16(a.base + 4 * a.ng * 16 + (a.l0 >> 1) * 16);
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = ldg16(a.base + (i * a.ng + a.l0 + h) * 16);
  }
};
// Q6_K: ql[128] (8 x 16), qh[64] (4 x 16), scales[16], d
template <>
struct RawBlock<T_Q6_K> {
  uint4 ql[8], qh[4];
  uint2 sc[2];
  uint32_t d;
  __device__ __forceinline__ void load(const uint8_t* row, int K, int b) {
    const BlockAddr a = block_addr(T_Q6_K, row, K, b);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int i = 0; i < 4; ++i) ql[h * 4 + i] = ldg16(a.base + (i * a.ng + a.l0 + h) * 16);
#pragma unroll
      for (int i = 4; i < 6; ++i) qh[h * 2 + i - 4] = ldg16(a.base + (i * a.ng + a.l0 + h) * 16);
      sc[h] = __ldg(reinterpret_cast<const uint2*>(a.base + 6 * a.ng * 16 + (a.l0 + h) * 8));
    }
    d = __ldg(reinterpret_cast<const unsigned short*>(a.base + 6 * a.ng * 16 + (a.ng / 2) * 16 + (a.l0 >> 1) * 2));
  }
};
// Q8_0: the block's two 128-column units: chunk i of unit h is the 16-byte
// half (i & 1) of 32-column block 4h + i / 2; four f16 scales per unit
template <>
struct RawBlock<T_Q8_0> {
  uint4 q[16];
  uint2 sc[2];
  __device__ __forceinline__ void load(const uint8_t* row, int K, int b) {
    const BlockAddr a = block_addr(T_Q8_0, row, K, b);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int i = 0; i < 8; ++i) q[h * 8 + i] = ldg16(a.base + (i * a.ng + a.l0 + h) * 16);
      sc[h] = __ldg(reinterpret_cast<const uint2*>(a.base + 8 * a.ng * 16 + (a.l0 + h) * 8));
    }
  }
};

// Row scales kept in the unpacking thread's registers for its epilogue.
template <int TYPE>
struct RowScales;
template <>
struct RowScales<T_Q6_K> {
  float d;
  uint2 sc0, sc1;  // the 16 int8 sub-block scales
};
template <>
struct RowScales<T_Q8_0> {
  float d[8];
};

// ---- unpack: raw block -> A tile row + row scales ---------------------------
// A row r lives at (r >> 3) * 256 + (r & 7) * 16 within each 4 KB chunk.
// Q4_K half h of row r: sub-blocks 4h .. 4h + 3 into the A_hi / A_lo tiles
// (sub-block j = 2c + hi holds the low (hi = 0) or high nibbles of qs chunk c,
// its K half kh in q[2 (c - 2h) + kh]); the header's d and dmin out; half 0
// also writes the row's mins into K half 0 of the min tile (columns 0..7).
__device__ __forceinline__ void unpack_q4k_half(const RawQ4Half& raw, int h, uint8_t* Arow, uint8_t* Amrow,
                                                float* d, float* dmin) {
  *d = half_lo(raw.hdr.x);
  *dmin = half_hi(raw.hdr.x);
  // ggml get_scale_min_k4 over the 12 scale bytes (header bytes 4..15)
  uint32_t sb[12];
#pragma unroll
  for (int i = 0; i < 12; ++i) sb[i] = byte_of(raw.hdr, 4 + i);
  uint32_t sc[8], mn[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (j < 4) {
      sc[j] = sb[j] & 63;
      mn[j] = sb[j + 4] & 63;
    } else {
      sc[j] = (sb[j + 4] & 0xF) | ((sb[j - 4] >> 6) << 4);
      mn[j] = (sb[j + 4] >> 4) | ((sb[j] >> 6) << 4);
    }
  }
  if (h == 0)
    sts16(Amrow, mn[0] | (mn[1] << 8) | (mn[2] << 16) | (mn[3] << 24), mn[4] | (mn[5] << 8) | (mn[6] << 16) | (mn[7] << 24),
          0u, 0u);
#pragma unroll
  for (int jj = 0; jj < 4; ++jj) {
    const int j = 4 * h + jj;
    const uint32_t sh = sc[j] >> 3, sl = sc[j] & 7;
#pragma unroll
    for (int kh = 0; kh < 2; ++kh) {
      const uint4 v = raw.q[2 * (jj >> 1) + kh];
      const int s = (jj & 1) ? 4 : 0;
      const uint32_t c0 = (v.x >> s) & 0x0F0F0F0Fu, c1 = (v.y >> s) & 0x0F0F0F0Fu;
      const uint32_t c2 = (v.z >> s) & 0x0F0F0F0Fu, c3 = (v.w >> s) & 0x0F0F0F0Fu;
      // bytes <= 15 * 7: the products stay inside their bytes
      sts16(Arow + j * 4096 + kh * 128, c0 * sh, c1 * sh, c2 * sh, c3 * sh);
      sts16(Arow + 32768 + j * 4096 + kh * 128, c0 * sl, c1 * sl, c2 * sl, c3 * sl);
    }
  }
}

// Q6_K codes q - 32 as signed bytes, four at a time: q = low nibble | (2 high
// bits << 4) in 0..63, and (q + 0x60) ^ 0x80 is q - 32 in two's complement
// without carries between bytes.
__device__ __forceinline__ uint32_t q6_word(uint32_t lo4, uint32_t hi2) {
  return (((lo4 & 0x0F0F0F0Fu) | (hi2 & 0x30303030u)) + 0x60606060u) ^ 0x80808080u;
}
__device__ __forceinline__ void unpack(const RawBlock<T_Q6_K>& raw, uint8_t* Arow, RowScales<T_Q6_K>& rs) {
  rs.d = half_lo(raw.d);
  rs.sc0 = raw.sc[0];
  rs.sc1 = raw.sc[1];
  // ggml dequantize_row_q6_K: in half n (128 values) with l in 0..31,
  // y[l] = ql[l] lo | qh[l] bits 0-1, y[l+32] = ql[l+32] lo | bits 2-3,
  // y[l+64] = ql[l] hi | bits 4-5, y[l+96] = ql[l+32] hi | bits 6-7.
  // 16-column sub-block m = 8n + 2 part + (l >= 16) goes to masked chunk m,
  // K half m & 1 (the other half is zero, written once).
#pragma unroll
  for (int n = 0; n < 2; ++n)
#pragma unroll
    for (int hl = 0; hl < 2; ++hl) {
      const uint4 L = raw.ql[4 * n + hl], L2 = raw.ql[4 * n + 2 + hl], H = raw.qh[2 * n + hl];
      const int m0 = 8 * n + hl;
      uint8_t* a = Arow + hl * 128;
      sts16(a + (m0 + 0) * 4096, q6_word(L.x, H.x << 4), q6_word(L.y, H.y << 4), q6_word(L.z, H.z << 4),
            q6_word(L.w, H.w << 4));
      sts16(a + (m0 + 2) * 4096, q6_word(L2.x, H.x << 2), q6_word(L2.y, H.y << 2), q6_word(L2.z, H.z << 2),
            q6_word(L2.w, H.w << 2));
      sts16(a + (m0 + 4) * 4096, q6_word(L.x >> 4, H.x), q6_word(L.y >> 4, H.y), q6_word(L.z >> 4, H.z),
            q6_word(L.w >> 4, H.w));
      sts16(a + (m0 + 6) * 4096, q6_word(L2.x >> 4, H.x >> 2), q6_word(L2.y >> 4, H.y >> 2),
            q6_word(L2.z >> 4, H.z >> 2), q6_word(L2.w >> 4, H.w >> 2));
    }
}

__device__ __forceinline__ void unpack(const RawBlock<T_Q8_0>& raw, uint8_t* Arow, RowScales<T_Q8_0>& rs) {
#pragma unroll
  for (int h = 0; h < 2; ++h) {
#pragma unroll
    for (int i = 0; i < 8; ++i) *reinterpret_cast<uint4*>(Arow + (4 * h + i / 2) * 4096 + (i & 1) * 128) = raw.q[h * 8 + i];
    rs.d[4 * h + 0] = half_lo(raw.sc[h].x);
    rs.d[4 * h + 1] = half_hi(raw.sc[h].x);
    rs.d[4 * h + 2] = half_lo(raw.sc[h].y);
    rs.d[4 * h + 3] = half_hi(raw.sc[h].y);
  }
}

template <int TYPE>
struct TcShape;
template <>
struct TcShape<T_Q6_K> {  // sixteen accumulators of 32 rows
  static constexpr int N = 32, A_BYTES = 65536, MINB = 1;
  static constexpr uint32_t NCOL = 512;
};
template <>
struct TcShape<T_Q8_0> {  // eight accumulators of 64 rows
  static constexpr int N = 64, A_BYTES = 32768, MINB = 1;
  static constexpr uint32_t NCOL = 512;
};

// ---- MMAs of one block ----------------------------------------------------------
// Bs: the slab's codes, already offset to this CTA's N rows of the tile.
template <int TYPE>
__device__ __forceinline__ void issue_mmas(uint32_t tmem, const uint8_t* A, const uint8_t* Bs) {
  constexpr int N = TcShape<TYPE>::N;
  constexpr uint32_t idesc = idesc_i8(TC_M, N);
  if (TYPE == T_Q6_K) {
#pragma unroll 1
    for (int m = 0; m < 16; ++m)
      mma_i8(tmem + (uint32_t)(m * N), smem_desc(A + m * 4096, 128, 256), smem_desc(Bs + (m >> 1) * 2048, 128, 256),
             idesc, 0u);
  } else {
#pragma unroll 1
    for (int c = 0; c < 8; ++c)
      mma_i8(tmem + (uint32_t)(c * N), smem_desc(A + c * 4096, 128, 256), smem_desc(Bs + c * 2048, 128, 256), idesc,
             0u);
  }
}

// ---- epilogue of one block: acc[i] += this block's dot of row r, row i ------
// tb: this warp's TMEM lane base; slab: the block's slab; i0: first
// activation row of the CTA within the tile.
__device__ __forceinline__ int sbyte(uint2 v, int i) {
  const uint32_t w = i < 4 ? v.x : v.y;
  return (int)(int8_t)((w >> (8 * (i & 3))) & 0xFF);
}
__device__ __forceinline__ void block_epilogue(const RowScales<T_Q6_K>& s, uint32_t tb, const uint8_t* slab, int i0,
                                               float (&acc)[32]) {
  const float* dxs = reinterpret_cast<const float*>(slab + TC_SLAB_DX) + i0;
#pragma unroll
  for (int t0 = 0; t0 < 32; t0 += 16) {
    int isum[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) isum[i] = 0;
#pragma unroll
    for (int m = 0; m < 16; m += 2) {
      int D0[16], D1[16];
      tmem_ld16x2(tb + (uint32_t)(m * 32 + t0), tb + (uint32_t)((m + 1) * 32 + t0), D0, D1);
      const uint2 sv = m < 8 ? s.sc0 : s.sc1;
      const int s0 = sbyte(sv, m & 7), s1 = sbyte(sv, (m + 1) & 7);
#pragma unroll
      for (int i = 0; i < 16; ++i) isum[i] += s0 * D0[i] + s1 * D1[i];
    }
#pragma unroll
    for (int i = 0; i < 16; ++i)
      acc[t0 + i] = __fadd_rn(acc[t0 + i], __fmul_rn(__fmul_rn(s.d, dxs[t0 + i]), (float)isum[i]));
  }
}

__device__ __forceinline__ void block_epilogue(const RowScales<T_Q8_0>& s, uint32_t tb, const uint8_t* slab, int i0,
                                               float (&acc)[64]) {
  const float* dxs = reinterpret_cast<const float*>(slab + TC_SLAB_DX) + i0 * 8;
  // ggml vec_dot_q8_0_q8_0: each 32-column block added in order
#pragma unroll
  for (int c = 0; c < 8; ++c) {
#pragma unroll
    for (int t0 = 0; t0 < 64; t0 += 16) {
      int D[16];
      tmem_ld16w(tb + (uint32_t)(c * 64 + t0), D);
#pragma unroll
      for (int i = 0; i < 16; ++i)
        acc[t0 + i] = __fadd_rn(acc[t0 + i], __fmul_rn((float)D[i], __fmul_rn(s.d[c], dxs[(t0 + i) * 8 + c])));
    }
  }
}

// Q6_K: the zero K half of every masked chunk of row r
__device__ __forceinline__ void zero_masked_halves(uint8_t* Arow) {
#pragma unroll
  for (int m = 0; m < 16; ++m) sts16(Arow + m * 4096 + ((m & 1) ^ 1) * 128, 0u, 0u, 0u, 0u);
}

// ---- activations -------------------------------------------------------------
// One warp per (activation row, 256-column block): ggml quantize_row_q8_K_ref
// (or quantize_row_q8_0_ref) of the block, codes into the slab's core-matrix
// layout, the scale(s), and for Q8_K the 32-column code sums (high and low
// parts, the min term's B operand).
__global__ void __launch_bounds__(256) tc_quant_kernel(int act_type, const float* x, int64_t ldx, const int* rows,
                                                       int n_src, int npad, int K, uint8_t* out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = K / 256;
  for (int w = blockIdx.x * 8 + warp; w < npad * nb; w += gridDim.x * 8) {
    const int t = w / nb, blk = w % nb;
    const int src = rows ? rows[t] : t;
    const bool valid = src >= 0 && src < n_src;
    float v[8];
    if (valid) {
      const float4* xp = reinterpret_cast<const float4*>(x + (int64_t)src * ldx + blk * 256 + lane * 8);
      const float4 a = xp[0], b = xp[1];
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.0f;
    }
    uint8_t* slab = out + ((int64_t)(t / TC_TT) * nb + blk) * TC_SLAB;
    const int tl = t % TC_TT;
    int q[8];
    if (act_type == T_Q8_K) {
      float d;
      int s16;
      q8k_block(v, lane, q, &d, &s16);
      int s = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) s += q[i];
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      if (lane == 0) reinterpret_cast<float*>(slab + TC_SLAB_DX)[tl] = d;
      // S_j = 128 hi + lo as column j of the two sum chunks (row tl, K half 0)
      const int rowoff = (tl >> 3) * 256 + (tl & 7) * 16;
      if ((lane & 3) == 0) {
        slab[TC_SLAB_SHI + rowoff + (lane >> 2)] = (uint8_t)(int8_t)(s >> 7);
        slab[TC_SLAB_SLO + rowoff + (lane >> 2)] = (uint8_t)(s & 127);
      }
      if (lane == 0) {
        *reinterpret_cast<uint2*>(slab + TC_SLAB_SHI + rowoff + 8) = make_uint2(0u, 0u);
        *reinterpret_cast<uint2*>(slab + TC_SLAB_SLO + rowoff + 8) = make_uint2(0u, 0u);
      }
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
      if ((lane & 3) == 0)
        reinterpret_cast<float*>(slab + TC_SLAB_DX)[tl * 8 + (lane >> 2)] = __half2float(__float2half_rn(d));
    }
    // columns lane*8 .. +7: chunk lane / 4, K half (lane / 2) & 1, byte (lane & 1) * 8
    *reinterpret_cast<uint2*>(slab + (lane >> 2) * 2048 + (tl >> 3) * 256 + ((lane >> 1) & 1) * 128 + (tl & 7) * 16 +
                              (lane & 1) * 8) = pack8(q);
  }
}

// ---- the GEMM ----------------------------------------------------------------
// grid.x: activation tiles x (64 / N) (the CTAs that share a weight tile run
// together); grid.y: 128-row weight tiles.
template <int TYPE>
__global__ void __launch_bounds__(TC_THREADS, TcShape<TYPE>::MINB) tc_gemm_kernel(const __grid_constant__ TcGemmParams p) {
  constexpr int N = TcShape<TYPE>::N;
  constexpr uint32_t NCOL = TcShape<TYPE>::NCOL;
  constexpr int SUB = TC_TT / N;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* A = smem;
  uint8_t* B = smem + TcShape<TYPE>::A_BYTES;                     // [2][TC_SLAB]
  uint64_t* bars = reinterpret_cast<uint64_t*>(B + 2 * TC_SLAB);  // [0..1] slab full, [2] MMAs done
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 3);

  const int t64 = blockIdx.x / SUB, sub = blockIdx.x % SUB;
  if (t64 >= p.ntile) return;
  int expert = 0;
  if (p.tile_expert) {
    expert = p.tile_expert[t64];
    if (expert < 0) return;  // uniform: the whole CTA leaves before any allocation
  }
  const int tid = threadIdx.x, warp = tid >> 5;
  const int row = blockIdx.y * TC_M + tid;
  const bool live = row < p.rows;
  const int nb = p.K / 256;
  const int nmat = p.epi == TC_EPI_SWIGLU ? 2 : 1;
  const int total = nmat * nb;
  const uint8_t* slabs = p.xq + (int64_t)t64 * nb * TC_SLAB;
  uint8_t* Arow = A + (tid >> 3) * 256 + (tid & 7) * 16;
  // rows past the matrix compute row 0 again; their results are not stored
  const int64_t woff = (int64_t)expert * p.expert_stride + (int64_t)(live ? row : 0) * p.rowstride;

  if (warp == 0) {
    tmem_alloc(tslot, NCOL);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    mbar_init(&bars[2], 1);
    fence_mbar_init();
  }
  if (TYPE == T_Q6_K) zero_masked_halves(Arow);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t tb = tmem + ((uint32_t)(warp * 32) << 16);

  if (tid == 0) {
    mbar_arrive_expect_tx(&bars[0], TC_SLAB);
    bulk_g2s(B, slabs, TC_SLAB, &bars[0]);
  }
  RawBlock<TYPE> raw;
  raw.load(p.w + woff, p.K, 0);
  float acc[N];
#pragma unroll
  for (int i = 0; i < N; ++i) acc[i] = 0.0f;
  bool ok = true;
  bool mma_pending = false;
  int g = 0;
  for (; g < total; ++g) {
    const int mat = g >= nb ? 1 : 0, b = g - mat * nb;
    if (tid == 0 && g + 1 < total) {  // the next slab into the other buffer (its last readers are done)
      mbar_arrive_expect_tx(&bars[(g + 1) & 1], TC_SLAB);
      bulk_g2s(B + ((g + 1) & 1) * TC_SLAB, slabs + (int64_t)((g + 1) % nb) * TC_SLAB, TC_SLAB, &bars[(g + 1) & 1]);
    }
    RowScales<TYPE> rs;
    unpack(raw, Arow, rs);
    if (g + 1 < total) {
      const int nm = (g + 1) >= nb ? 1 : 0;
      raw.load((nm ? p.w2 : p.w) + woff, p.K, (g + 1) - nm * nb);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the generic stores -> the tensor core's reads
    __syncthreads();
    ok = mbar_wait_tc(&bars[g & 1], (uint32_t)((g >> 1) & 1), p.status);
    ok = __syncthreads_and(ok) != 0;  // every thread leaves together
    if (!ok) break;
    tc_fence_after();
    const uint8_t* slab = B + (g & 1) * TC_SLAB;
    if (tid == 0) {
      issue_mmas<TYPE>(tmem, A, slab + sub * N * 32);
      mma_commit(&bars[2]);
    }
    mma_pending = true;
    ok = mbar_wait_tc(&bars[2], (uint32_t)(g & 1), p.status);
    ok = __syncthreads_and(ok) != 0;
    if (!ok) break;
    mma_pending = false;
    tc_fence_after();
    block_epilogue(rs, tb, slab, sub * N, acc);
    // this slab buffer's generic reads before the bulk copy that refills it
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();  // A, this slab buffer and TMEM are rewritten next
    if (b == nb - 1) {
      if (live) {
#pragma unroll
        for (int i = 0; i < N; ++i) {
          const int ir = t64 * TC_TT + sub * N + i;
          if (!p.tile_expert && ir >= p.n) continue;
          float* yp = p.y + (int64_t)ir * p.ldy + row;
          if (p.epi == TC_EPI_RESID) {
            *yp = __fadd_rn(acc[i], p.res[(int64_t)ir * p.ldres + row]);
          } else if (p.epi == TC_EPI_SWIGLU && mat == 1) {
            // h = silu(gate) * up (ggml_swiglu_split, engine.cpp:1969); this
            // thread stored the gate value here at the end of matrix 0
            const float gv = *yp;
            *yp = __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, sfk_expf(-gv))), acc[i]);
          } else {
            *yp = acc[i];
          }
        }
      }
#pragma unroll
      for (int i = 0; i < N; ++i) acc[i] = 0.0f;
    }
  }
  if (!ok && tid == 0) {
    // drain what is still in flight before the TMEM and shared memory go:
    // the MMAs of block g (when issued) and the slab copies g and g + 1
    if (mma_pending) mbar_wait_tc(&bars[2], (uint32_t)(g & 1), p.status);
    else mbar_wait_tc(&bars[g & 1], (uint32_t)((g >> 1) & 1), p.status);
    if (g + 1 < total) mbar_wait_tc(&bars[(g + 1) & 1], (uint32_t)(((g + 1) >> 1) & 1), p.status);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, NCOL);
}

// ---- Q4_K: warp-specialized pipeline ------------------------------------------
// One CTA per (64-row activation tile, 128 weight rows), 14 warps:
//   warps 0-3   unpack: thread r turns row r's next block into A_hi / A_lo and
//               the min tile, in one of two A stages;
//   warps 4-11  epilogue: two warps per TMEM lane quadrant (tokens 0-31 and
//               32-63 of the tile) apply the block's scales to the four
//               accumulators of one of two TMEM stages; they copy the
//               activation scales out of the slab first and release it;
//   warp 12     MMA issue (one thread): 18 MMAs per block, then commits that
//               free the A stage and fill the TMEM stage;
//   warp 13     activation slabs (one thread): bulk copies into three stages.
// Each hand-off is an mbarrier (full / empty per stage), so the unpack of
// block b + 2, the MMAs of block b + 1 and the epilogue of block b overlap.
// The MMAs of a block are committed once, to acc_full: the epilogue waits on
// it for the accumulators and the unpack warps for the A stage.
// TMEM stage columns: D_hi [0, 64), D_lo [64, 128), M_hi [128, 192),
// M_lo [192, 256); sum_j sc_j D_j = 8 D_hi + D_lo, sum_j m_j S_j =
// 128 M_hi + M_lo.  Every wait is bounded; a role that gives up raises the
// CTA's abort flag, the others leave at their next wait, and the copies and
// MMAs still in flight are drained before TMEM is freed.
constexpr int Q4_UNPACK_WARPS = 4, Q4_EPI_WARPS = 8;
constexpr int Q4_MMA_WARP = Q4_UNPACK_WARPS + Q4_EPI_WARPS, Q4_TMA_WARP = Q4_MMA_WARP + 1;
constexpr int Q4_THREADS = (Q4_TMA_WARP + 1) * 32;
constexpr uint32_t Q4_NCOL = 512;          // two TMEM stages of 256 columns
constexpr int Q4_ASTAGE = 65536 + 4096;    // A_hi | A_lo | min tile
constexpr int Q4_ASTAGES = 2;  // A tiles and TMEM accumulator sets
constexpr int Q4_BSTAGES = 3;  // activation slabs
constexpr int Q4_SMEM = Q4_ASTAGES * Q4_ASTAGE + Q4_BSTAGES * TC_SLAB + 16 * 8 + 16;  // + barriers, TMEM slot, abort flag

struct Q4Bars {
  uint64_t a_full[Q4_ASTAGES], b_full[Q4_BSTAGES], b_empty[Q4_BSTAGES], acc_full[Q4_ASTAGES], acc_empty[Q4_ASTAGES];
};

// bounded wait that also leaves when another role raised the abort flag
__device__ __forceinline__ bool q4_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 15) == 0) {
      if (*abort_flag) return false;
      if (clock64() - t0 > (1ll << 31)) {
        atomicExch(status, ERR_TIMEOUT);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

__global__ void __launch_bounds__(Q4_THREADS, 1) tc_gemm_q4k_kernel(const __grid_constant__ TcGemmParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* Ast = smem;                                           // [Q4_ASTAGES][Q4_ASTAGE]
  uint8_t* Bst = smem + Q4_ASTAGES * Q4_ASTAGE;                  // [Q4_BSTAGES][TC_SLAB]
  Q4Bars* bars = reinterpret_cast<Q4Bars*>(Bst + Q4_BSTAGES * TC_SLAB);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int t64 = blockIdx.x;
  if (t64 >= p.ntile) return;
  int expert = 0;
  if (p.tile_expert) {
    expert = p.tile_expert[t64];
    if (expert < 0) return;  // uniform: the whole CTA leaves before any allocation
  }
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nb = p.K / 256;
  const int nmat = p.epi == TC_EPI_SWIGLU ? 2 : 1;
  const int total = nmat * nb;
  const uint8_t* slabs = p.xq + (int64_t)t64 * nb * TC_SLAB;

  if (warp == 0) {
    tmem_alloc(tslot, Q4_NCOL);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int i = 0; i < Q4_ASTAGES; ++i) {
      mbar_init(&bars->a_full[i], Q4_UNPACK_WARPS);  // one arrival per unpack warp
      mbar_init(&bars->acc_full[i], 1);
      mbar_init(&bars->acc_empty[i], Q4_EPI_WARPS);
    }
    for (int i = 0; i < Q4_BSTAGES; ++i) {
      mbar_init(&bars->b_full[i], 1);
      mbar_init(&bars->b_empty[i], Q4_EPI_WARPS);  // one arrival per epilogue warp
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp < Q4_UNPACK_WARPS) {  // min tile columns 16..31 stay zero in both stages
    const int r = tid;
    for (int st = 0; st < Q4_ASTAGES; ++st)
      sts16(Ast + st * Q4_ASTAGE + 65536 + (r >> 3) * 256 + (r & 7) * 16 + 128, 0u, 0u, 0u, 0u);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp < Q4_UNPACK_WARPS) {
    // ---- unpack -------------------------------------------------------------
    const int r = tid;
    const int row = blockIdx.y * TC_M + r;
    const int64_t woff = (int64_t)expert * p.expert_stride + (int64_t)(row < p.rows ? row : 0) * p.rowstride;
    const int rowoff = (r >> 3) * 256 + (r & 7) * 16;
    RawQ4Half lo, hi;  // the block's two 128-column units
    lo.load(p.w + woff, p.K, 0, 0);
    hi.load(p.w + woff, p.K, 0, 1);
    for (int g = 0; g < total; ++g) {
      const int st = g % Q4_ASTAGES;
      // A stage st is free once the MMAs of block g - Q4_ASTAGES have
      // completed: the one commit per block, on acc_full, is waited on here too
      if (g >= Q4_ASTAGES &&
          !q4_wait(&bars->acc_full[st], (uint32_t)((g / Q4_ASTAGES + 1) & 1), abort_flag, p.status))
        break;
      uint8_t* A = Ast + st * Q4_ASTAGE;
      float dd, dm;
      unpack_q4k_half(lo, 0, A + rowoff, A + 65536 + rowoff, &dd, &dm);
      unpack_q4k_half(hi, 1, A + rowoff, A + 65536 + rowoff, &dd, &dm);
      // each thread orders its generic stores before the tensor core's reads
      // (proxy fence); the warp then arrives once
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->a_full[st]);
      if (g + 1 < total) {
        const int nm = (g + 1) >= nb ? 1 : 0;
        const uint8_t* w = (nm ? p.w2 : p.w) + woff;
        lo.load(w, p.K, (g + 1) - nm * nb, 0);
        hi.load(w, p.K, (g + 1) - nm * nb, 1);
      }
    }
  } else if (warp < Q4_MMA_WARP) {
    // ---- epilogue -------------------------------------------------------------
    const int ew = warp - Q4_UNPACK_WARPS;
    const int quad = warp & 3, th = ew >> 2;  // TMEM lanes 32 quad .. +31; tokens 32 th .. +31
    const int r = quad * 32 + lane;
    const int row = blockIdx.y * TC_M + r;
    const bool live = row < p.rows;
    const int64_t woff = (int64_t)expert * p.expert_stride + (int64_t)(live ? row : 0) * p.rowstride;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(32 * th);
    uint4 hdr;  // this block's header (d, dmin) for row r
    {
      const BlockAddr a = block_addr(T_Q4_K, p.w + woff, p.K, 0);
      hdr = ldg16(a.base + 4 * a.ng * 16 + (a.l0 >> 1) * 16);
    }
    float acc[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) acc[i] = 0.0f;
    for (int g = 0; g < total; ++g) {
      const int mat = g >= nb ? 1 : 0, b = g - mat * nb;
      const float rd = half_lo(hdr.x), rdmin = half_hi(hdr.x);
      if (g + 1 < total) {
        const int nm = (g + 1) >= nb ? 1 : 0;
        const BlockAddr a = block_addr(T_Q4_K, (nm ? p.w2 : p.w) + woff, p.K, (g + 1) - nm * nb);
        hdr = ldg16(a.base + 4 * a.ng * 16 + (a.l0 >> 1) * 16);
      }
      const int ts = g % Q4_ASTAGES, bs = g % Q4_BSTAGES;
      if (!q4_wait(&bars->acc_full[ts], (uint32_t)((g / Q4_ASTAGES) & 1), abort_flag, p.status)) break;
      // the slab's scales are read here too: observe its copy's completion
      if (!q4_wait(&bars->b_full[bs], (uint32_t)((g / Q4_BSTAGES) & 1), abort_flag, p.status)) break;
      // the lanes left their waits one by one: reconverge before the
      // warp-collective (.sync.aligned) TMEM loads
      __syncwarp();
      tc_fence_after();
      // the block's activation scales into registers, then the slab goes back
      // to the copy warp: each thread's reads complete (use32) and are ordered
      // before the async proxy's next write into the stage (proxy fence); the
      // warp then arrives once
      const float* dxsm = reinterpret_cast<const float*>(Bst + bs * TC_SLAB + TC_SLAB_DX) + 32 * th;
      float dxs[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) dxs[i] = dxsm[i];
      use32(dxs);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->b_empty[bs]);
      const uint32_t tb = lane_base + (uint32_t)(ts * 256);
      // ggml vec_dot_q4_K_q8_K per block: (d dx) sum_j sc_j D_j - (dmin dx) sum_j m_j S_j;
      // the loads of the next 8 tokens are in flight during this group's math
      int Dh[2][8], Dl[2][8], Mh[2][8], Ml[2][8];
      tmem_issue8x4(tb, tb + 64u, tb + 128u, tb + 192u, Dh[0], Dl[0], Mh[0], Ml[0]);
#pragma unroll
      for (int grp = 0; grp < 4; ++grp) {
        const int cb = grp & 1, t0 = grp * 8;
        tmem_wait8x4(Dh[cb], Dl[cb], Mh[cb], Ml[cb]);
        if (grp < 3) {
          const uint32_t a = tb + (uint32_t)(t0 + 8);
          tmem_issue8x4(a, a + 64u, a + 128u, a + 192u, Dh[cb ^ 1], Dl[cb ^ 1], Mh[cb ^ 1], Ml[cb ^ 1]);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int isum = Dh[cb][i] * 8 + Dl[cb][i];
          const int imin = Mh[cb][i] * 128 + Ml[cb][i];
          const float dx = dxs[t0 + i];
          const float d = __fmul_rn(rd, dx), dmn = __fmul_rn(rdmin, dx);
          acc[t0 + i] = __fadd_rn(acc[t0 + i], __fsub_rn(__fmul_rn(d, (float)isum), __fmul_rn(dmn, (float)imin)));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bars->acc_empty[ts]);
      }
      if (b == nb - 1) {
        if (live) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int ir = t64 * TC_TT + 32 * th + i;
            if (!p.tile_expert && ir >= p.n) continue;
            float* yp = p.y + (int64_t)ir * p.ldy + row;
            if (p.epi == TC_EPI_RESID) {
              *yp = __fadd_rn(acc[i], p.res[(int64_t)ir * p.ldres + row]);
            } else if (p.epi == TC_EPI_SWIGLU && mat == 1) {
              // h = silu(gate) * up (ggml_swiglu_split, engine.cpp:1969); this
              // thread stored the gate value here at the end of matrix 0
              const float gv = *yp;
              *yp = __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, sfk_expf(-gv))), acc[i]);
            } else {
              *yp = acc[i];
            }
          }
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = 0.0f;
      }
    }
  } else if (warp == Q4_MMA_WARP) {
    // ---- MMA issue ----------------------------------------------------------------
    int issued = 0;  // blocks whose MMAs were committed
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_i8(TC_M, 64);
      for (int g = 0; g < total; ++g) {
        const int as = g % Q4_ASTAGES, bs = g % Q4_BSTAGES, ts = as;
        if (!q4_wait(&bars->a_full[as], (uint32_t)((g / Q4_ASTAGES) & 1), abort_flag, p.status)) break;
        if (!q4_wait(&bars->b_full[bs], (uint32_t)((g / Q4_BSTAGES) & 1), abort_flag, p.status)) break;
        if (!q4_wait(&bars->acc_empty[ts], (uint32_t)((g / Q4_ASTAGES + 1) & 1), abort_flag, p.status)) break;
        tc_fence_after();
        // descriptors: the start field is the address >> 4, so +4096 bytes
        // (next A chunk) is +256 and +2048 (next B chunk) is +128; all
        // addresses stay below 256 KB, the field never carries
        const uint64_t da = smem_desc(Ast + as * Q4_ASTAGE, 128, 256);
        const uint64_t db = smem_desc(Bst + bs * TC_SLAB, 128, 256);
        const uint32_t d0 = tmem + (uint32_t)(ts * 256);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          mma_i8(d0, da + (uint64_t)(c * 256), db + (uint64_t)(c * 128), idesc, c > 0 ? 1u : 0u);
          mma_i8(d0 + 64u, da + (uint64_t)(2048 + c * 256), db + (uint64_t)(c * 128), idesc, c > 0 ? 1u : 0u);
        }
        mma_i8(d0 + 128u, da + (uint64_t)4096, db + (uint64_t)(TC_SLAB_SHI >> 4), idesc, 0u);
        mma_i8(d0 + 192u, da + (uint64_t)4096, db + (uint64_t)(TC_SLAB_SLO >> 4), idesc, 0u);
        mma_commit(&bars->acc_full[ts]);  // frees A stage `as` and fills TMEM stage `ts`
        issued = g + 1;
      }
      // before TMEM goes: the last committed MMAs have completed
      if (issued > 0) {
        const int g = issued - 1;
        mbar_wait_tc(&bars->acc_full[g % Q4_ASTAGES], (uint32_t)((g / Q4_ASTAGES) & 1), p.status);
      }
    }
  } else {
    // ---- activation slabs ----------------------------------------------------------
    if (lane == 0) {
      int copied = 0;
      for (int g = 0; g < total; ++g) {
        const int bs = g % Q4_BSTAGES;
        if (!q4_wait(&bars->b_empty[bs], (uint32_t)(((g / Q4_BSTAGES) + 1) & 1), abort_flag, p.status)) break;
        mbar_arrive_expect_tx(&bars->b_full[bs], TC_SLAB);
        bulk_g2s(Bst + bs * TC_SLAB, slabs + (int64_t)(g % nb) * TC_SLAB, TC_SLAB, &bars->b_full[bs]);
        copied = g + 1;
      }
      // before shared memory goes: every copy issued has landed
      for (int g = (copied > Q4_BSTAGES ? copied - Q4_BSTAGES : 0); g < copied; ++g)
        mbar_wait_tc(&bars->b_full[g % Q4_BSTAGES], (uint32_t)((g / Q4_BSTAGES) & 1), p.status);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, Q4_NCOL);
}

cudaError_t launch_gemm_q4k(const TcGemmParams& p, cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(tc_gemm_q4k_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Q4_SMEM);
  if (e != cudaSuccess) return e;
  const dim3 grid((unsigned)p.ntile, (unsigned)((p.rows + TC_M - 1) / TC_M));
  tc_gemm_q4k_kernel<<<grid, Q4_THREADS, Q4_SMEM, st>>>(p);
  return cudaGetLastError();
}

template <int TYPE>
cudaError_t launch_gemm_t(const TcGemmParams& p, cudaStream_t st) {
  constexpr int N = TcShape<TYPE>::N;
  size_t smem = (size_t)TcShape<TYPE>::A_BYTES + 2 * TC_SLAB + 3 * 8 + 16;
  // the 512-column kinds take all of an SM's TMEM: one CTA per SM
  if (TcShape<TYPE>::NCOL == 512 && smem < 120 * 1024) smem = 120 * 1024;
  auto kern = tc_gemm_kernel<TYPE>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const dim3 grid((unsigned)(p.ntile * (TC_TT / N)), (unsigned)((p.rows + TC_M - 1) / TC_M));
  kern<<<grid, TC_THREADS, smem, st>>>(p);
  return cudaGetLastError();
}

}  // namespace

size_t tc_act_bytes(int rows, int K) {
  const size_t tiles = (size_t)(rows + TC_TT - 1) / TC_TT;
  return tiles * (size_t)(K / 256) * TC_SLAB;
}

cudaError_t launch_tc_quant(int act_type, const float* x, int64_t ldx, const int* rows, int n_src, int npad, int K,
                            uint8_t* buf, cudaStream_t st) {
  if (npad % TC_TT || K % 256 || npad <= 0) return cudaErrorInvalidValue;
  const int items = npad * (K / 256);
  const int blocks = (items + 7) / 8 < 8192 ? (items + 7) / 8 : 8192;
  tc_quant_kernel<<<blocks, 256, 0, st>>>(act_type, x, ldx, rows, n_src, npad, K, buf);
  return cudaGetLastError();
}

cudaError_t launch_tc_gemm(const TcGemmParams& p, cudaStream_t st) {
  if (p.epi == TC_EPI_SWIGLU && !p.w2) return cudaErrorInvalidValue;
  if (p.K % 256 || p.rows < 1 || p.ntile < 1) return cudaErrorInvalidValue;
  switch (p.wtype) {
    case T_Q4_K: return launch_gemm_q4k(p, st);
    case T_Q6_K: return launch_gemm_t<T_Q6_K>(p, st);
    case T_Q8_0: return launch_gemm_t<T_Q8_0>(p, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace sfk
