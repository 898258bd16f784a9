// sfk_act.cuh -- warp-level activation quantizers writing the qact layout.
//
// Restates ggml's quantize_row_q8_K_ref and quantize_row_q8_0_ref (ggml b11379,
// reached by every quantized mul_mat / mul_mat_id of
// src/model/engine/engine.cpp:1882-1970,2994): the activation row is quantized
// to the weight type's dot type before the integer dot product.
#pragma once
#include "sfk_device.cuh"

namespace sfk {

// Q8_K math for one 256-column block held by a warp (8 values per lane):
// returns the lane's 8 codes, the block scale d and the lane's 16-column sum
// (lanes 2m and 2m+1 share sum m).
__device__ __forceinline__ void q8k_block(const float v[8], int lane, int q[8], float* d_out, int* bsum) {
  float ax = -1.0f, mv = 0.0f;
  int idx = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float a = fabsf(v[i]);
    if (a > ax) { ax = a; mv = v[i]; idx = 8 * lane + i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float oax = __shfl_xor_sync(0xffffffffu, ax, o);
    const float omv = __shfl_xor_sync(0xffffffffu, mv, o);
    const int oidx = __shfl_xor_sync(0xffffffffu, idx, o);
    if (oax > ax || (oax == ax && oidx < idx)) { ax = oax; mv = omv; idx = oidx; }
  }
  float d = 0.0f;
  if (ax == 0.0f) {
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = 0;
  } else {
    const float iscale = __fdiv_rn(-127.0f, mv);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int t = nearest_int(__fmul_rn(iscale, v[i]));
      q[i] = t < 127 ? t : 127;
    }
    d = __fdiv_rn(1.0f, iscale);
  }
  int s = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) s += q[i];
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  *d_out = d;
  *bsum = s;
}

__device__ __forceinline__ uint2 pack8(const int q[8]) {
  const uint32_t lo = (uint32_t)(q[0] & 0xFF) | ((uint32_t)(q[1] & 0xFF) << 8) | ((uint32_t)(q[2] & 0xFF) << 16) |
                      ((uint32_t)(q[3] & 0xFF) << 24);
  const uint32_t hi = (uint32_t)(q[4] & 0xFF) | ((uint32_t)(q[5] & 0xFF) << 8) | ((uint32_t)(q[6] & 0xFF) << 16) |
                      ((uint32_t)(q[7] & 0xFF) << 24);
  return make_uint2(lo, hi);
}

// One warp quantizes one 256-column block `blk` of a K-column vector to Q8_K
// (ggml quantize_row_q8_K_ref): amax = max |x| (first index on ties),
// max = that signed value, iscale = -127/max, q = min(127, nearest(iscale*x)),
// d = 1/iscale, bsums = 16-column sums of q.  Written in the qact layout.
__device__ __forceinline__ void qact_put_q8k(uint8_t* qa, int K, int blk, const float v[8], int lane) {
  int q[8], s;
  float d;
  q8k_block(v, lane, q, &d, &s);
  const int u = 2 * blk + (lane >> 4);
  const int g = u / GROUP_UNITS, ul = u % GROUP_UNITS, ng = group_units(K, g);
  uint8_t* gb = qa + qact_group_offset(g);
  const int m = (lane & 15) >> 1;
  *reinterpret_cast<uint2*>(gb + (m * ng + ul) * 16 + (lane & 1) * 8) = pack8(q);
  if ((lane & 1) == 0) *reinterpret_cast<int16_t*>(gb + 8 * ng * 16 + ul * 16 + m * 2) = (int16_t)s;
  if ((lane & 15) == 0) *reinterpret_cast<float*>(gb + 8 * ng * 16 + ng * 16 + ul * 4) = d;
}

// One warp quantizes 256 columns (8 Q8_0 blocks of 32) of a K-column vector:
// d = amax/127, id = d ? 1/d : 0, q = roundf(x*id), block scale stored f16.
__device__ __forceinline__ void qact_put_q80(uint8_t* qa, int K, int blk, const float v[8], int lane) {
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  const float d = __fdiv_rn(amax, 127.0f);
  const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
  int q[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) q[i] = (int)roundf(__fmul_rn(v[i], id));
  const int u = 2 * blk + (lane >> 4);
  const int g = u / GROUP_UNITS, ul = u % GROUP_UNITS, ng = group_units(K, g);
  uint8_t* gb = qa + qact_group_offset(g);
  const int m = (lane & 15) >> 1;
  const uint32_t lo = (uint32_t)(q[0] & 0xFF) | ((uint32_t)(q[1] & 0xFF) << 8) | ((uint32_t)(q[2] & 0xFF) << 16) |
                      ((uint32_t)(q[3] & 0xFF) << 24);
  const uint32_t hi = (uint32_t)(q[4] & 0xFF) | ((uint32_t)(q[5] & 0xFF) << 8) | ((uint32_t)(q[6] & 0xFF) << 16) |
                      ((uint32_t)(q[7] & 0xFF) << 24);
  *reinterpret_cast<uint2*>(gb + (m * ng + ul) * 16 + (lane & 1) * 8) = make_uint2(lo, hi);
  if ((lane & 3) == 0) {
    const float dh = __half2float(__float2half_rn(d));
    const int jb = (lane & 15) >> 2;  // Q8_0 block within the unit
    *reinterpret_cast<float*>(gb + 8 * ng * 16 + ul * 16 + jb * 4) = dh;
  }
  if ((lane & 15) == 0) *reinterpret_cast<float*>(gb + 8 * ng * 16 + ng * 16 + ul * 4) = 0.0f;
}

// Several Q8_K blocks of one warp at once (blocks blk0, blk0 + stride, ...,
// the first nb of RB): the same arithmetic as qact_put_q8k, with the warp
// reductions of the blocks interleaved.  The largest |x| (first index on ties)
// is found through one 64-bit key per lane: |x| bits (monotonic for x >= 0),
// then 255 - index, then the sign.
__device__ __forceinline__ unsigned long long shfl_xor_u64(unsigned long long v, int o) {
  const unsigned lo = __shfl_xor_sync(0xffffffffu, (unsigned)v, o);
  const unsigned hi = __shfl_xor_sync(0xffffffffu, (unsigned)(v >> 32), o);
  return ((unsigned long long)hi << 32) | lo;
}
template <int RB>
__device__ __forceinline__ void qact_put_q8k_blocks(uint8_t* qa, int K, int blk0, int stride, int nb,
                                                    const float (&v)[RB][8], int lane) {
  unsigned long long key[RB];
#pragma unroll
  for (int i = 0; i < RB; ++i) {
    key[i] = 0ull;
    if (i < nb) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const unsigned bits = __float_as_uint(v[i][j]);
        const unsigned long long kj = ((unsigned long long)(bits & 0x7fffffffu) << 32) |
                                      ((unsigned long long)(255 - (8 * lane + j)) << 1) | (bits >> 31);
        key[i] = kj > key[i] ? kj : key[i];
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
    for (int i = 0; i < RB; ++i) {
      const unsigned long long ok = shfl_xor_u64(key[i], o);
      key[i] = ok > key[i] ? ok : key[i];
    }
  }
  int q[RB][8], sums[RB];
  float d[RB];
#pragma unroll
  for (int i = 0; i < RB; ++i) {
    const float ax = __uint_as_float((unsigned)(key[i] >> 32));
    const float mv = (key[i] & 1ull) ? -ax : ax;
    d[i] = 0.0f;
    if (ax == 0.0f) {
#pragma unroll
      for (int j = 0; j < 8; ++j) q[i][j] = 0;
    } else {
      const float iscale = __fdiv_rn(-127.0f, mv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int t = nearest_int(__fmul_rn(iscale, v[i][j]));
        q[i][j] = t < 127 ? t : 127;
      }
      d[i] = __fdiv_rn(1.0f, iscale);
    }
    int s = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) s += q[i][j];
    sums[i] = s;
  }
#pragma unroll
  for (int i = 0; i < RB; ++i) sums[i] += __shfl_xor_sync(0xffffffffu, sums[i], 1);
#pragma unroll
  for (int i = 0; i < RB; ++i) {
    if (i < nb) {
      const int blk = blk0 + i * stride;
      const int u = 2 * blk + (lane >> 4);
      const int g = u / GROUP_UNITS, ul = u % GROUP_UNITS, ng = group_units(K, g);
      uint8_t* gb = qa + qact_group_offset(g);
      const int m = (lane & 15) >> 1;
      *reinterpret_cast<uint2*>(gb + (m * ng + ul) * 16 + (lane & 1) * 8) = pack8(q[i]);
      if ((lane & 1) == 0) *reinterpret_cast<int16_t*>(gb + 8 * ng * 16 + ul * 16 + m * 2) = (int16_t)sums[i];
      if ((lane & 15) == 0) *reinterpret_cast<float*>(gb + 8 * ng * 16 + ng * 16 + ul * 4) = d[i];
    }
  }
}

__device__ __forceinline__ void qact_put(int act_type, uint8_t* qa, int K, int blk, const float v[8], int lane) {
  if (act_type == T_Q8_0)
    qact_put_q80(qa, K, blk, v, lane);
  else
    qact_put_q8k(qa, K, blk, v, lane);
}

}  // namespace sfk
