// sfk_dequant.cuh -- element-wise dequantization of GGUF-layout rows.
//
// Bit-exact restatement of ggml's dequantize_row_q8_0 / _q4_K / _q6_K (the
// arithmetic gguf-py 0.19.0 quants.py also restates): every product and
// difference rounds once, in the order ggml writes it, with no FMA contraction.
// Used by the embedding lookup (ggml_get_rows, src/model/engine/engine.cpp:2712)
// and by the sfk_dequantize entry point.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>
#include "sfk_device.cuh"

namespace sfk {

__host__ __device__ inline int64_t dev_gguf_row_bytes(int t, int64_t n) {
  switch (t) {
    case T_F32: return n * 4;
    case T_F16: return n * 2;
    case T_Q8_0: return n / 32 * 34;
    case T_Q4_K: return n / 256 * 144;
    case T_Q6_K: return n / 256 * 210;
    default: return 0;
  }
}

__device__ __forceinline__ float ld_half(const uint8_t* p) {
  return __half2float(*reinterpret_cast<const __half*>(p));
}

__device__ __forceinline__ void scale_min_k4(int j, const uint8_t* q, int* d, int* m) {
  if (j < 4) {
    *d = q[j] & 63;
    *m = q[j + 4] & 63;
  } else {
    *d = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
    *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

// value of element i of a GGUF row of type t
__device__ __forceinline__ float gguf_dequant_one(int t, const uint8_t* row, int64_t i) {
  switch (t) {
    case T_F32: return reinterpret_cast<const float*>(row)[i];
    case T_F16: return __half2float(reinterpret_cast<const __half*>(row)[i]);
    case T_Q8_0: {
      const uint8_t* b = row + (i / 32) * 34;
      const float d = ld_half(b);
      return __fmul_rn((float)(int8_t)b[2 + (i % 32)], d);
    }
    case T_Q4_K: {
      const uint8_t* b = row + (i / 256) * 144;
      const int j = (int)(i % 256);
      const int c = j / 64, hi = (j % 64) >= 32, l = j % 32;
      int sc, m;
      scale_min_k4(2 * c + hi, b + 4, &sc, &m);
      const float d1 = __fmul_rn(ld_half(b), (float)sc);
      const float m1 = __fmul_rn(ld_half(b + 2), (float)m);
      const uint8_t qb = b[16 + 32 * c + l];
      const int q = hi ? (qb >> 4) : (qb & 0xF);
      return __fsub_rn(__fmul_rn(d1, (float)q), m1);
    }
    case T_Q6_K: {
      const uint8_t* b = row + (i / 256) * 210;
      const int j = (int)(i % 256);
      const int n = j / 128, jj = j % 128, quarter = jj / 32, l = jj % 32, is = l / 16;
      const uint8_t* ql = b + 64 * n;
      const uint8_t* qh = b + 128 + 32 * n;
      const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192 + 8 * n);
      int q;
      switch (quarter) {
        case 0: q = (ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4); break;
        case 1: q = (ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4); break;
        case 2: q = (ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4); break;
        default: q = (ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4); break;
      }
      const float d = ld_half(b + 208);
      return __fmul_rn(__fmul_rn(d, (float)sc[is + 2 * quarter]), (float)(q - 32));
    }
    default: return 0.0f;
  }
}

}  // namespace sfk
