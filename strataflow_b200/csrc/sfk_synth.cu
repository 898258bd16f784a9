// sfk_synth.cu -- load-time and utility kernels:
//   * seeded synthetic weights, bit-identical to the CPU fixture generator
//     (splitmix64 counters -> Irwin-Hall(12) normal approximation -> the
//     build's Q4_K / Q6_K / Q8_0 quantizers), so a GPU-resident model of any
//     size can be checked against the CPU oracle byte for byte;
//   * GGUF row layout <-> HBM "lane-interleaved group" layout (repack/unpack);
//   * bit-exact dequantization and standalone activation quantization.
// This file is compiled with -fmad=false: every float expression rounds exactly
// as written, matching the CPU generator built with -ffp-contract=off.
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "sfk_act.cuh"
#include "sfk_dequant.cuh"
#include "sfk_device.cuh"
#include "sfk_kernels.cuh"

namespace sfk {

__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// (sum of twelve 16-bit uniforms - 6*65536) / 65536
__device__ __forceinline__ float synth_z(uint64_t seed, int64_t i) {
  uint32_t s = 0;
#pragma unroll
  for (int w = 0; w < 3; ++w) {
    const uint64_t r = splitmix64(seed + (uint64_t)i * 3u + (uint64_t)w);
    s += (uint32_t)(r & 0xFFFF) + (uint32_t)((r >> 16) & 0xFFFF) + (uint32_t)((r >> 32) & 0xFFFF) +
         (uint32_t)(r >> 48);
  }
  return (float)((int32_t)s - 393210) * (1.0f / 65536.0f);
}

__device__ __forceinline__ uint16_t f16_bits(float f) { return __half_as_ushort(__float2half_rn(f)); }
__device__ __forceinline__ float f16_val(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// Q4_K block quantizer (one warp, lane holds columns 8l..8l+7).  Same steps as
// the CPU fixture quantizer: sub-block min/max -> scale=(max-min)/15, min=-min
// (min clamped to <= 0); 6-bit codes of scales and mins under f16 super-scales
// max/63; q = nearest((x + dmin*m) / (d*sc)) clamped to [0,15].
__device__ void synth_block_q4k(const float v[8], uint8_t* out, uint8_t* sh, int lane) {
  float mn = v[0], mx = v[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) {
    mn = fminf(mn, v[i]);
    mx = fmaxf(mx, v[i]);
  }
#pragma unroll
  for (int o = 1; o < 4; o <<= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  if (mn > 0.0f) mn = 0.0f;
  const float scale = (mx - mn) / 15.0f;
  const float mins = -mn;
  float max_scale = scale, max_min = mins;
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    max_scale = fmaxf(max_scale, __shfl_xor_sync(0xffffffffu, max_scale, o));
    max_min = fmaxf(max_min, __shfl_xor_sync(0xffffffffu, max_min, o));
  }
  max_scale = fmaxf(max_scale, 0.0f);
  max_min = fmaxf(max_min, 0.0f);
  const float inv_scale = max_scale > 0.0f ? 63.0f / max_scale : 0.0f;
  const float inv_min = max_min > 0.0f ? 63.0f / max_min : 0.0f;
  int ls = nearest_int(inv_scale * scale), lm = nearest_int(inv_min * mins);
  ls = ls > 63 ? 63 : (ls < 0 ? 0 : ls);
  lm = lm > 63 ? 63 : (lm < 0 ? 0 : lm);
  const uint16_t dbits = f16_bits(max_scale / 63.0f), mbits = f16_bits(max_min / 63.0f);
  const float d = f16_val(dbits), dmin = f16_val(mbits);
  const float dd = d * (float)ls, dm = dmin * (float)lm;
  uint8_t L[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int q = 0;
    if (dd != 0.0f) {
      float t = (v[i] + dm) / dd;
      t = fminf(fmaxf(t, -1.0f), 16.0f);
      q = nearest_int(t);
      q = q < 0 ? 0 : (q > 15 ? 15 : q);
    }
    L[i] = (uint8_t)q;
  }
  // L codes -> shared, then pack
#pragma unroll
  for (int i = 0; i < 8; ++i) sh[lane * 8 + i] = L[i];
  if ((lane & 3) == 0) {
    sh[256 + lane / 4] = (uint8_t)ls;
    sh[264 + lane / 4] = (uint8_t)lm;
  }
  __syncwarp();
  if (lane < 12) {
    // scales byte `lane`
    uint8_t b;
    const uint8_t* S = sh + 256;
    const uint8_t* M = sh + 264;
    if (lane < 4)
      b = (uint8_t)(S[lane] | ((S[lane + 4] >> 4) << 6));
    else if (lane < 8)
      b = (uint8_t)(M[lane - 4] | ((M[lane] >> 4) << 6));
    else
      b = (uint8_t)((S[lane - 4] & 0xF) | ((M[lane - 4] & 0xF) << 4));
    out[4 + lane] = b;
  }
  if (lane == 0) {
    *reinterpret_cast<uint16_t*>(out) = dbits;
    *reinterpret_cast<uint16_t*>(out + 2) = mbits;
  }
  // qs[32c + l] = L[64c + l] | L[64c + 32 + l] << 4 ; lane writes 4 bytes
  {
    const int byte0 = lane * 4;  // 0..127
    const int c = byte0 / 32, l0 = byte0 % 32;
    uint32_t w = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint8_t b = (uint8_t)(sh[64 * c + l0 + i] | (sh[64 * c + 32 + l0 + i] << 4));
      w |= (uint32_t)b << (8 * i);
    }
    out[16 + byte0 + 0] = (uint8_t)(w);
    out[16 + byte0 + 1] = (uint8_t)(w >> 8);
    out[16 + byte0 + 2] = (uint8_t)(w >> 16);
    out[16 + byte0 + 3] = (uint8_t)(w >> 24);
  }
  __syncwarp();
}

// Q6_K block quantizer: 16-column sub-blocks, scale = (signed max) / -32,
// int8 scales under f16 d = 1/iscale (iscale = -128/max_scale), codes
// nearest(x / (d*sc)) clamped to [-32,31] stored +32.
__device__ void synth_block_q6k(const float v[8], uint8_t* out, uint8_t* sh, int lane) {
  float amax = -1.0f, mv = 0.0f;
  int idx = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float a = fabsf(v[i]);
    if (a > amax) { amax = a; mv = v[i]; idx = lane * 8 + i; }
  }
  {
    const float oa = __shfl_xor_sync(0xffffffffu, amax, 1);
    const float om = __shfl_xor_sync(0xffffffffu, mv, 1);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, 1);
    if (oa > amax || (oa == amax && oi < idx)) { amax = oa; mv = om; idx = oi; }
  }
  const float scale = amax > 0.0f ? mv / -32.0f : 0.0f;
  // first sub-block with the largest |scale|
  float ba = fabsf(scale), bs = scale;
  int bj = lane >> 1;
#pragma unroll
  for (int o = 2; o < 32; o <<= 1) {
    const float oa = __shfl_xor_sync(0xffffffffu, ba, o);
    const float os = __shfl_xor_sync(0xffffffffu, bs, o);
    const int oj = __shfl_xor_sync(0xffffffffu, bj, o);
    if (oa > ba || (oa == ba && oj < bj)) { ba = oa; bs = os; bj = oj; }
  }
  uint8_t L[8];
  uint16_t dbits = 0;
  int8_t scq = 0;
  if (ba == 0.0f) {
#pragma unroll
    for (int i = 0; i < 8; ++i) L[i] = 32;
  } else {
    const float iscale = -128.0f / bs;
    dbits = f16_bits(1.0f / iscale);
    int s = nearest_int(iscale * scale);
    s = s > 127 ? 127 : (s < -128 ? -128 : s);
    scq = (int8_t)s;
    const float dj = f16_val(dbits) * (float)scq;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      int q = 0;
      if (dj != 0.0f) {
        float t = v[i] / dj;
        t = fminf(fmaxf(t, -40.0f), 40.0f);
        q = nearest_int(t);
        q = q < -32 ? -32 : (q > 31 ? 31 : q);
      }
      L[i] = (uint8_t)(q + 32);
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) sh[lane * 8 + i] = L[i];
  __syncwarp();
  // ql: 128 bytes (4 per lane), qh: 64 bytes (2 per lane), scales, d
  for (int bi = 0; bi < 4; ++bi) {
    const int j = lane * 4 + bi;  // ql byte 0..127
    const int n = j / 64, r = j % 64;
    uint8_t b;
    if (r < 32)
      b = (uint8_t)((sh[128 * n + r] & 0xF) | ((sh[128 * n + r + 64] & 0xF) << 4));
    else
      b = (uint8_t)((sh[128 * n + (r - 32) + 32] & 0xF) | ((sh[128 * n + (r - 32) + 96] & 0xF) << 4));
    out[j] = b;
  }
  for (int bi = 0; bi < 2; ++bi) {
    const int j = lane * 2 + bi;  // qh byte 0..63
    const int n = j / 32, l = j % 32;
    const uint8_t q1 = sh[128 * n + l], q2 = sh[128 * n + l + 32], q3 = sh[128 * n + l + 64],
                  q4 = sh[128 * n + l + 96];
    out[128 + j] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
  }
  if ((lane & 1) == 0) out[192 + (lane >> 1)] = (uint8_t)scq;
  if (lane == 0) *reinterpret_cast<uint16_t*>(out + 208) = dbits;
  __syncwarp();
}

// Q8_0 (ggml quantize_row_q8_0_ref) for 8 blocks of 32 held by one warp
__device__ void synth_blocks_q80(const float v[8], uint8_t* out, int lane) {
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  const float d = amax / 127.0f;
  const float id = d != 0.0f ? 1.0f / d : 0.0f;
  uint8_t* blk = out + (lane >> 2) * 34;
  if ((lane & 3) == 0) *reinterpret_cast<__half*>(blk) = __float2half_rn(d);
#pragma unroll
  for (int i = 0; i < 8; ++i) blk[2 + (lane & 3) * 8 + i] = (uint8_t)(int8_t)roundf(v[i] * id);
}

// one warp per 256-column block of a [nrows x K] tensor; GGUF layout output
__global__ void __launch_bounds__(256) synth_kernel(int type, uint64_t seed, float std_, uint8_t* dst, int64_t nrows,
                                                     int K, int64_t row0, int64_t col0, int64_t kfull) {
  __shared__ uint8_t sh[8][288];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t nb_row = K / 256;
  const int64_t total = nrows * nb_row;
  const int64_t rb = dev_gguf_row_bytes(type, K);
  for (int64_t blk = (int64_t)blockIdx.x * 8 + warp; blk < total; blk += (int64_t)gridDim.x * 8) {
    const int64_t row = blk / nb_row, bc = blk % nb_row;
    // element index in the full tensor (rows row0.., columns col0.. of kfull)
    const int64_t e0 = (row0 + row) * kfull + col0 + bc * 256 + lane * 8;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = synth_z(seed, e0 + i) * std_;
    uint8_t* out = dst + row * rb;
    switch (type) {
      case T_Q4_K: synth_block_q4k(v, out + bc * 144, sh[warp], lane); break;
      case T_Q6_K: synth_block_q6k(v, out + bc * 210, sh[warp], lane); break;
      case T_Q8_0: synth_blocks_q80(v, out + bc * 8 * 34, lane); break;
      case T_F32:
#pragma unroll
        for (int i = 0; i < 8; ++i) reinterpret_cast<float*>(out)[bc * 256 + lane * 8 + i] = v[i];
        break;
      default: break;
    }
  }
}

__global__ void synth_f32_kernel(uint64_t seed, float std_, float* dst, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = synth_z(seed, i) * std_;
}

// ---------------------------------------------------------------------------
// GGUF <-> HBM layout.  One warp per (row, group), lane = unit.
// ---------------------------------------------------------------------------
template <bool UNPACK>
__global__ void __launch_bounds__(256) repack_kernel(int type, const uint8_t* src, uint8_t* dst, int64_t nrows, int K) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = n_groups(K);
  const int64_t gg_rb = dev_gguf_row_bytes(type, K);
  const int64_t dv_rb = dev_row_bytes(type, K);
  for (int64_t w = (int64_t)blockIdx.x * 8 + warp; w < nrows * G; w += (int64_t)gridDim.x * 8) {
    const int64_t row = w / G;
    const int g = (int)(w % G);
    const int ng = group_units(K, g);
    uint8_t* grow = (UNPACK ? dst : const_cast<uint8_t*>(src)) + row * gg_rb;  // GGUF row
    uint8_t* drow = (UNPACK ? const_cast<uint8_t*>(src) : dst) + row * dv_rb + group_offset(type, K, g);
    if (lane >= ng) continue;
    const int u = g * GROUP_UNITS + lane;
    auto mv = [&](int64_t goff, int64_t doff, int n) {
      for (int i = 0; i < n; ++i) {
        if (UNPACK)
          grow[goff + i] = drow[doff + i];
        else
          drow[doff + i] = grow[goff + i];
      }
    };
    if (type == T_Q4_K) {
      const int b = u >> 1, h = u & 1;
      for (int i = 0; i < 4; ++i) mv((int64_t)b * 144 + 16 + 64 * h + 16 * i, (i * ng + lane) * 16, 16);
      if (h == 0) mv((int64_t)b * 144, 4 * ng * 16 + (lane >> 1) * 16, 16);
    } else if (type == T_Q6_K) {
      const int b = u >> 1, h = u & 1;
      for (int i = 0; i < 4; ++i) mv((int64_t)b * 210 + 64 * h + 16 * i, (i * ng + lane) * 16, 16);
      for (int i = 4; i < 6; ++i) mv((int64_t)b * 210 + 128 + 32 * h + 16 * (i - 4), (i * ng + lane) * 16, 16);
      mv((int64_t)b * 210 + 192 + 8 * h, 6 * ng * 16 + lane * 8, 8);
      if (h == 0) mv((int64_t)b * 210 + 208, 6 * ng * 16 + (ng / 2) * 16 + (lane >> 1) * 2, 2);
      if (!UNPACK && lane == 0) {
        // zero the pad after the d array
        const int dbytes = (ng / 2) * 2, padded = (dbytes + 15) & ~15;
        for (int i = dbytes; i < padded; ++i) drow[6 * ng * 16 + (ng / 2) * 16 + i] = 0;
      }
    } else if (type == T_Q8_0) {
      for (int i = 0; i < 8; ++i) mv((int64_t)(4 * u + i / 2) * 34 + 2 + 16 * (i & 1), (i * ng + lane) * 16, 16);
      for (int j = 0; j < 4; ++j) mv((int64_t)(4 * u + j) * 34, 8 * ng * 16 + lane * 8 + 2 * j, 2);
    }
  }
}

__global__ void dequant_kernel(int type, const uint8_t* src, float* dst, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = gguf_dequant_one(type, src, i);
}

// qact of b vectors [b][K] (no norm), one warp per 256-column block
__global__ void quant_act_kernel(int act_type, const float* x, int b, int K, uint8_t* dst) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = K / 256;
  for (int w = blockIdx.x * 8 + warp; w < b * nb; w += gridDim.x * 8) {
    const int t = w / nb, blk = w % nb;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = x[(int64_t)t * K + blk * 256 + lane * 8 + i];
    qact_put(act_type, dst + (int64_t)t * qact_bytes(K), K, blk, v, lane);
  }
}

// GGUF-layout activation blocks: Q8_K (f32 d, 256 x i8, 16 x i16 bsums) or
// Q8_0 (f16 d, 32 x i8), one warp per 256 columns
__global__ void quant_act_gguf_kernel(int act_type, const float* x, int b, int K, uint8_t* dst) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = K / 256;
  for (int w = blockIdx.x * 8 + warp; w < b * nb; w += gridDim.x * 8) {
    const int t = w / nb, blk = w % nb;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = x[(int64_t)t * K + blk * 256 + lane * 8 + i];
    if (act_type == T_Q8_K) {
      int q[8], s;
      float d;
      q8k_block(v, lane, q, &d, &s);
      uint8_t* o = dst + ((int64_t)t * nb + blk) * 292;
      if (lane == 0) *reinterpret_cast<float*>(o) = d;
#pragma unroll
      for (int i = 0; i < 8; ++i) o[4 + lane * 8 + i] = (uint8_t)(q[i] & 0xFF);
      if ((lane & 1) == 0) *reinterpret_cast<int16_t*>(o + 260 + (lane >> 1) * 2) = (int16_t)s;
    } else {
      float amax = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      const float d = amax / 127.0f;
      const float id = d != 0.0f ? 1.0f / d : 0.0f;
      uint8_t* o = dst + ((int64_t)t * K / 32 + blk * 8 + (lane >> 2)) * 34;
      if ((lane & 3) == 0) *reinterpret_cast<__half*>(o) = __float2half_rn(d);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[2 + (lane & 3) * 8 + i] = (uint8_t)(int8_t)roundf(v[i] * id);
    }
  }
}

__global__ void fill_kernel(float* dst, float v, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = v;
}

static int grid_for(int64_t work, int per_block) {
  int64_t g = (work + per_block - 1) / per_block;
  if (g > 148 * 16) g = 148 * 16;
  if (g < 1) g = 1;
  return (int)g;
}

cudaError_t launch_synth(int type, uint64_t seed, float std_, uint8_t* dst, int64_t nrows, int K, cudaStream_t st,
                         int64_t row0, int64_t col0, int64_t kfull) {
  if (K % 256) return cudaErrorInvalidValue;
  if (kfull <= 0) kfull = K;
  synth_kernel<<<grid_for(nrows * (K / 256), 8), 256, 0, st>>>(type, seed, std_, dst, nrows, K, row0, col0, kfull);
  return cudaGetLastError();
}
cudaError_t launch_synth_f32(uint64_t seed, float std_, float* dst, int64_t n, cudaStream_t st) {
  synth_f32_kernel<<<grid_for(n, 256), 256, 0, st>>>(seed, std_, dst, n);
  return cudaGetLastError();
}
cudaError_t launch_repack(int type, const uint8_t* src, uint8_t* dst, int64_t nrows, int K, cudaStream_t st) {
  if (K % 256) return cudaErrorInvalidValue;
  repack_kernel<false><<<grid_for(nrows * n_groups(K), 8), 256, 0, st>>>(type, src, dst, nrows, K);
  return cudaGetLastError();
}
cudaError_t launch_unpack(int type, const uint8_t* src, uint8_t* dst, int64_t nrows, int K, cudaStream_t st) {
  if (K % 256) return cudaErrorInvalidValue;
  repack_kernel<true><<<grid_for(nrows * n_groups(K), 8), 256, 0, st>>>(type, src, dst, nrows, K);
  return cudaGetLastError();
}
cudaError_t launch_dequant(int type, const uint8_t* src, float* dst, int64_t n, cudaStream_t st) {
  dequant_kernel<<<grid_for(n, 256), 256, 0, st>>>(type, src, dst, n);
  return cudaGetLastError();
}
cudaError_t launch_quant_act(int act_type, const float* x, int b, int K, uint8_t* dst, cudaStream_t st) {
  if (K % 256) return cudaErrorInvalidValue;
  quant_act_kernel<<<grid_for((int64_t)b * (K / 256), 8), 256, 0, st>>>(act_type, x, b, K, dst);
  return cudaGetLastError();
}
cudaError_t launch_quant_act_gguf(int act_type, const float* x, int b, int K, uint8_t* dst, cudaStream_t st) {
  if (K % 256) return cudaErrorInvalidValue;
  quant_act_gguf_kernel<<<grid_for((int64_t)b * (K / 256), 8), 256, 0, st>>>(act_type, x, b, K, dst);
  return cudaGetLastError();
}
cudaError_t launch_fill_f32(float* dst, float v, int64_t n, cudaStream_t st) {
  fill_kernel<<<grid_for(n, 256), 256, 0, st>>>(dst, v, n);
  return cudaGetLastError();
}

}  // namespace sfk
