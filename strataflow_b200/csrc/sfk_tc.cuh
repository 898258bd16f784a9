// sfk_tc.cuh -- the tensor-core (tcgen05) quantized GEMM of sfk_tc.cu.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace sfk {

constexpr int TC_TT = 64;  // tokens per activation tile (codes of a tile are contiguous per 256-block)

struct TcGemmParams {
  const uint8_t* w;    // weight rows in the HBM layout
  int64_t rowstride;   // bytes between rows
  int rows, K, wtype;  // rows, columns, ggml type (Q4_K / Q6_K / Q8_0)
  int act_type;        // T_Q8_K (K-quants) or T_Q8_0
  const int8_t* xq;    // activation codes in the tile layout (tc_quant)
  const float* dx;     // activation scales: [npad][K/256] (Q8_K) or [npad][K/32] (Q8_0, f16-rounded)
  const int16_t* bs;   // Q8_K 16-column sums [npad][K/16]
  int n, npad;         // tokens, and tokens padded to a multiple of TC_TT
  float* y;            // [n][ldy] output
  int64_t ldy;
  int* status;
};

// Bytes of the activation buffer of n tokens x K columns and the offsets of
// its scale and sum arrays (codes first).
size_t tc_act_bytes(int act_type, int n, int K, size_t* off_dx, size_t* off_bs);
// Quantize x [n][K] (f32) the ggml way into `buf` (tc_act_bytes bytes).
cudaError_t launch_tc_quant(int act_type, const float* x, int n, int K, uint8_t* buf, cudaStream_t st);
cudaError_t launch_tc_gemm(const TcGemmParams& p, cudaStream_t st);

}  // namespace sfk
