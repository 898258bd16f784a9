// sfk_tc.cuh -- the tensor-core (tcgen05) quantized GEMM of sfk_tc.cu.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace sfk {

constexpr int TC_TT = 64;       // activation rows (tokens / routed pairs) per tile
constexpr int TC_SLAB = 20736;  // bytes of one (tile, 256-column block) activation slab
// Slab layout: codes [0, 16384) in the tensor core's K-major core-matrix layout
// (32-column chunk c at c * 2048, 8-row group at 256, 16-byte K half at 128,
// row at 16); then the block's scales.  Q8_K: d [64] f32 at 16384, and two
// more 32-column chunks in the same layout whose columns 0..7 hold the high
// and low parts of the eight 32-column code sums S_j = 128 hi_j + lo_j
// (hi_j in -32..31, lo_j in 0..127; columns 8..15 zero).  Q8_0: d [64][8] f32
// at 16384.
constexpr int TC_SLAB_DX = 16384;
constexpr int TC_SLAB_SHI = 16640;
constexpr int TC_SLAB_SLO = 18688;

enum TcEpilogue : int {
  TC_EPI_STORE = 0,   // y = W x
  TC_EPI_RESID = 1,   // y = W x + res
  TC_EPI_SWIGLU = 2,  // y = silu(W x) * (W2 x)  (gate, up)
};

struct TcGemmParams {
  const uint8_t* w;        // weight rows in the HBM layout (expert 0 when grouped)
  const uint8_t* w2;       // TC_EPI_SWIGLU: the second matrix (up)
  int64_t rowstride;       // bytes between rows
  int64_t expert_stride;   // bytes between experts' matrices (grouped)
  int rows, K, wtype;      // rows, columns, ggml type (Q4_K / Q6_K / Q8_0)
  int act_type;            // T_Q8_K (K-quants) or T_Q8_0
  const uint8_t* xq;       // activation slabs (tc_quant): [tile][K/256][TC_SLAB]
  int n;                   // dense: valid activation rows (outputs past n are not stored)
  int ntile;               // activation tiles launched
  const int* tile_expert;  // grouped: the expert of each tile (-1: unused); null: dense
  float* y;                // [tile * 64 + i][ldy] output
  int64_t ldy;
  const float* res;        // TC_EPI_RESID: [row i][ldres]
  int64_t ldres;
  int epi;
  int* status;
};

// Bytes of the activation slabs of `rows` rows (padded to TC_TT) x K columns.
size_t tc_act_bytes(int rows, int K);
// Quantize the ggml way (Q8_K or Q8_0) into slabs: activation row i of the
// slabs is x[src][:] with src = rows ? rows[i] : i, zeros where src is
// negative or >= n_src; npad rows (a multiple of TC_TT) are written.
cudaError_t launch_tc_quant(int act_type, const float* x, int64_t ldx, const int* rows, int n_src, int npad, int K,
                            uint8_t* buf, cudaStream_t st);
cudaError_t launch_tc_gemm(const TcGemmParams& p, cudaStream_t st);

}  // namespace sfk
