// sfk_prefill.cuh -- the per-token kernels of the batched prompt prefill
// (sfk_prefill.cu) around the tensor-core GEMMs of sfk_tc.cu.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

#include "sfk_kernels.cuh"

namespace sfk {

// x[t][:] = dequantized embedding row of tok[t] (ggml_get_rows); pos[t] =
// pos0 + t; *pos_next (optional) = pos0 + n.
cudaError_t launch_pf_embed(const uint8_t* tok_embd, int type, int d, int V, const int* tok, int n, int pos0, float* x,
                            int* pos, int* pos_next, int* status, cudaStream_t st);
// y[t][:] = rmsnorm(x[t][:]) * w (the decode kernels' formula).
cudaError_t launch_pf_norm(const float* x, const float* w, int n, int d, float eps, float* y, cudaStream_t st);
// RoPE of the Q and K rows of qkv [n][nq + 2 nk] at positions pos0 + t; q
// to q_out [n][nq], K and V appended to the paged pool through the
// sequence's page-table row.
cudaError_t launch_pf_rope_kv(const float* qkv, int n, int n_head, const KvView& kv, const int* pt_row,
                              const float* rope, int pos0, float* q_out, int* status, cudaStream_t st);
// Causal attention of n prompt tokens (positions pos0 + t) over the paged KV
// through the sequence's page table: out [n][nq] (head widths 32, 64, 128, 256;
// the query heads per kv head dividing 64), in the arithmetic of the
// token-by-token attention.  scratch: pf_attn_scratch_bytes(n, pos0, ...).
bool pf_attn_supported(int head_dim, int n_head, int n_head_kv);
size_t pf_attn_scratch_bytes(int n, int pos0, int n_head, int n_head_kv);
cudaError_t launch_pf_attn(const float* q, const KvView& kv, const int* pt_row, int n, int pos0, int n_head,
                           float* out, float* scratch, int* status, cudaStream_t st);
// pt_out[t][:] = pt_row[:] for t < n (every prompt token reads the
// sequence's pages).
cudaError_t launch_pf_pt(const int* pt_row, int max_pages, int n, int* pt_out, cudaStream_t st);
// page_table[idx] = id, in stream order (the id travels as a kernel argument,
// so the host may enqueue later changes without waiting for this one)
cudaError_t launch_pt_set(int* page_table, int idx, int id, cudaStream_t st);
// ffn_norm + router + softmax + top-k of n tokens: ids / w [n][k], xn [n][d]
// (the normed rows); xq_scratch [n][qact_bytes(d)] is written and unused.
cudaError_t launch_pf_route(const float* x, const float* norm_w, const float* w_r, int n, int d, int E, int k,
                            float eps, int act_type, uint8_t* xq_scratch, float* xn, int* ids, float* w, int* status,
                            cudaStream_t st);
// Group the n*k routed pairs by expert: each expert's pairs (ascending) get
// consecutive activation rows from a 64-aligned start; pos_of_pair[i] is
// pair i's row, rows_tok[row] its token (-1 on padding), rows_self[row] the
// row itself (-1 on padding), tile_expert[tile] the expert of each 64-row
// tile (-1 past the last).  max_tiles >= ceil(np / 64) + min(E, np).
cudaError_t launch_pf_group(const int* ids, int np, int k, int E, int max_tiles, int* pos_of_pair, int* rows_tok,
                            int* rows_self, int* tile_expert, int* status, cudaStream_t st);
// x[t][c] = sum_j w[t k + j] * yd[pos_of_pair[t k + j]][c] + res[t][c],
// the experts added in slot order (engine.cpp:1973-1986).
cudaError_t launch_pf_combine(const float* yd, const int* pos_of_pair, const float* w, int k, int n, int d,
                              const float* res, float* x, cudaStream_t st);
// y[i][c] = src[pos_of_pair[i]][c] for i < np, c < rows: the expert-grouped
// GEMM rows put back in pair order.
cudaError_t launch_pf_ungroup(const float* src, const int* pos_of_pair, int np, int64_t rows, float* y,
                              cudaStream_t st);

}  // namespace sfk
