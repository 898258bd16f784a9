// sfk_mega.cu -- the persistent decode-step kernel.
//
// One cooperative launch = one decode step of engine::Engine::forward
// (src/model/engine/engine.cpp:2498-3025 of Coaade-Inc/strataflow) for b
// sequences: embedding (:2708-2723), then per layer the router segment
// (attn_norm, Q/K/V, RoPE, KV append, attention, O-proj + residual, ffn_norm,
// router softmax / top-k: :1854-1947, :1633-1762) and the expert segment
// (routed gate/up, SwiGLU, down, weighted combine, residual: :1956-1989),
// then output_norm + lm_head + greedy argmax (:2988-3006).
//
// Structure.  One CTA per SM, 16 warps.  A layer is five phases separated
// by grid barriers (QKV | attention | O | routing + gate/up | down); every CTA
// owns a row range of each matrix.  The weight tiles of a CTA's rows are
// dealt to its warps round-robin, and every warp streams its own tiles
// through a ring of S shared-memory slots with 1-D bulk copies (TMA) that it
// issues itself.  The ring runs ahead of the warp across phase boundaries:
// while a CTA waits at a grid barrier, computes attention or routes, its
// warps' slots are already filling with the next matrices' tiles, including
// the F32 router rows, which arrive during the O projection.  Only the
// routed gate/up tiles wait for the routing of their layer.
//
// Numerics are the decode kernels' (sfk_kernels.cu): activations quantized to
// Q8_K / Q8_0 as ggml does, exact integer sub-block dots, the same float
// combination order, and attention in ggml's two-pass order -- scores summed
// in double, the softmax max and sum taken over the whole context before any
// probability is formed, outputs summed in double -- split over CTAs: each
// CTA scores a chunk of positions, the last CTA of a (sequence, kv head) to
// finish forms the softmax statistics, and the last to finish the V pass adds
// the chunks' partial outputs in chunk order.  Every wait is bounded (about a
// second), after which the kernel records ERR_TIMEOUT, lets its in-flight
// copies land and returns; nothing traps.
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "sfk_act.cuh"
#include "sfk_dequant.cuh"
#include "sfk_device.cuh"
#include "sfk_kernels.cuh"
#include "sfk_mega.cuh"
#include "sfk_route.cuh"

namespace sfk {
namespace {

constexpr int NWS = MEGA_NWS;
constexpr int NT = NWS * 32;
constexpr int NC = NWS - 1;   // consumer warps; warp NC (the producer) issues every weight tile
constexpr int NCT = NC * 32;  // consumer threads
// the consumer warps' CTA barrier (the producer warp never joins it)
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory"); }

// streamed phases of a layer (attention streams no weights)
enum : int { SP_QKV = 0, SP_O = 1, SP_RT = 2, SP_GU = 3, SP_DN = 4, SP_N = 5 };
enum : int { K_DENSE = 0, K_ROUTED = 1, K_ROUTER = 2 };

extern __shared__ __align__(128) uint8_t mega_smem[];

struct SDesc {
  const uint8_t* w0;
  const uint8_t* w1;
  int64_t rs, es;
  int r0, r1, R, nmat, kind;
  int H, gpp;  // tiles per row (cut into column-group ranges) and groups per such tile
  int wt, K;   // weight type and row length (columns)
};

__device__ __forceinline__ SDesc stream_desc(const MegaParams& p, int gp) {
  SDesc s;
  s.w1 = nullptr;
  s.es = 0;
  s.nmat = 1;
  s.kind = K_DENSE;
  s.H = 1;
  s.gpp = 8;
  const int c = blockIdx.x;
  if (gp >= p.n_layer * SP_N) {  // lm_head
    s.w0 = p.output;
    s.rs = p.rs_out;
    s.R = p.R[MEGA_PK_OUT];
    s.H = p.H[MEGA_PK_OUT];
    s.gpp = p.gpp[MEGA_PK_OUT];
    s.wt = p.t_out;
    s.K = p.d;
    s.r0 = c * p.rpc_out;
    s.r1 = min(p.V, s.r0 + p.rpc_out);
    return s;
  }
  const int l = gp / SP_N, ph = gp - l * SP_N;
  const MegaLayer* L = reinterpret_cast<const MegaLayer*>(mega_smem + p.off_layers) + l;  // copied at launch
  switch (ph) {
    case SP_QKV:
      s.w0 = reinterpret_cast<const uint8_t*>(L->qkv);
      s.rs = p.rs_attn;
      s.R = p.R[MEGA_PK_QKV];
      s.H = p.H[MEGA_PK_QKV];
      s.gpp = p.gpp[MEGA_PK_QKV];
      s.wt = p.t_attn;
      s.K = p.d;
      s.r0 = c * p.rpc_qkv;
      s.r1 = min(p.nqkv, s.r0 + p.rpc_qkv);
      break;
    case SP_O:
      s.w0 = reinterpret_cast<const uint8_t*>(L->wo);
      s.rs = p.rs_o;
      s.R = p.R[MEGA_PK_O];
      s.H = p.H[MEGA_PK_O];
      s.gpp = p.gpp[MEGA_PK_O];
      s.wt = p.t_attn;
      s.K = p.nq;
      s.r0 = c * p.rpc_o;
      s.r1 = min(p.d, s.r0 + p.rpc_o);
      break;
    case SP_RT:
      s.w0 = reinterpret_cast<const uint8_t*>(L->router);
      s.rs = 0;
      s.R = 1;
      s.r0 = 0;
      s.r1 = 0;
      s.kind = K_ROUTER;
      s.wt = T_F32;
      s.K = p.d;
      break;
    case SP_GU:
      s.w0 = reinterpret_cast<const uint8_t*>(L->gate);
      s.w1 = reinterpret_cast<const uint8_t*>(L->up);
      s.rs = p.rs_gu;
      s.es = (int64_t)p.F * p.rs_gu;
      s.R = p.R[MEGA_PK_GU];
      s.H = p.H[MEGA_PK_GU];
      s.gpp = p.gpp[MEGA_PK_GU];
      s.wt = p.t_gu;
      s.K = p.d;
      s.r0 = c * p.rpc_gu;
      s.r1 = min(p.F, s.r0 + p.rpc_gu);
      s.nmat = 2;
      s.kind = K_ROUTED;
      break;
    default:  // SP_DN
      s.w0 = reinterpret_cast<const uint8_t*>(L->down);
      s.rs = p.rs_down;
      s.es = (int64_t)p.d * p.rs_down;
      s.R = p.R[MEGA_PK_DN];
      s.H = p.H[MEGA_PK_DN];
      s.gpp = p.gpp[MEGA_PK_DN];
      s.wt = p.t_down;
      s.K = p.F;
      s.r0 = c * p.rpc_down;
      s.r1 = min(p.d, s.r0 + p.rpc_down);
      s.kind = K_ROUTED;
      break;
  }
  return s;
}

// Work units of a phase in this CTA: row blocks (x routed experts), or the
// router's row pieces (every CTA takes all of them).  Unit u belongs to consumer warp u % NC and streams as H
// consecutive tiles (column-group ranges of its row when a row is longer than
// a ring slot, else the whole row block).
__device__ __forceinline__ int n_units(const MegaParams& p, const SDesc& s, int n_slots) {
  if (s.kind == K_ROUTER) return p.E * p.rt_parts;
  const int n_rb = s.r0 < s.r1 ? (s.r1 - s.r0 + s.R - 1) / s.R : 0;
  return s.kind == K_ROUTED ? n_rb * n_slots : n_rb;
}

// Shared memory of one CTA; the offsets come from the host plan (MegaParams).

struct Smem {
  const MegaParams& p;
  __device__ explicit Smem(const MegaParams& pp) : p(pp) {}
  // consumer warp c's ring slot s: full[c * S + s] (tile landed), empty[c * S + s] (slot released)
  __device__ uint64_t* full() const { return reinterpret_cast<uint64_t*>(mega_smem); }
  __device__ uint64_t* empty() const { return reinterpret_cast<uint64_t*>(mega_smem) + NWS * MEGA_MAXS; }
  __device__ uint64_t* pro_bar() const { return reinterpret_cast<uint64_t*>(mega_smem) + 2 * NWS * MEGA_MAXS; }
  __device__ uint64_t* kbar() const { return pro_bar() + 1; }
  __device__ uint64_t* vbar() const { return pro_bar() + 2; }
  __device__ uint8_t* slot(int warp, int s) const {
    return mega_smem + p.off_ring + ((int64_t)warp * p.S + s) * p.slot;
  }
  __device__ uint8_t* xq() const { return mega_smem + p.off_xq; }
  __device__ float* acc() const { return reinterpret_cast<float*>(mega_smem + p.off_acc); }
  // the routing of layer l lives in buffer l & 1 (the producer may still read a
  // layer's routing while the consumers route the next one)
  __device__ Route* route(int l) const { return reinterpret_cast<Route*>(mega_smem + p.off_route) + (l & 1); }
  __device__ double* red() const { return reinterpret_cast<double*>(mega_smem + p.off_red); }
  __device__ float* probs() const { return reinterpret_cast<float*>(mega_smem + p.off_probs); }
  __device__ uint8_t* att() const { return mega_smem + p.off_att; }
  __device__ int* toks() const { return reinterpret_cast<int*>(mega_smem + p.off_misc); }
  __device__ int* pos() const { return toks() + MAXB; }
  __device__ int* route_layer(int l) const { return toks() + 2 * MAXB + (l & 1); }  // layer routed into buffer l & 1
  __device__ int* flag() const { return toks() + 2 * MAXB + 2; }
  __device__ int* gp_limit() const { return toks() + 2 * MAXB + 3; }  // last streamed phase the producer may issue
};

// A consumer warp's count of the tiles it has consumed (its ring position).
struct Ring {
  uint32_t n_con;
};

__device__ __forceinline__ bool spin_ge(const unsigned* addr, unsigned target, int* status) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  if (v >= target) return true;
  const long long t0 = clock64();
  for (unsigned i = 1;; ++i) {
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
    if (v >= target) return true;
    if ((i & 31) == 0) {
      if (clock64() - t0 > (1ll << 31)) {
        atomicExch(status, ERR_TIMEOUT);
        return false;
      }
      if (*(volatile int*)status != ERR_NONE) return false;
    }
  }
}

// Bounded mbarrier wait that backs off between polls: a warp waiting for a
// tile sleeps instead of spinning through issue slots the computing warps need.
// ~2^31 cycles (about a second) then ERR_TIMEOUT in *status and false.
__device__ __forceinline__ bool mbar_wait_backoff(uint64_t* bar, uint32_t parity, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (uint32_t i = 1;; ++i) {
    __nanosleep(i < 8 ? 32 : 128);
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 15) == 0) {
      if (clock64() - t0 > (1ll << 31)) {
        atomicExch(status, ERR_TIMEOUT);
        return false;
      }
      if (*(volatile int*)status == ERR_TIMEOUT) return false;
    }
  }
}

__device__ __forceinline__ void st_release_gpu(unsigned* addr, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Grid barrier: every CTA arrives once; returns false when the step failed
// (a bounded wait ran out or a CTA reported an error).
__device__ __forceinline__ bool grid_sync(const MegaParams& p, unsigned& target, int* flag) {
  csync();
  target += gridDim.x;
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(p.gbar, 1u);
    bool ok = spin_ge(p.gbar, target, p.status);
    __threadfence();
    fence_proxy_async_global();  // bulk copies after the barrier read what other CTAs stored before it
    *flag = ok && *(volatile int*)p.status == ERR_NONE;
  }
  csync();
  return *(volatile int*)flag != 0;
}

__device__ __forceinline__ void issue_tile(const MegaParams& p, const SDesc& s, int it, int part, int n_slots,
                                           const Route* rt, uint64_t* bar, uint8_t* dst, uint64_t pol) {
  if (s.kind == K_ROUTER) {  // piece `it`: columns [part * piece, +piece) of router row e
    const int piece = p.d / p.rt_parts;  // floats
    const int e = it / p.rt_parts, pt = it - e * p.rt_parts;
    mbar_arrive_expect_tx(bar, (uint32_t)(piece * 4));
    bulk_g2s(dst, s.w0 + ((int64_t)e * p.d + (int64_t)pt * piece) * 4, (uint32_t)(piece * 4), bar);
    return;
  }
  const int rb = it / n_slots, si = it - rb * n_slots;
  const int rbase = s.r0 + rb * s.R;
  const int expert = s.kind == K_ROUTED ? rt->slot_expert[si] : 0;
  int64_t eoff = (int64_t)expert * s.es + (int64_t)rbase * s.rs;
  uint32_t bytes;
  if (s.H > 1) {  // column groups [g0, g1) of one row
    const int G = n_groups(s.K);
    const int g0 = part * s.gpp, g1 = min(G, g0 + s.gpp);
    const int64_t o0 = group_offset(s.wt, s.K, g0);
    const int64_t o1 = g1 == G ? dev_row_bytes(s.wt, s.K) : group_offset(s.wt, s.K, g1);
    eoff += o0;
    bytes = (uint32_t)(o1 - o0);
  } else {
    bytes = (uint32_t)(min(s.R, s.r1 - rbase) * s.rs);
  }
  mbar_arrive_expect_tx(bar, bytes * s.nmat);
  bulk_g2s_hint(dst, s.w0 + eoff, bytes, bar, pol);
  if (s.nmat == 2) bulk_g2s_hint(dst + (int64_t)s.R * s.rs, s.w1 + eoff, bytes, bar, pol);
}

__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// The producer warp.  Lane c < NC feeds consumer warp c: it walks that warp's
// tiles in stream order (phase gp, the warp's j-th tile of the phase: unit
// c + (j / H) * NC, part j % H) and issues each tile's bulk copies into the
// warp's next ring slot as soon as the warp has released it (empty barrier),
// running ahead across phase boundaries up to the CTA's phase limit; routed
// tiles wait until their layer's routing is in shared memory.  The lanes work
// independently, so one slow consumer does not hold up the others' copies.
// Returns once every tile of the step is issued (or the step failed), after
// letting its last copies land.
__device__ void producer(const MegaParams& p, const Smem& sm, int lane) {
  const int NP = p.n_layer * SP_N + 1;
  const uint64_t pol = l2_evict_first_policy();
  const int c = lane;
  uint32_t n_iss = 0;
  int gp = c < NC ? 0 : NP, j = 0;
  const long long t0 = clock64();
  int idle = 0;
  while (true) {
    bool did = false;
    if (gp < NP && gp <= *(volatile int*)sm.gp_limit()) {
      const int slot = (int)(n_iss & (uint32_t)(p.S - 1));
      // the slot's previous tile (n_iss - S) must have been consumed
      const bool free_slot = n_iss < (uint32_t)p.S || mbar_test(&sm.empty()[c * p.S + slot], ((n_iss >> p.S_log2) + 1) & 1);
      if (free_slot) {
        const SDesc s = stream_desc(p, gp);
        const int l = gp / SP_N;
        int ns = 1;
        bool ready = true;
        if (s.kind == K_ROUTED) {
          ready = *(volatile int*)sm.route_layer(l) == l;  // routing of that layer known
          if (ready) ns = sm.route(l)->n_slots;
        }
        if (ready) {
          const int ju = j / s.H, part = j - ju * s.H;
          const int u = c + ju * NC;
          if (u >= n_units(p, s, ns)) {
            ++gp;
            j = 0;
            did = true;  // progress: look again at once
          } else {
            issue_tile(p, s, u, part, ns, sm.route(l), &sm.full()[c * p.S + slot], sm.slot(c, slot), pol);
            ++n_iss;
            ++j;
            did = true;
          }
        }
      }
    }
    const unsigned any = __ballot_sync(0xffffffffu, did);
    const unsigned live = __ballot_sync(0xffffffffu, gp < NP);
    if (!live) break;
    if (!any) {
      if ((++idle & 63) == 0) {
        if (*(volatile int*)p.status != ERR_NONE) break;  // the step failed: stop issuing
        if (clock64() - t0 > (1ll << 33)) break;          // far beyond any step (bounded loop)
      }
      __nanosleep(64);
    }
  }
  // let this lane's copies in flight land before the CTA may exit
  for (uint32_t k = n_iss > (uint32_t)p.S ? n_iss - p.S : 0u; k < n_iss; ++k)
    mbar_wait_backoff(&sm.full()[c * p.S + (int)(k & (uint32_t)(p.S - 1))], (k >> p.S_log2) & 1, p.status);
}

// The 32-lane butterfly of 8 lane-distributed values (value v ends in the
// lanes with bit 2 = v>>2, bit 3 = (v>>1)&1, bit 4 = v&1), as sfk_kernels.cu.
__device__ __forceinline__ float reduce8m(const float v[8], int lane) {
  const bool b16 = lane & 16, b8 = lane & 8, b4 = lane & 4;
  float w[4], x[2];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float A = v[2 * i], B = v[2 * i + 1];
    const float r = __shfl_xor_sync(0xffffffffu, b16 ? A : B, 16);
    w[i] = b16 ? __fadd_rn(B, r) : __fadd_rn(A, r);
  }
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const float A = w[2 * j], B = w[2 * j + 1];
    const float r = __shfl_xor_sync(0xffffffffu, b8 ? A : B, 8);
    x[j] = b8 ? __fadd_rn(B, r) : __fadd_rn(A, r);
  }
  float y;
  {
    const float r = __shfl_xor_sync(0xffffffffu, b4 ? x[0] : x[1], 4);
    y = b4 ? __fadd_rn(x[1], r) : __fadd_rn(x[0], r);
  }
  y = __fadd_rn(y, __shfl_xor_sync(0xffffffffu, y, 2));
  y = __fadd_rn(y, __shfl_xor_sync(0xffffffffu, y, 1));
  return y;
}

template <int WT>
__device__ __forceinline__ float unit_dot_t(const uint8_t* wg, const XQ8& x, int ng, int lane) {
  if constexpr (WT == T_Q4_K) {
    WQ4K w;
    w.load(wg, ng, lane);
    return dot_unit_q4k(w, x, lane);
  } else if constexpr (WT == T_Q6_K) {
    WQ6K w;
    w.load(wg, ng, lane);
    return dot_unit_q6k(w, x);
  } else {
    WQ80 w;
    w.load(wg, ng, lane);
    return dot_unit_q80(w, x);
  }
}

// The unit dots of one tile for one activation vector xv: value v = rm * Gp +
// g ((row, matrix) rm, local column group g) lands in pv[v].  One-group rows
// (the common case) run up to four independent dots in one basic block.
template <int WT>
__device__ __forceinline__ void tile_dots(const uint8_t* tile, int64_t rs, int R, int nmat, int RM, int K, int g0,
                                          int Gp, const uint8_t* xv, float pv[8], int lane) {
#pragma unroll
  for (int j = 0; j < 8; ++j) pv[j] = 0.0f;
  const int64_t tbase = group_offset(WT, K, g0);
  if (Gp == 1) {
    const int ng = group_units(K, g0);
    if (lane < ng) {
      XQ8 xc;
      xc.load(xv + qact_group_offset(g0), ng, lane);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (q < RM) {
          const int r = nmat == 2 ? (q >> 1) : q, m = nmat == 2 ? (q & 1) : 0;
          pv[q] = unit_dot_t<WT>(tile + ((int64_t)m * R + r) * rs, xc, ng, lane);
        }
      }
    }
    return;
  }
#pragma unroll 1
  for (int g = 0; g < Gp; ++g) {
    const int ng = group_units(K, g0 + g);
    const int64_t goff = group_offset(WT, K, g0 + g) - tbase;
    float d[2] = {0.0f, 0.0f};
    if (lane < ng) {
      XQ8 xc;
      xc.load(xv + qact_group_offset(g0 + g), ng, lane);
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        if (q < RM) {
          const int r = nmat == 2 ? (q >> 1) : q, m = nmat == 2 ? (q & 1) : 0;
          d[q] = unit_dot_t<WT>(tile + ((int64_t)m * R + r) * rs + goff, xc, ng, lane);
        }
      }
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) pv[q] = (q == g) ? d[0] : ((q == Gp + g && RM > 1) ? d[1] : pv[q]);
  }
}

// Consume this warp's tiles of one phase (dense or routed): dot every tile
// row against the phase's activation vectors in xq and store the row sums in
// acc[((row - r0) * n_pairs + pair) * nmat + m].  After each tile the warp
// releases its slot to the producer.  One copy of this
// loop serves every phase (the weight type is a run-time switch per unit dot).
__device__ bool consume(const MegaParams& p, Ring& rg, const Smem& sm, const SDesc& s, const Route* rt, int n_slots,
                        int xq_vec, int by_pair, int n_pairs, int warp, int lane) {
  const int wt = s.wt, K = s.K;
  const int G = n_groups(K);
  const int nu = n_units(p, s, n_slots);
  const int64_t rs = s.rs;
  const int nmat = s.nmat;
  for (int u = warp; u < nu; u += NC) {
    const int rb = u / n_slots, si = u - rb * n_slots;
    const int rbase = s.r0 + rb * s.R;
    const int nrows = min(s.R, s.r1 - rbase);
    const int RM = nrows * nmat;
    int pb = 0, pe = p.b;
    if (s.kind == K_ROUTED) {
      pb = rt->slot_off[si];
      pe = rt->slot_off[si + 1];
    }
    for (int part = 0; part < s.H; ++part) {
      const int slot = (int)(rg.n_con & (uint32_t)(p.S - 1));
      if (!mbar_wait_backoff(&sm.full()[warp * p.S + slot], (rg.n_con >> p.S_log2) & 1, p.status)) return false;
      const uint8_t* tile = sm.slot(warp, slot);
      // this tile's column groups [g0, g0 + Gp); a cut row (H > 1) has one row
      const int g0 = part * s.gpp, Gp = min(G - g0, s.gpp);
      for (int pi = pb; pi < pe; ++pi) {
        const int pair = s.kind == K_ROUTED ? rt->slot_pairs[pi] : pi;
        const int vi = by_pair ? pair : (s.kind == K_ROUTED ? pair / p.k : pair);
        const uint8_t* xv = sm.xq() + (int64_t)vi * xq_vec;
        float pv[8];
        // the weight type is fixed for the whole tile: one straight-line dot
        // block per type, so independent unit dots interleave
        if (wt == T_Q4_K)
          tile_dots<T_Q4_K>(tile, rs, s.R, nmat, RM, K, g0, Gp, xv, pv, lane);
        else if (wt == T_Q6_K)
          tile_dots<T_Q6_K>(tile, rs, s.R, nmat, RM, K, g0, Gp, xv, pv, lane);
        else
          tile_dots<T_Q8_0>(tile, rs, s.R, nmat, RM, K, g0, Gp, xv, pv, lane);
        const float sum = reduce8m(pv, lane);
        // (row, matrix) rm = lane adds its group sums in column order; a cut
        // row continues the sum its previous tile left in acc
        const int r = nmat == 2 ? (lane >> 1) : lane, m = nmat == 2 ? (lane & 1) : 0;
        float* ap = &sm.acc()[((rbase - s.r0 + r) * n_pairs + pair) * nmat + m];
        float tot = (part > 0 && lane < RM) ? *ap : 0.0f;
        for (int g = 0; g < Gp; ++g) {
          const int v = (lane * Gp + g) & 7;
          const int src = ((v >> 2) & 1) << 2 | ((v >> 1) & 1) << 3 | (v & 1) << 4;
          tot = __fadd_rn(tot, __shfl_sync(0xffffffffu, sum, src));
        }
        if (lane < RM) *ap = tot;
      }
      fence_proxy_async_smem();  // the slot's generic reads before the bulk copy that refills it
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.empty()[warp * p.S + slot]);  // the producer may refill the slot
      ++rg.n_con;
    }
  }
  return true;
}

// RMSNorm (times w) of b vectors of K columns and their quantization to the
// activation type `act` into xq (vector stride xq_vec), as ggml: squares
// summed in double, mean = (float)(sum / K), scale = 1/sqrtf(mean + eps),
// y = (x * scale) * w.  norm_w == null: no norm.  The source is global memory
// written by other CTAs (read through L2, one round trip for x and the norm
// weight).  xn (optional): the normalised values in shared memory [b][K].
__device__ void pro_quant(const MegaParams& p, const float* src, const float* norm_w, int K, int act, uint8_t* xq,
                          int xq_vec, float* xn, double* red) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nblk = K / QK_K;
  for (int t = 0; t < p.b; ++t) {
    const float* x = src + (int64_t)t * K;
    auto load8 = [&](int blk, float v[8]) {
      const int c0 = blk * QK_K + lane * 8;
      const float4 a = __ldcg(reinterpret_cast<const float4*>(x + c0));
      const float4 b = __ldcg(reinterpret_cast<const float4*>(x + c0 + 4));
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    };
    float scale = 1.0f;
    if (norm_w) {
      double s = 0.0;
      for (int blk = warp; blk < nblk; blk += NC) {
        float v[8];
        load8(blk, v);
#pragma unroll
        for (int i = 0; i < 8; ++i) s += (double)__fmul_rn(v[i], v[i]);
      }
      s = warp_sum_d(s);
      if (lane == 0) red[warp] = s;
      csync();
      double tot = 0.0;
      for (int w = 0; w < NC; ++w) tot += red[w];  // every thread, same order
      const float mean = (float)(tot / (double)K);
      scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
      csync();  // red is reused
    }
    uint8_t* qa = xq + (int64_t)t * xq_vec;
    for (int blk = warp; blk < nblk; blk += NC) {
      float v[8];
      load8(blk, v);  // an L2 hit: the first pass brought the lines in
      if (norm_w) {
        const float4 wa = __ldg(reinterpret_cast<const float4*>(norm_w + blk * QK_K + lane * 8));
        const float4 wb = __ldg(reinterpret_cast<const float4*>(norm_w + blk * QK_K + lane * 8 + 4));
        const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(__fmul_rn(v[i], scale), wv[i]);
      }
      if (xn) {
        float4* xo = reinterpret_cast<float4*>(xn + (int64_t)t * K + blk * QK_K + lane * 8);
        xo[0] = make_float4(v[0], v[1], v[2], v[3]);
        xo[1] = make_float4(v[4], v[5], v[6], v[7]);
      }
      qact_put(act, qa, K, blk, v, lane);
    }
  }
  csync();
}

__device__ __forceinline__ float kv_load(const MegaParams& p, const uint8_t* base, int64_t idx) {
  return p.kv_f16 ? __half2float(reinterpret_cast<const __half*>(base)[idx]) : reinterpret_cast<const float*>(base)[idx];
}

// ---------------------------------------------------------------------------
// attention of layer l (engine.cpp:1751-1761, ggml's op order):
//   y_j = (float) sum_i (double)(k_ji * q_i) * (1/sqrt(hd))
//   M = max_j y_j,  S = sum_j (double) exp(y_j - M),  p_j = exp(y_j - M) * (float)(1/S)
//   o_i = (float) sum_j (double)(v_ji * p_j)
// Work items are (sequence, kv head, chunk of att_ch positions).
// ---------------------------------------------------------------------------
struct AttItem {
  int t, h, c, nc;
};

__device__ __forceinline__ int att_nc(const MegaParams& p, int n_kv) { return (n_kv + p.att_ch - 1) / p.att_ch; }

__device__ __forceinline__ AttItem att_item(const MegaParams& p, const int* pos_s, int i) {
  AttItem a{0, 0, 0, 0};
  for (int t = 0; t < p.b; ++t) {
    const int nc = att_nc(p, pos_s[t] + 1);
    const int n = nc * p.n_head_kv;
    if (i < n) {
      a.t = t;
      a.h = i / nc;
      a.c = i - a.h * nc;
      a.nc = nc;
      return a;
    }
    i -= n;
  }
  a.nc = 0;
  return a;
}

// thread 0: the K (isv = 0) or V pages of item `a` into the staging buffer
__device__ void att_issue(const MegaParams& p, int l, const AttItem& a, const int* pos_s, int isv, uint8_t* dst,
                          uint64_t* bar) {
  const int n_kv = pos_s[a.t] + 1;
  const int j0 = a.c * p.att_ch;
  const int npg = (min(p.att_ch, n_kv - j0) + 15) >> 4;
  const int kvb = p.kv_f16 ? 2 : 4;
  const uint32_t pg_bytes = (uint32_t)(16 * p.hd * kvb);
  const uint8_t* pool = static_cast<const uint8_t*>(isv ? p.v_pool : p.k_pool) + (int64_t)l * p.kv_layer_bytes;
  uint32_t total = 0;
  for (int i = 0; i < npg; ++i) {
    const int pg = p.page_table[a.t * p.max_pages + (j0 >> 4) + i];
    if (pg >= 0 && pg < p.n_pages) total += pg_bytes;
  }
  mbar_arrive_expect_tx(bar, total);
  for (int i = 0; i < npg; ++i) {
    const int pg = p.page_table[a.t * p.max_pages + (j0 >> 4) + i];
    if (pg < 0 || pg >= p.n_pages) {  // never copy from outside the pool
      atomicExch(p.status, ERR_BAD_PAGE);
      continue;
    }
    bulk_g2s(dst + (int64_t)i * pg_bytes, pool + ((int64_t)pg * p.n_head_kv + a.h) * pg_bytes, pg_bytes, bar);
  }
}

__device__ bool attention(const MegaParams& p, int l, const Smem& sm, const int* pos_s, uint32_t& kph, uint32_t& vph) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gqa = p.gqa, hd = p.hd, CH = p.att_ch;
  const int kvb = p.kv_f16 ? 2 : 4;
  uint8_t* kst = sm.xq();
  uint8_t* vst = sm.xq() + (int64_t)CH * hd * kvb;
  float* qs = reinterpret_cast<float*>(sm.att());          // [gqa][hd]
  float* ys = qs + gqa * hd;                             // [gqa][CH]
  float* ps = ys + gqa * CH;                             // [gqa][CH]
  float* st = ps + gqa * CH;                             // [gqa][2]
  int* flag = sm.flag();
  int total = 0;
  for (int t = 0; t < p.b; ++t) total += att_nc(p, pos_s[t] + 1) * p.n_head_kv;
  const bool single = total <= (int)gridDim.x;  // at most one item per CTA: V staged with K
  unsigned* cnt1 = reinterpret_cast<unsigned*>(p.att_cnt);
  unsigned* cnt2 = cnt1 + p.b * p.n_head_kv;

  // ---- pass 1: scores and chunk maxima; the last chunk forms the statistics
  for (int ii = blockIdx.x; ii < total; ii += gridDim.x) {
    const AttItem a = att_item(p, pos_s, ii);
    const int n_kv = pos_s[a.t] + 1;
    const int j0 = a.c * CH, nj = min(CH, n_kv - j0);
    fence_proxy_async_smem();  // the staging buffer was last read by generic loads
    csync();
    if (tid == 0) {
      att_issue(p, l, a, pos_s, 0, kst, sm.kbar());
      if (single) att_issue(p, l, a, pos_s, 1, vst, sm.vbar());
    }
    for (int i = tid; i < gqa * hd; i += NCT) qs[i] = __ldcg(p.q + (int64_t)a.t * p.nq + (int64_t)a.h * gqa * hd + i);
    csync();
    if (!mbar_wait_backoff(sm.kbar(), kph & 1, p.status)) return false;
    ++kph;
    // y[g][j]: one (position, head) dot per thread, four double chains, the
    // dimensions walked from a per-thread rotation (fewer bank conflicts)
    for (int w = tid; w < nj * gqa; w += NCT) {
      const int jj = w / gqa, g = w - jj * gqa;
      const int rot = (2 * jj + 8 * g) % hd;
      const float* qg = qs + g * hd;
      double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
      int ix = rot;
#pragma unroll 1
      for (int i = 0; i < hd; i += 4) {
        float kv4[4], q4[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          int id = ix + u;
          if (id >= hd) id -= hd;
          kv4[u] = kv_load(p, kst, (int64_t)jj * hd + id);
          q4[u] = qg[id];
        }
        a0 += (double)__fmul_rn(kv4[0], q4[0]);
        a1 += (double)__fmul_rn(kv4[1], q4[1]);
        a2 += (double)__fmul_rn(kv4[2], q4[2]);
        a3 += (double)__fmul_rn(kv4[3], q4[3]);
        ix += 4;
        if (ix >= hd) ix -= hd;
      }
      const float y = __fmul_rn((float)((a0 + a1) + (a2 + a3)), p.att_scale);
      ys[g * CH + jj] = y;
      p.att_y[((int64_t)a.t * p.n_head + a.h * gqa + g) * p.n_ctx + j0 + jj] = y;
    }
    csync();
    if (warp < gqa) {
      float m = -INFINITY;
      for (int jj = lane; jj < nj; jj += 32) m = fmaxf(m, ys[warp * CH + jj]);
      m = warp_max(m);
      if (lane == 0) p.att_cmax[(((int64_t)a.t * p.n_head_kv + a.h) * p.att_nc + a.c) * gqa + warp] = m;
    }
    __threadfence();
    csync();
    if (tid == 0) *flag = atomicAdd(&cnt1[a.t * p.n_head_kv + a.h], 1u) == (unsigned)(a.nc - 1);
    csync();
    if (*(volatile int*)flag) {
      __threadfence();
      // M_g over the chunk maxima, S_g over every score of the context
      if (warp < gqa) {
        float m = -INFINITY;
        for (int c = lane; c < a.nc; c += 32)
          m = fmaxf(m, __ldcg(&p.att_cmax[(((int64_t)a.t * p.n_head_kv + a.h) * p.att_nc + c) * gqa + warp]));
        m = warp_max(m);
        if (lane == 0) st[2 * warp] = m;
      }
      csync();
      const int tpg = (NC / gqa) * 32;  // threads per head: whole warps (gqa <= 8)
      const int g = tid / tpg, r = tid - g * tpg;
      double s = 0.0;
      if (g < gqa) {
        const float M = st[2 * g];
        const float* yg = p.att_y + ((int64_t)a.t * p.n_head + a.h * gqa + g) * p.n_ctx;
        for (int j = r; j < n_kv; j += tpg) s += (double)sfk_expf(__fsub_rn(__ldcg(yg + j), M));
      }
      s = warp_sum_d(s);
      if (lane == 0) sm.red()[warp] = s;
      csync();
      if (tid < gqa) {
        double S = 0.0;
        for (int w = tid * (tpg / 32); w < (tid + 1) * (tpg / 32); ++w) S += sm.red()[w];  // this head's warps, in order
        float* sp = p.att_stat + ((int64_t)a.t * p.n_head + a.h * gqa + tid) * 2;
        sp[0] = st[2 * tid];
        sp[1] = (float)(1.0 / S);
      }
      __threadfence();
      csync();
      if (tid == 0) {
        cnt1[a.t * p.n_head_kv + a.h] = 0u;
        st_release_gpu(&p.att_ready[a.t * p.n_head_kv + a.h], (unsigned)(l + 1));
      }
    }
  }
  // ---- pass 2: probabilities and the V sums; the last chunk adds the chunks
  for (int ii = blockIdx.x; ii < total; ii += gridDim.x) {
    const AttItem a = att_item(p, pos_s, ii);
    const int n_kv = pos_s[a.t] + 1;
    const int j0 = a.c * CH, nj = min(CH, n_kv - j0);
    if (!single) {
      fence_proxy_async_smem();
      csync();
      if (tid == 0) att_issue(p, l, a, pos_s, 1, vst, sm.vbar());
    }
    if (tid == 0) *flag = spin_ge(&p.att_ready[a.t * p.n_head_kv + a.h], (unsigned)(l + 1), p.status) ? 1 : 0;
    csync();
    if (!*(volatile int*)flag) return false;
    if (tid < 2 * gqa) st[tid] = __ldcg(p.att_stat + ((int64_t)a.t * p.n_head + a.h * gqa) * 2 + tid);
    csync();
    for (int w = tid; w < nj * gqa; w += NCT) {
      const int g = w / nj, jj = w - g * nj;
      const float y = single ? ys[g * CH + jj]
                             : __ldcg(p.att_y + ((int64_t)a.t * p.n_head + a.h * gqa + g) * p.n_ctx + j0 + jj);
      ps[g * CH + jj] = __fmul_rn(sfk_expf(__fsub_rn(y, st[2 * g])), st[2 * g + 1]);
    }
    csync();
    if (!mbar_wait_backoff(sm.vbar(), vph & 1, p.status)) return false;
    ++vph;
    double* op = p.att_opart + (((int64_t)a.t * p.n_head_kv + a.h) * p.att_nc + a.c) * gqa * hd;
    for (int w = tid; w < gqa * hd; w += NCT) {
      const int g = w / hd, i = w - g * hd;
      const float* pg = ps + g * CH;
      double s0 = 0.0, s1 = 0.0;
      int jj = 0;
#pragma unroll 1
      for (; jj + 1 < nj; jj += 2) {
        s0 += (double)__fmul_rn(kv_load(p, vst, (int64_t)jj * hd + i), pg[jj]);
        s1 += (double)__fmul_rn(kv_load(p, vst, (int64_t)(jj + 1) * hd + i), pg[jj + 1]);
      }
      if (jj < nj) s0 += (double)__fmul_rn(kv_load(p, vst, (int64_t)jj * hd + i), pg[jj]);
      op[w] = s0 + s1;
    }
    __threadfence();
    csync();
    if (tid == 0) *flag = atomicAdd(&cnt2[a.t * p.n_head_kv + a.h], 1u) == (unsigned)(a.nc - 1);
    csync();
    if (*(volatile int*)flag) {
      __threadfence();
      const double* base = p.att_opart + ((int64_t)a.t * p.n_head_kv + a.h) * p.att_nc * gqa * hd;
      for (int w = tid; w < gqa * hd; w += NCT) {
        double s = 0.0;
        for (int c = 0; c < a.nc; ++c) s += __ldcg(base + (int64_t)c * gqa * hd + w);
        p.attn_out[(int64_t)a.t * p.nq + (int64_t)a.h * gqa * hd + w] = (float)s;
      }
      if (tid == 0) cnt2[a.t * p.n_head_kv + a.h] = 0u;
    }
    csync();
  }
  return true;
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
// Steps of a layer; each ends at a grid barrier except routing, which gate/up
// follows directly.  The lm_head step closes the launch.
enum : int { ST_QKV = 0, ST_ATT = 1, ST_O = 2, ST_RT = 3, ST_GU = 4, ST_DN = 5, ST_N = 6 };

// The F32 router pieces of this warp (one per ring slot, in stream order)
// against the normalised inputs xn [b][d]: double partial logits
// part[t * items + i].
__device__ bool router_partials(const MegaParams& p, Ring& rg, const Smem& sm, const float* xn, double* part, int warp,
                                int lane) {
  const int items = p.E * p.rt_parts, piece = p.d / p.rt_parts;
  for (int i = warp; i < items; i += NC) {
    const int slot = (int)(rg.n_con & (uint32_t)(p.S - 1));
    if (!mbar_wait_backoff(&sm.full()[warp * p.S + slot], (rg.n_con >> p.S_log2) & 1, p.status)) return false;
    const float* ws = reinterpret_cast<const float*>(sm.slot(warp, slot));
    const int pt = i % p.rt_parts;
    for (int t = 0; t < p.b; ++t) {
      // logit = sum_c (double)(w_r[e][c] * xn[c]) (ggml's F32 mul_mat): four
      // chains per lane; the pieces of a row are added in order afterwards
      const float* xs = xn + (int64_t)t * p.d + pt * piece;
      double a0 = 0.0, a1 = 0.0, a2 = 0.0, a3 = 0.0;
      for (int c = lane * 4; c < piece; c += 128) {
        const float4 w4 = *reinterpret_cast<const float4*>(ws + c);
        const float4 x4 = *reinterpret_cast<const float4*>(xs + c);
        a0 += (double)__fmul_rn(w4.x, x4.x);
        a1 += (double)__fmul_rn(w4.y, x4.y);
        a2 += (double)__fmul_rn(w4.z, x4.z);
        a3 += (double)__fmul_rn(w4.w, x4.w);
      }
      const double a = warp_sum_d((a0 + a1) + (a2 + a3));
      if (lane == 0) part[t * items + i] = a;
    }
    fence_proxy_async_smem();  // the slot's generic reads before the bulk copy that refills it
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty()[warp * p.S + slot]);
    ++rg.n_con;
  }
  return true;
}

// Epilogue of QKV: RoPE on q and k (engine.cpp:1892-1897), q to its buffer,
// K and V appended to this step's KV pages (:1646-1656).
__device__ void epi_qkv(const MegaParams& p, int l, const float* acc, int r0, int r1, const int* pos_s) {
  const int hd = p.hd, nq = p.nq, nk = p.nk;
  const int npr = (r1 - r0) / 2;
  for (int idx = threadIdx.x; idx < npr * p.b; idx += NCT) {
    const int t = idx / npr;
    const int r = r0 + 2 * (idx - t * npr);
    const float x0 = acc[(r - r0) * p.b + t];
    const float x1 = acc[(r + 1 - r0) * p.b + t];
    const int pos = pos_s[t];
    float o0 = x0, o1 = x1;
    if (r < nq + nk) {
      const int i = (r % hd) >> 1;
      const float2 cs = reinterpret_cast<const float2*>(p.rope)[(int64_t)pos * (hd >> 1) + i];
      o0 = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
      o1 = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
    }
    if (r < nq) {
      p.q[(int64_t)t * nq + r] = o0;
      p.q[(int64_t)t * nq + r + 1] = o1;
    } else {
      const bool is_k = r < nq + nk;
      const int rr = r - nq - (is_k ? 0 : nk);
      const int hh = rr / hd, i0 = rr % hd;
      const int page = p.page_table[t * p.max_pages + pos / 16];
      if (page < 0 || page >= p.n_pages) {  // never write outside the pool
        atomicExch(p.status, ERR_BAD_PAGE);
        continue;
      }
      const int64_t off = (((int64_t)page * p.n_head_kv + hh) * 16 + (pos & 15)) * hd + i0;
      uint8_t* base = static_cast<uint8_t*>(is_k ? p.k_pool : p.v_pool) + (int64_t)l * p.kv_layer_bytes;
      if (p.kv_f16) {
        __half* kb = reinterpret_cast<__half*>(base);
        kb[off] = __float2half_rn(o0);
        kb[off + 1] = __float2half_rn(o1);
      } else {
        float* kb = reinterpret_cast<float*>(base);
        kb[off] = o0;
        kb[off + 1] = o1;
      }
    }
  }
}

// Epilogue of gate/up: h = silu(gate) * up (ggml_swiglu_split, engine.cpp:1969);
// the CTA that completes a 256-row group of h quantizes it for the down
// projection (group counters, reset by that CTA).
__device__ void epi_gateup(const MegaParams& p, const Smem& sm, const float* acc, int r0, int r1) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int np = p.b * p.k, nr = r1 - r0;
  for (int idx = tid; idx < nr * np; idx += NCT) {
    const int row = idx % nr, pr = idx / nr;
    const float g = acc[(row * np + pr) * 2 + 0];
    const float u = acc[(row * np + pr) * 2 + 1];
    const float sl = __fdiv_rn(g, __fadd_rn(1.0f, sfk_expf(-g)));
    p.h[(int64_t)pr * p.F + r0 + row] = __fmul_rn(sl, u);
  }
  __threadfence();
  csync();
  int* gflag = reinterpret_cast<int*>(sm.red());
  const int q0 = r0 / QK_K, q1 = (r1 - 1) / QK_K;
  if (tid == 0) {
    for (int q = q0; q <= q1; ++q) {
      const int lo = max(r0, q * QK_K), hi = min(r1, (q + 1) * QK_K);
      const int old = atomicAdd(&p.grp_counter[q], hi - lo);
      gflag[q - q0] = (old + (hi - lo) == QK_K) ? 1 : 0;
    }
  }
  csync();
  for (int q = q0; q <= q1; ++q) {
    if (!gflag[q - q0]) continue;
    __threadfence();
    for (int pr = warp; pr < np; pr += NC) {
      const float* hp = p.h + (int64_t)pr * p.F + q * QK_K + lane * 8;
      const float4 a4 = __ldcg(reinterpret_cast<const float4*>(hp));
      const float4 b4 = __ldcg(reinterpret_cast<const float4*>(hp + 4));
      const float v[8] = {a4.x, a4.y, a4.z, a4.w, b4.x, b4.y, b4.z, b4.w};
      qact_put(p.a_down, p.hq + (int64_t)pr * qact_bytes(p.F), p.F, q, v, lane);
    }
    if (tid == 0) atomicExch(&p.grp_counter[q], 0);
  }
}

// Epilogue of lm_head: logits and the greedy argmax (first max wins,
// ggml_model.cpp:284-292; engine.cpp:3111-3121) folded into a 64-bit key.
__device__ void epi_lmhead(const MegaParams& p, const Smem& sm, const float* acc, int r0, int r1) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nr = r1 - r0;
  unsigned long long* kred = reinterpret_cast<unsigned long long*>(sm.red());
  for (int t = 0; t < p.b; ++t) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int row = tid; row < nr; row += NCT) {
      const float v = acc[row * p.b + t];
      if (p.store_logits) p.logits[(int64_t)t * p.V + r0 + row] = v;
      if (v > best) { best = v; bi = r0 + row; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if (lane == 0) {
      const unsigned bb = __float_as_uint(best);
      const unsigned ord = (bb & 0x80000000u) ? ~bb : (bb | 0x80000000u);
      kred[warp] = bi == 0x7fffffff
                       ? 0ull
                       : (((unsigned long long)ord << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)bi));
    }
    csync();
    if (tid == 0) {
      unsigned long long m = 0;
      for (int w = 0; w < NC; ++w) m = kred[w] > m ? kred[w] : m;
      if (m) atomicMax(&p.argmax_key[t], m);
    }
    csync();
  }
}

// Routing of layer l (engine.cpp:1913-1924): logits from the router rows in
// the ring, softmax, top-k, renormalised weights, slot lists; then the
// producer may issue the routed gate/up tiles.
__device__ bool route_layer(const MegaParams& p, int l, Ring& rg, const Smem& sm, const float* xn, int warp, int lane) {
  const int tid = threadIdx.x;
  double* part = reinterpret_cast<double*>(sm.probs());
  bool ok = true;
  if (!router_partials(p, rg, sm, xn, part, warp, lane)) ok = false;
  csync();
  if (!ok) return false;
  const int items = p.E * p.rt_parts;
  float* probs = const_cast<float*>(xn) + (int64_t)p.b * p.d;  // [b][E]
  for (int i = tid; i < p.b * p.E; i += NCT) {
    const int t = i / p.E, e = i - t * p.E;
    double a = 0.0;
    for (int pt = 0; pt < p.rt_parts; ++pt) a += part[t * items + e * p.rt_parts + pt];
    probs[i] = (float)a;
  }
  csync();
  Route* rt = sm.route(l);
  for (int t = warp; t < p.b; t += NC) route_select(probs + t * p.E, p.E, p.k, &rt->ids[t * p.k], &rt->w[t * p.k], lane);
  csync();
  if (warp == 0) build_slots_warp(rt->ids, p.b * p.k, rt, lane);
  if (tid == 0) {
    rt->k = p.k;
    rt->b = p.b;
  }
  csync();
  if (tid == 0) *(volatile int*)sm.route_layer(l) = l;  // the producer may issue this layer's routed tiles
  if (blockIdx.x == 0) {  // the routing of the last layer, for the host
    const int* src = reinterpret_cast<const int*>(rt);
    int* dst = reinterpret_cast<int*>(p.route_out);
    for (int i = tid; i < (int)(sizeof(Route) / 4); i += NCT) dst[i] = src[i];
  }
  csync();
  return true;
}

__global__ void __launch_bounds__(NT, 1) mega_kernel(const __grid_constant__ MegaParams p) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  Smem sm(p);
  int* toks = sm.toks();
  int* pos_s = sm.pos();
  int* flag = sm.flag();
  const int cta = blockIdx.x;

  {  // the per-layer weight pointers, read on every tile issue, live in shared memory
    const int n = p.n_layer * (int)(sizeof(MegaLayer) / 8);
    unsigned long long* dst = reinterpret_cast<unsigned long long*>(mega_smem + p.off_layers);
    const unsigned long long* src = reinterpret_cast<const unsigned long long*>(p.layers);
    for (int i = tid; i < n; i += NT) dst[i] = __ldg(src + i);
  }
  if (tid == 0) {
    for (int i = 0; i < NC * p.S; ++i) {
      mbar_init(&sm.full()[i], 1);   // the producer lane's arrival + the copies' bytes
      mbar_init(&sm.empty()[i], 1);  // the consumer warp's release
    }
    mbar_init(sm.pro_bar(), 1);
    mbar_init(sm.kbar(), 1);
    mbar_init(sm.vbar(), 1);
    fence_mbar_init();
    *sm.route_layer(0) = -1;
    *sm.route_layer(1) = -1;
    *sm.gp_limit() = p.lookahead;  // the first step streams QKV of layer 0
  }
  // tokens and positions of the step (the embed kernel's duties)
  if (tid < p.b) {
    int tok;
    if (p.greedy) {
      const unsigned long long key = __ldcg(&p.argmax_key[tid]);
      tok = (int)(0xFFFFFFFFu - (unsigned)(key & 0xFFFFFFFFull));
    } else {
      tok = __ldcg(&p.tok_in[tid]);
    }
    if (tok < 0 || tok >= p.V) {
      if (cta == 0) atomicExch(p.status, ERR_BAD_ID);
      tok = 0;
    }
    int pos = p.pos_in ? __ldcg(&p.pos_in[tid]) : __ldcg(&p.pos_state[tid]);
    if (pos < 0 || pos >= p.n_ctx || pos >= p.max_pages * 16) {
      if (cta == 0) atomicExch(p.status, ERR_BAD_POS);
      pos = 0;
    }
    toks[tid] = tok;
    pos_s[tid] = pos;
  }
  __syncthreads();  // the last barrier of the whole CTA: the producer warp leaves here
  if (warp == NC) {
    producer(p, sm, lane);
    return;
  }
  Ring rg{0u};
  unsigned target = 0;
  {  // the embedding rows (ggml_get_rows, engine.cpp:2708-2723), a column slice per CTA
    const int64_t erb = dev_gguf_row_bytes(p.t_embd, p.d);
    const int per = (p.d + gridDim.x - 1) / gridDim.x;
    const int c0 = cta * per, c1 = min(p.d, c0 + per);
    for (int t = 0; t < p.b; ++t)
      for (int i = c0 + tid; i < c1; i += NCT)
        p.x[(int64_t)t * p.d + i] = gguf_dequant_one(p.t_embd, p.tok_embd + (int64_t)toks[t] * erb, i);
  }
  uint32_t pro_ph = 0, kph = 0, vph = 0;
  const int n_steps = p.n_layer * ST_N + 1;
  const int np = p.b * p.k;
  bool ok = grid_sync(p, target, flag);  // x holds the embeddings
  if (cta == 0 && tid < p.b) {  // every CTA has read the argmax keys by now
    p.argmax_key[tid] = 0ull;
    p.pos_cur[tid] = pos_s[tid];
    if (p.pos_state) p.pos_state[tid] = pos_s[tid] + 1;
    p.tok_hist[tid] = toks[tid];
  }
  for (int gs = 0; gs < n_steps && ok; ++gs) {
    const int l = gs / ST_N;
    const int st = gs == n_steps - 1 ? -1 : gs - l * ST_N;  // -1: lm_head
    const MegaLayer* LW = reinterpret_cast<const MegaLayer*>(mega_smem + p.off_layers) + (l < p.n_layer ? l : 0);
    {  // how far the rings may run ahead: this step's streamed phase + lookahead
      const int cur = st == -1 ? SP_N * p.n_layer
                               : l * SP_N + (st <= ST_QKV ? SP_QKV : st <= ST_O ? SP_O : st == ST_RT ? SP_RT
                                                                   : st == ST_GU ? SP_GU : SP_DN);
      if (tid == 0) *(volatile int*)sm.gp_limit() = cur + p.lookahead;
    }
    if (st == ST_ATT) {  // attention over the paged KV (engine.cpp:1751-1761)
      ok = attention(p, l, sm, pos_s, kph, vph) && grid_sync(p, target, flag);
      continue;
    }
    // ---- prologue: the step's activation vectors into xq
    float* xn = reinterpret_cast<float*>(sm.xq() + (((int64_t)p.b * qact_bytes(p.d) + 15) & ~(int64_t)15));
    if (st == ST_DN) {  // the quantized SwiGLU activations of every pair
      const int xv = (int)qact_bytes(p.F);
      fence_proxy_async_smem();
      csync();
      if (tid == 0) {
        mbar_arrive_expect_tx(sm.pro_bar(), (uint32_t)(np * xv));
        for (int pr = 0; pr < np; ++pr)
          bulk_g2s(sm.xq() + (int64_t)pr * xv, p.hq + (int64_t)pr * xv, (uint32_t)xv, sm.pro_bar());
      }
      if (!mbar_wait_backoff(sm.pro_bar(), pro_ph & 1, p.status)) { ok = false; break; }
      ++pro_ph;
    } else if (st != ST_GU) {
      // attn_norm (QKV), none (O), ffn_norm (routing), output_norm (lm_head)
      const float* src = st == ST_O ? p.attn_out : (st == ST_RT ? p.ffn_inp : p.x);
      const float* nw = st == ST_QKV ? LW->attn_norm : (st == ST_RT ? LW->ffn_norm : (st == -1 ? p.out_norm : nullptr));
      const int K = st == ST_O ? p.nq : p.d;
      const int act = st == ST_RT ? p.a_gu : (st == -1 ? p.a_out : p.a_attn);
      pro_quant(p, src, nw, K, act, sm.xq(), (int)qact_bytes(K), st == ST_RT ? xn : nullptr, sm.red());
    }
    if (st == ST_RT) {
      if (!route_layer(p, l, rg, sm, xn, warp, lane)) { ok = false; break; }
      continue;  // gate/up follows without a barrier
    }
    // ---- the step's weight tiles
    const int sp = st == -1 ? SP_N * p.n_layer
                            : l * SP_N + (st == ST_QKV ? SP_QKV : st == ST_O ? SP_O : st == ST_GU ? SP_GU : SP_DN);
    const SDesc s = stream_desc(p, sp);
    {
      const bool routed = st == ST_GU || st == ST_DN;
      const Route* rt = sm.route(l);
      if (!consume(p, rg, sm, s, rt, routed ? rt->n_slots : 1, (int)qact_bytes(s.K), st == ST_DN ? 1 : 0,
                   routed ? np : p.b, warp, lane)) {
        ok = false;
        break;
      }
    }
    csync();
    // ---- epilogue
    const int nr = s.r0 < s.r1 ? s.r1 - s.r0 : 0;
    const float* acc = sm.acc();
    if (st == ST_QKV) {
      epi_qkv(p, l, acc, s.r0, s.r0 + nr, pos_s);
    } else if (st == ST_O) {  // + residual (engine.cpp:1905-1906)
      for (int idx = tid; idx < nr * p.b; idx += NCT) {
        const int t = idx / nr, row = idx - t * nr;
        const int64_t o = (int64_t)t * p.d + s.r0 + row;
        p.ffn_inp[o] = __fadd_rn(acc[row * p.b + t], __ldcg(p.x + o));
      }
    } else if (st == ST_GU) {
      if (nr > 0) epi_gateup(p, sm, acc, s.r0, s.r1);
    } else if (st == ST_DN) {  // experts * weights, moe_out = e0 + e1 + ..., + ffn_inp (engine.cpp:1973-1986)
      const Route* rt = sm.route(l);
      const int k = p.k;
      for (int idx = tid; idx < nr * p.b; idx += NCT) {
        const int row = idx % nr, t = idx / nr;
        float a = __fmul_rn(acc[row * np + t * k], rt->w[t * k]);
        for (int j = 1; j < k; ++j) a = __fadd_rn(a, __fmul_rn(acc[row * np + t * k + j], rt->w[t * k + j]));
        const int64_t o = (int64_t)t * p.d + s.r0 + row;
        p.x[o] = __fadd_rn(a, __ldcg(p.ffn_inp + o));
      }
    } else {
      epi_lmhead(p, sm, acc, s.r0, s.r0 + nr);
      break;  // the last step: no barrier
    }
    if (!grid_sync(p, target, flag)) { ok = false; break; }
  }
  if (!ok) return;  // the producer lets the copies it issued land; the host clears the counters
  // the last CTA out re-arms the barrier words and the attention flags for the next launch
  csync();
  if (tid == 0) {
    __threadfence();
    const unsigned old = atomicAdd(p.gbar + 1, 1u);
    if (old == gridDim.x - 1) {
      for (int i = 0; i < p.b * p.n_head_kv; ++i) p.att_ready[i] = 0u;
      p.gbar[0] = 0u;
      p.gbar[1] = 0u;
      __threadfence();
    }
  }
}

cudaError_t launch_k(const MegaParams& p, int grid, cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(mega_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, p.smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once: the grid barriers rely on it
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, mega_kernel, p);
}

}  // namespace

bool mega_types_supported(int ta, int tg, int td, int to) {
  auto q = [](int t) { return t == T_Q4_K || t == T_Q6_K || t == T_Q8_0; };
  return q(ta) && q(tg) && q(td) && q(to);
}

cudaError_t launch_mega(const MegaParams& p, int grid, cudaStream_t st) { return launch_k(p, grid, st); }

}  // namespace sfk
