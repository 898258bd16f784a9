// sfk_noalloc.cu -- sfk_moe_ffn_noalloc: the fused routed-expert FFN of
// sfk_moe_ffn, for callers that must not allocate device memory.
//
// sfk_moe_ffn keeps a per-device scratch area that it grows with cudaMalloc.
// Some callers cannot let a library do that: a host engine that has already
// carved all of HBM into its own pools (the planner's HBM budget) and treats
// any further cudaMalloc as a budget violation, a process whose device memory
// is owned by another framework's allocator, or a latency-critical loop where
// cudaMalloc / cudaFree would synchronize the whole device.  This entry point
// takes the same inputs and outputs and keeps its scratch (routing table,
// quantized activations, SwiGLU activations, group counters, status word) in
// one fixed array compiled into the library, so it never allocates.
//
// The array is SFK_NOALLOC_SCRATCH_BYTES (4 MiB) of device memory per GPU that
// loads the library, held until the process exits.  Requests that do not fit
// are rejected before any work is queued.  All calls share the array: two
// calls whose work overlaps on the GPU (different streams, or different host
// threads on one device) overwrite each other's scratch.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "../../include/sfk.h"
#include "sfk_device.cuh"
#include "sfk_kernels.cuh"

using namespace sfk;

static __device__ __align__(256) uint8_t sfk_noalloc_scratch[SFK_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_mu;
uint8_t* g_scratch[kMaxDevices] = {};  // device address of sfk_noalloc_scratch, per device
sfk_status nfail(sfk_status st, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  sfk::set_last_error(buf);  // what sfk_last_error() returns on this thread
  return st;
}

// Resolve the array's device address on the current device (once per device).
sfk_status scratch_for_current_device(uint8_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return nfail(SFK_ERR_RUNTIME, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return nfail(SFK_ERR_UNSUPPORTED, "device %d beyond %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, sfk_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return nfail(SFK_ERR_RUNTIME, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
    g_scratch[dev] = static_cast<uint8_t*>(p);
  }
  *out = g_scratch[dev];
  return SFK_OK;
}

size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }
int act_of(int wtype) { return wtype == T_Q8_0 ? T_Q8_0 : T_Q8_K; }
bool quant_type(int t) { return t == T_Q4_K || t == T_Q6_K || t == T_Q8_0; }

}  // namespace

#define NCK(call)                                                                                 \
  do {                                                                                            \
    cudaError_t e_ = (call);                                                                      \
    if (e_ != cudaSuccess) return nfail(SFK_ERR_RUNTIME, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

extern "C" {

sfk_status sfk_moe_ffn_noalloc(int type_gu, int type_down, const void* gate, const void* up, const void* down,
                               int32_t n_expert, int64_t d, int64_t F, const float* x, const float* res,
                               const int32_t* ids, const float* wts, int32_t b, int32_t k, float* out,
                               void* stream) {
  if (!quant_type(type_gu) || !quant_type(type_down) || d % 256 || F % 256 || !gate || !up || !down || !x || !ids ||
      !wts || !out || b < 1 || b > MAXB || k < 1 || b * k > MAXP || n_expert < 1)
    return nfail(SFK_ERR_INVALID_ARGUMENT, "moe_ffn_noalloc arguments");
  // scratch layout inside the fixed array, every part 256-byte aligned
  const size_t off_status = 0;
  const size_t off_route = 256;
  const size_t off_cnt = off_route + align256(sizeof(Route));
  const size_t off_xq = off_cnt + align256(sizeof(int) * (size_t)(F / 256));
  const size_t off_h = off_xq + align256((size_t)qact_bytes((int)d) * b);
  const size_t off_hq = off_h + align256(sizeof(float) * (size_t)b * k * F);
  const size_t need = off_hq + align256((size_t)qact_bytes((int)F) * b * k);
  if (need > (size_t)SFK_NOALLOC_SCRATCH_BYTES)
    return nfail(SFK_ERR_INVALID_ARGUMENT,
                 "moe_ffn_noalloc: b=%d, k=%d, d=%lld, F=%lld needs %zu bytes of scratch; the fixed area holds %zu",
                 b, k, (long long)d, (long long)F, need, (size_t)SFK_NOALLOC_SCRATCH_BYTES);
  uint8_t* base = nullptr;
  sfk_status s = scratch_for_current_device(&base);
  if (s) return s;
  int* status = reinterpret_cast<int*>(base + off_status);
  Route* route = reinterpret_cast<Route*>(base + off_route);
  int* counters = reinterpret_cast<int*>(base + off_cnt);
  uint8_t* xq = base + off_xq;
  float* h = reinterpret_cast<float*>(base + off_h);
  uint8_t* hq = base + off_hq;
  cudaStream_t st = (cudaStream_t)stream;
  // the status word and the group counters must start at zero
  NCK(cudaMemsetAsync(status, 0, sizeof(int), st));
  NCK(cudaMemsetAsync(counters, 0, sizeof(int) * (size_t)(F / 256), st));

  int dev = 0, sms = 0, grid = 0;
  NCK(cudaGetDevice(&dev));
  NCK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  NCK(launch_route_build(ids, wts, b, k, n_expert, route, status, st));
  NCK(launch_quant_act(act_of(type_gu), x, b, (int)d, xq, st));
  {
    StreamParams p{};
    p.w0 = (const uint8_t*)gate;
    p.w1 = (const uint8_t*)up;
    p.rowstride = dev_row_bytes(type_gu, (int)d);
    p.expert_stride = F * p.rowstride;
    p.rows = (int)F;
    p.K = (int)d;
    p.wtype = type_gu;
    p.nmat = 2;
    p.act_type = act_of(type_gu);
    p.row_align = 1;
    p.b = b; p.k = k; p.n_pairs = b * k; p.n_vec = b;
    p.route = route;
    p.pro = PRO_LOAD;
    p.qact = xq;
    p.qact_stride = qact_bytes((int)d);
    p.epi = EPI_GATEUP;
    p.h = h;
    p.hq = hq;
    p.grp_counter = counters;
    p.h_act_type = act_of(type_down);
    p.status = status;
    if ((s = plan_stream(p, sms, &grid))) return s;
    NCK(launch_stream(p, grid, st, false));
  }
  {
    StreamParams p{};
    p.w0 = (const uint8_t*)down;
    p.rowstride = dev_row_bytes(type_down, (int)F);
    p.expert_stride = d * p.rowstride;
    p.rows = (int)d;
    p.K = (int)F;
    p.wtype = type_down;
    p.nmat = 1;
    p.act_type = act_of(type_down);
    p.row_align = 1;
    p.b = b; p.k = k; p.n_pairs = b * k; p.n_vec = b * k;
    p.route = route;
    p.pro = PRO_LOAD;
    p.qact = hq;
    p.qact_stride = qact_bytes((int)F);
    p.xq_by_pair = 1;
    p.epi = EPI_DOWN;
    p.y = out;
    p.res = res;
    p.y_stride = d;
    p.status = status;
    if ((s = plan_stream(p, sms, &grid))) return s;
    NCK(launch_stream(p, grid, st, false));
  }
  int host_status = 0;
  NCK(cudaMemcpyAsync(&host_status, status, sizeof(int), cudaMemcpyDeviceToHost, st));
  NCK(cudaStreamSynchronize(st));
  if (host_status != ERR_NONE)
    return nfail(SFK_ERR_RUNTIME, "moe_ffn_noalloc: device reported error %d (%s)", host_status,
                 host_status == ERR_BAD_ID ? "expert id out of range" : "bounded wait expired");
  return SFK_OK;
}

}  // extern "C"
