// gemm_static.cu — nk_gemm_w8row_f32_static: the int8-row projection with f32
// activations for callers that must not allocate device memory.
//
// The regular entry point (nk_gemm_w8row with x_dtype NK_F32) splits the f32
// activations into bf16 hi | lo halves in a library-grown scratch buffer,
// which may call cudaMalloc.  Some hosts cannot let a library do that: a
// server or engine that owns all device memory through its own pool and
// forbids other allocations, or code on a latency-critical path where a
// cudaMalloc would synchronise the device and stall unrelated streams.
// This variant keeps its split buffer in a fixed file-scope device array
// instead, so a call allocates nothing.
//
// Limits and rules of use:
//   * The array holds kStaticSplitBytes = 8 MiB: m * 2 * ceil(k/64)*64 bf16
//     values (m * 4 * ceil(k/64)*64 bytes) must fit, e.g. m = 64, k = 2048
//     needs 512 KiB.  Larger requests fail with NK_WORKSPACE_TOO_SMALL.
//   * Every GPU that loads libnk holds these 8 MiB until the process exits.
//   * All calls on a device share the one array.  Calls whose kernels overlap
//     on the GPU (other streams, other host threads) race on it; serialise
//     them on one stream.  Each call rewrites every byte it reads (padding
//     included), so no state carries over between calls.
//   * The first call on each device looks up the array's device address
//     (cudaGetSymbolAddress, with that device current); make that first call
//     before any stream capture.
#include <mutex>

#include "gemm_tc.h"

namespace nk {

constexpr size_t kStaticSplitBytes = size_t(8) << 20;

// Device storage for the split activations.  In host code this symbol is only
// a handle: its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_static_split[kStaticSplitBytes];

namespace {

std::mutex g_static_mu;
void *g_static_addr[64];

// Once per device, with that device current: the device address of the array.
nk_status static_split_buffer(void **out) {
  int dev = 0;
  NK_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(NK_DEVICE_ERROR, "device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_static_mu);
  if (!g_static_addr[dev]) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_static_split);
    if (e != cudaSuccess) return fail_cuda(e, "cudaGetSymbolAddress(g_static_split)");
    g_static_addr[dev] = p;
  }
  *out = g_static_addr[dev];
  return NK_OK;
}

}  // namespace
}  // namespace nk

using namespace nk;

extern "C" nk_status nk_gemm_w8row_f32_static(const float *x, const int8_t *wq,
                                              const float *scales, const float *bias, void *y,
                                              int32_t y_dtype, int64_t m, int64_t k, int64_t n,
                                              int32_t flags, void *stream) {
  if (m <= 0 || k <= 0 || n <= 0) return fail(NK_INVALID_SHAPE, "m, k and n must be positive");
  if (y_dtype != NK_BF16 && y_dtype != NK_F32) return fail(NK_UNSUPPORTED, "y_dtype");
  if (m > (1ll << 30) || n > (1ll << 30) || k > (1ll << 30))
    return fail(NK_INVALID_SHAPE, "dimension too large");
  if ((k % 16) != 0 || (reinterpret_cast<uintptr_t>(wq) & 15) != 0)
    return fail(NK_UNSUPPORTED, "the allocation-free variant needs k % 16 == 0 and 16-byte "
                                "aligned weights");
  const int64_t kp = ceil_div(k, 64) * 64;
  const uint64_t need = (uint64_t)m * (uint64_t)(2 * kp) * 2u;
  if (need > kStaticSplitBytes) {
    nk_status st = fail(NK_WORKSPACE_TOO_SMALL,
                        "m * 4 * ceil(k/64)*64 bytes exceed the 8 MiB static split buffer");
    tls_error().expected = need;
    tls_error().actual = kStaticSplitBytes;
    return st;
  }
  void *buf = nullptr;
  nk_status st = static_split_buffer(&buf);
  if (st != NK_OK) return st;
  cudaStream_t s = as_stream(stream);
  // the same split as the regular entry point (every byte rewritten per call)
  st = launch_split_f32(x, m, k, kp, reinterpret_cast<uint16_t *>(buf), s);
  if (st != NK_OK) return st;

  const int bn = m <= 16 ? 16 : (m <= 64 ? 64 : 256);
  TcArgs a{};
  a.f_tiles = (int)ceil_div(n, 128);
  a.t_tiles = (int)ceil_div(m, bn);
  a.n_features = (int)n;
  a.n_tokens = (int)m;
  a.w_k_period = (int)(kp / 64);
  a.k_blocks = 2 * a.w_k_period;
  a.y = y;
  a.ldy = n;
  a.y_f32 = y_dtype == NK_F32;
  a.w_scale = 1.0f;
  a.row_scale = scales;
  a.bias = bias;
  a.relu2 = (flags & NK_EPI_RELU2) != 0;
  a.err = device_error_ptr();
  int64_t tiles = (int64_t)a.f_tiles * a.t_tiles;
  int grid = (int)(tiles < num_sms() ? tiles : num_sms());
  st = tc_gemm(WK_INT8, wq, n, k, k, reinterpret_cast<const uint16_t *>(buf), m, 2 * kp, 2 * kp,
               bn, a, grid, s);
  return st == NK_OK ? ok() : st;
}
