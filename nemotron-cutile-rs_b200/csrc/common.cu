// common.cu — thread-local error record, per-device error word and scratch
// arena, and the library-level entry points of nk.h.
#include <map>
#include <mutex>
#include <utility>
#include <vector>

#include "nk_common.cuh"
#include "nk_ptx.cuh"

namespace nk {

// One thread waits on an mbarrier phase that nothing completes: the bounded
// wait every libnk kernel uses gives up after NK_WAIT_LIMIT_NS and records
// NK_TIMEOUT in the device error word, and the kernel returns.
__global__ void wait_selftest_kernel(int *err) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    mbar_wait(&bar, 0, err);
  }
}

nk_error_info &tls_error() {
  static thread_local nk_error_info e{};
  return e;
}

// One error word per device: kernels write NK_TIMEOUT / NK_DEVICE_ERROR here
// instead of trapping.
static __device__ int g_device_error;

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
int *g_err_ptr[kMaxDevices];
int g_sms[kMaxDevices];

// Library scratch: one block per (device, stream), so calls on different
// streams never share split-K partials or staging buffers.
struct Arena {
  void *ptr = nullptr;
  size_t bytes = 0;
};
std::map<std::pair<int, cudaStream_t>, Arena> g_arenas;

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}
}  // namespace

int *device_error_ptr() {
  int d = current_device();
  if (d < 0 || d >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_err_ptr[d]) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    g_err_ptr[d] = static_cast<int *>(p);
  }
  return g_err_ptr[d];
}

int num_sms() {
  int d = current_device();
  if (d < 0 || d >= kMaxDevices) return 148;
  if (!g_sms[d]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, d);
    g_sms[d] = v > 0 ? v : 148;
  }
  return g_sms[d];
}

// The stream's block only grows.  Growth waits for the stream (only its own
// work uses the block) and is refused while the stream is being captured: a
// captured graph would keep the address of a block freed later.  Warm up at
// the largest shape before capturing.
nk_status scratch(size_t bytes, void **ptr, cudaStream_t stream) {
  int d = current_device();
  if (d < 0 || d >= kMaxDevices) return fail(NK_DEVICE_ERROR, "device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_mu);
  Arena &a = g_arenas[std::make_pair(d, stream)];
  if (a.bytes < bytes) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    NK_CUDA_TRY(cudaStreamIsCapturing(stream, &cs));
    if (cs != cudaStreamCaptureStatusNone) {
      nk_status st = fail(NK_WORKSPACE_TOO_SMALL,
                          "library scratch must grow, which is not allowed during stream capture: "
                          "run the call once at its largest shape before capturing");
      tls_error().expected = bytes;
      tls_error().actual = a.bytes;
      return st;
    }
    size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
    if (a.ptr) {
      NK_CUDA_TRY(cudaStreamSynchronize(stream));
      NK_CUDA_TRY(cudaFree(a.ptr));
      a.ptr = nullptr;
      a.bytes = 0;
    }
    NK_CUDA_TRY(cudaMalloc(&a.ptr, want));
    a.bytes = want;
  }
  *ptr = a.ptr;
  return NK_OK;
}

nk_status release_scratch(cudaStream_t stream) {
  int d = current_device();
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_arenas.find(std::make_pair(d, stream));
  if (it == g_arenas.end()) return NK_OK;
  if (it->second.ptr) {
    NK_CUDA_TRY(cudaStreamSynchronize(stream));
    NK_CUDA_TRY(cudaFree(it->second.ptr));
  }
  g_arenas.erase(it);
  return NK_OK;
}

}  // namespace nk

extern "C" {

nk_status nk_last_error(nk_error_info *out) {
  if (out) *out = nk::tls_error();
  return nk::tls_error().code;
}

int32_t nk_version(void) { return 100; }

nk_status nk_scratch_release(void *stream) {
  nk_status st = nk::release_scratch(nk::as_stream(stream));
  return st == NK_OK ? nk::ok() : st;
}

nk_status nk_selftest_wait_timeout(void *stream) {
  int *err = nk::device_error_ptr();
  if (!err) return nk::fail(NK_DEVICE_ERROR, "cannot resolve device error word");
  nk::wait_selftest_kernel<<<1, 32, 0, nk::as_stream(stream)>>>(err);
  return nk::check_launch("wait_selftest_kernel");
}

nk_status nk_device_status(void *stream) {
  NK_CUDA_TRY(cudaStreamSynchronize(nk::as_stream(stream)));
  int *p = nk::device_error_ptr();
  if (!p) return nk::fail(NK_DEVICE_ERROR, "cannot resolve device error word");
  int v = 0;
  NK_CUDA_TRY(cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost));
  if (v != 0) {
    int zero = 0;
    NK_CUDA_TRY(cudaMemcpy(p, &zero, sizeof(int), cudaMemcpyHostToDevice));
    return nk::fail(v, v == NK_TIMEOUT ? "a bounded device-side wait timed out"
                                       : "a device kernel reported an error");
  }
  return nk::ok();
}

}  // extern "C"
