// pipeline.cu — host-buffer MoE forwards with the PCIe copies overlapped.
//
// nk_moe_forward works on device buffers; a caller whose tokens live in host
// memory (the reference's *_into_host entry points, and any serving loop that
// receives activations from the CPU) pays a host->device copy of x and a
// device->host copy of out around every call.  Done back to back, a step
// costs copy-in + forward + copy-out.  The executor below keeps two device
// slots and three streams, so that step i+1's input copy and step i-1's output
// copy run while step i computes; in steady state a step costs the longest of
// the three:
//
//   h2d stream      x_host(i) -> x_dev[i%2]          after forward(i-2) consumed it
//   compute stream  nk_moe_forward(x_dev, out_dev)    after h2d(i) and d2h(i-2)
//   d2h stream      out_dev[i%2] -> out_host(i)       after forward(i)
//
// Ordering is carried by CUDA events only; no host synchronisation happens
// until nk_moe_pipeline_wait.  The forwards themselves run in submission
// order on one stream and share one workspace.
#include <cuda_runtime.h>

#include <new>

#include "nk_common.cuh"

struct nk_moe_pipeline {
  nk_moe_layer layer;
  int64_t max_tokens;
  int32_t out_dtype;
  int device;
  cudaStream_t h2d, compute, d2h;
  bool own_streams;
  void *x_dev[2] = {nullptr, nullptr};
  void *out_dev[2] = {nullptr, nullptr};
  int32_t *idx_dev[2] = {nullptr, nullptr};
  void *workspace = nullptr;
  size_t workspace_bytes = 0;
  cudaEvent_t h2d_done[2] = {}, comp_done[2] = {}, d2h_done[2] = {};
  int64_t submitted = 0;
};

namespace nk {
namespace {

void release(nk_moe_pipeline *p) {
  for (int s = 0; s < 2; ++s) {
    cudaFree(p->x_dev[s]);
    cudaFree(p->out_dev[s]);
    cudaFree(p->idx_dev[s]);
    if (p->h2d_done[s]) cudaEventDestroy(p->h2d_done[s]);
    if (p->comp_done[s]) cudaEventDestroy(p->comp_done[s]);
    if (p->d2h_done[s]) cudaEventDestroy(p->d2h_done[s]);
  }
  cudaFree(p->workspace);
  if (p->own_streams) {
    cudaStreamDestroy(p->h2d);
    cudaStreamDestroy(p->compute);
    cudaStreamDestroy(p->d2h);
  }
  delete p;
}

// Makes the executor's device current for the scope of a call and restores
// the caller's afterwards.
struct DeviceScope {
  int prev = -1;
  cudaError_t err = cudaSuccess;
  explicit DeviceScope(int dev) {
    err = cudaGetDevice(&prev);
    if (err == cudaSuccess && prev != dev) err = cudaSetDevice(dev);
  }
  ~DeviceScope() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

}  // namespace
}  // namespace nk

using namespace nk;

extern "C" {

nk_status nk_moe_pipeline_create(const nk_moe_layer *layer, int64_t max_tokens,
                                 int32_t out_dtype, void *h2d_stream, void *compute_stream,
                                 void *d2h_stream, nk_moe_pipeline **out) {
  if (!out) return fail(NK_INVALID_PARAMS, "out must not be NULL");
  *out = nullptr;
  if (!layer) return fail(NK_INVALID_PARAMS, "layer must not be NULL");
  if (max_tokens <= 0) return fail(NK_INVALID_ROW_COUNT, "row_count must be non-zero");
  if (out_dtype != NK_F32 && out_dtype != NK_BF16) return fail(NK_UNSUPPORTED, "out_dtype");
  const bool given = h2d_stream || compute_stream || d2h_stream;
  if (given && !(h2d_stream && compute_stream && d2h_stream))
    return fail(NK_INVALID_PARAMS, "pass all three streams or none");
  size_t ws = 0;
  nk_status st = nk_moe_workspace_bytes(layer, max_tokens, &ws);
  if (st != NK_OK) return st;

  nk_moe_pipeline *p = new (std::nothrow) nk_moe_pipeline();
  if (!p) return fail(NK_DEVICE_ERROR, "out of host memory");
  p->layer = *layer;
  p->max_tokens = max_tokens;
  p->out_dtype = out_dtype;
  p->own_streams = !given;
  cudaError_t e = cudaGetDevice(&p->device);
  if (e == cudaSuccess && given) {
    p->h2d = as_stream(h2d_stream);
    p->compute = as_stream(compute_stream);
    p->d2h = as_stream(d2h_stream);
  } else if (e == cudaSuccess) {
    p->h2d = p->compute = p->d2h = nullptr;
    e = cudaStreamCreateWithFlags(&p->h2d, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p->compute, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p->d2h, cudaStreamNonBlocking);
  }
  const size_t x_bytes = (size_t)max_tokens * layer->hidden * 2;
  const size_t o_bytes = (size_t)max_tokens * layer->hidden * (out_dtype == NK_F32 ? 4 : 2);
  const size_t i_bytes = (size_t)max_tokens * layer->top_k * 4;
  for (int s = 0; s < 2 && e == cudaSuccess; ++s) {
    e = cudaMalloc(&p->x_dev[s], x_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&p->out_dev[s], o_bytes);
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void **>(&p->idx_dev[s]), i_bytes);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->h2d_done[s], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->comp_done[s], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->d2h_done[s], cudaEventDisableTiming);
  }
  if (e == cudaSuccess) e = cudaMalloc(&p->workspace, ws);
  if (e != cudaSuccess) {
    release(p);
    return fail_cuda(e, "nk_moe_pipeline_create");
  }
  p->workspace_bytes = ws;
  *out = p;
  return ok();
}

nk_status nk_moe_pipeline_submit(nk_moe_pipeline *p, const uint16_t *x_host, int64_t tokens,
                                 void *out_host, int32_t *indices_host) {
  if (!p) return fail(NK_INVALID_PARAMS, "pipeline must not be NULL");
  if (tokens <= 0) return fail(NK_INVALID_ROW_COUNT, "row_count must be non-zero");
  if (tokens > p->max_tokens) return fail(NK_UNSUPPORTED, "tokens exceeds the pipeline's max_tokens");
  if (!x_host || !out_host) return fail(NK_INVALID_PARAMS, "x_host and out_host must not be NULL");
  DeviceScope dev(p->device);
  if (dev.err != cudaSuccess) return fail_cuda(dev.err, "nk_moe_pipeline_submit");
  const int s = (int)(p->submitted & 1);
  const bool reuse = p->submitted >= 2;  // slot s last served submission - 2
  const size_t x_bytes = (size_t)tokens * p->layer.hidden * 2;
  const size_t o_bytes = (size_t)tokens * p->layer.hidden * (p->out_dtype == NK_F32 ? 4 : 2);
  if (reuse) NK_CUDA_TRY(cudaStreamWaitEvent(p->h2d, p->comp_done[s], 0));
  NK_CUDA_TRY(cudaMemcpyAsync(p->x_dev[s], x_host, x_bytes, cudaMemcpyHostToDevice, p->h2d));
  NK_CUDA_TRY(cudaEventRecord(p->h2d_done[s], p->h2d));

  NK_CUDA_TRY(cudaStreamWaitEvent(p->compute, p->h2d_done[s], 0));
  if (reuse) NK_CUDA_TRY(cudaStreamWaitEvent(p->compute, p->d2h_done[s], 0));
  nk_status st = nk_moe_forward(&p->layer, reinterpret_cast<const uint16_t *>(p->x_dev[s]),
                                tokens, p->out_dev[s], p->out_dtype,
                                indices_host ? p->idx_dev[s] : nullptr, nullptr, p->workspace,
                                p->workspace_bytes, p->compute);
  if (st != NK_OK) return st;
  NK_CUDA_TRY(cudaEventRecord(p->comp_done[s], p->compute));

  NK_CUDA_TRY(cudaStreamWaitEvent(p->d2h, p->comp_done[s], 0));
  NK_CUDA_TRY(cudaMemcpyAsync(out_host, p->out_dev[s], o_bytes, cudaMemcpyDeviceToHost, p->d2h));
  if (indices_host)
    NK_CUDA_TRY(cudaMemcpyAsync(indices_host, p->idx_dev[s],
                                (size_t)tokens * p->layer.top_k * 4, cudaMemcpyDeviceToHost,
                                p->d2h));
  NK_CUDA_TRY(cudaEventRecord(p->d2h_done[s], p->d2h));
  ++p->submitted;
  return ok();
}

nk_status nk_moe_pipeline_wait(nk_moe_pipeline *p) {
  if (!p) return fail(NK_INVALID_PARAMS, "pipeline must not be NULL");
  DeviceScope dev(p->device);
  if (dev.err != cudaSuccess) return fail_cuda(dev.err, "nk_moe_pipeline_wait");
  NK_CUDA_TRY(cudaStreamSynchronize(p->h2d));
  NK_CUDA_TRY(cudaStreamSynchronize(p->compute));
  NK_CUDA_TRY(cudaStreamSynchronize(p->d2h));
  return nk_device_status(p->compute);
}

nk_status nk_moe_pipeline_destroy(nk_moe_pipeline *p) {
  if (!p) return ok();
  DeviceScope dev(p->device);
  cudaStreamSynchronize(p->h2d);
  cudaStreamSynchronize(p->compute);
  cudaStreamSynchronize(p->d2h);
  release(p);
  return ok();
}

}  // extern "C"
