// device.cu — the device bridge of the C ABI: streams, events, device and
// pinned host buffers and copies, as thin wrappers over the CUDA runtime, so a
// host written in another language (the Rust crate's extern "C" block) needs
// no second CUDA binding to drive the attention entry points.
//
// Reference counterparts (lisa-rs src/device/metal.rs, the Metal/objc bridge
// this replaces): MetalDevice::name / max_working_set (160-175), new_buffer /
// new_untracked_buffer (176-199), new_command_queue (200-206),
// CommandBuffer::commit / wait_until_completed (314-321), MetalBuffer::
// read_bytes / write_bytes (396-410) and the buffer's Drop (414-420). Metal
// buffers are CPU-visible unified memory; on a B200 device memory is separate,
// so reads and writes are explicit copies, ordered on a stream.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "../../include/lisa_attn.h"

namespace {

int st(cudaError_t e) { return e == cudaSuccess ? LISA_OK : LISA_ECUDA; }

int set_device(int device) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return LISA_EINVAL;
  return st(cudaSetDevice(device));
}

}  // namespace

#pragma GCC visibility push(default)
extern "C" {

int lisa_attn_dev_count(int* count) {
  if (!count) return LISA_EINVAL;
  *count = 0;
  return st(cudaGetDeviceCount(count));
}

int lisa_attn_dev_info(int device, char* name, size_t name_bytes, uint64_t* total_bytes, int* sm_count) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return LISA_EINVAL;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return LISA_ECUDA;
  if (name && name_bytes) {
    strncpy(name, prop.name, name_bytes - 1);
    name[name_bytes - 1] = 0;
  }
  if (total_bytes) *total_bytes = prop.totalGlobalMem;
  if (sm_count) *sm_count = prop.multiProcessorCount;
  return LISA_OK;
}

int lisa_attn_dev_select(int device) { return set_device(device); }

int lisa_attn_buffer_alloc(int device, size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return LISA_EINVAL;
  *ptr = nullptr;
  int s = set_device(device);
  if (s != LISA_OK) return s;
  return st(cudaMalloc(ptr, bytes));
}

int lisa_attn_buffer_free(void* ptr) {
  if (!ptr) return LISA_EINVAL;
  return st(cudaFree(ptr));
}

int lisa_attn_host_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return LISA_EINVAL;
  *ptr = nullptr;
  return st(cudaHostAlloc(ptr, bytes, cudaHostAllocPortable));
}

int lisa_attn_host_free(void* ptr) {
  if (!ptr) return LISA_EINVAL;
  return st(cudaFreeHost(ptr));
}

int lisa_attn_stream_create(int device, void** stream) {
  if (!stream) return LISA_EINVAL;
  *stream = nullptr;
  int s = set_device(device);
  if (s != LISA_OK) return s;
  cudaStream_t h = nullptr;
  s = st(cudaStreamCreateWithFlags(&h, cudaStreamNonBlocking));
  *stream = h;
  return s;
}

int lisa_attn_stream_destroy(void* stream) {
  if (!stream) return LISA_EINVAL;
  return st(cudaStreamDestroy(static_cast<cudaStream_t>(stream)));
}

int lisa_attn_stream_synchronize(void* stream) {
  return st(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
}

int lisa_attn_event_create(int device, int timing, void** event) {
  if (!event) return LISA_EINVAL;
  *event = nullptr;
  int s = set_device(device);
  if (s != LISA_OK) return s;
  cudaEvent_t e = nullptr;
  s = st(cudaEventCreateWithFlags(&e, timing ? cudaEventDefault : cudaEventDisableTiming));
  *event = e;
  return s;
}

int lisa_attn_event_destroy(void* event) {
  if (!event) return LISA_EINVAL;
  return st(cudaEventDestroy(static_cast<cudaEvent_t>(event)));
}

int lisa_attn_event_record(void* event, void* stream) {
  if (!event) return LISA_EINVAL;
  return st(cudaEventRecord(static_cast<cudaEvent_t>(event), static_cast<cudaStream_t>(stream)));
}

int lisa_attn_stream_wait_event(void* stream, void* event) {
  if (!event) return LISA_EINVAL;
  return st(cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), static_cast<cudaEvent_t>(event), 0));
}

int lisa_attn_event_synchronize(void* event) {
  if (!event) return LISA_EINVAL;
  return st(cudaEventSynchronize(static_cast<cudaEvent_t>(event)));
}

int lisa_attn_event_elapsed_ms(void* start, void* end, float* ms) {
  if (!start || !end || !ms) return LISA_EINVAL;
  return st(cudaEventElapsedTime(ms, static_cast<cudaEvent_t>(start), static_cast<cudaEvent_t>(end)));
}

int lisa_attn_copy_h2d(void* dst, const void* src, size_t bytes, void* stream) {
  if ((!dst || !src) && bytes) return LISA_EINVAL;
  return st(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream)));
}

int lisa_attn_copy_d2h(void* dst, const void* src, size_t bytes, void* stream) {
  if ((!dst || !src) && bytes) return LISA_EINVAL;
  return st(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, static_cast<cudaStream_t>(stream)));
}

int lisa_attn_copy_d2d(void* dst, const void* src, size_t bytes, void* stream) {
  if ((!dst || !src) && bytes) return LISA_EINVAL;
  return st(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream)));
}

int lisa_attn_memset(void* dst, int value, size_t bytes, void* stream) {
  if (!dst && bytes) return LISA_EINVAL;
  return st(cudaMemsetAsync(dst, value, bytes, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
#pragma GCC visibility pop
