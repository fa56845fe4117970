// Cross-GPU log-sum-exp merge over NVLink peer memory, for the long-context decode whose KV
// range is split across the GPUs of one box: the standalone form, one CTA per output row,
// for partials that an earlier kernel wrote to global memory.  The protocol and the buffer
// layout are in xrank.cuh; the long-context attention's split merge runs the same exchange
// in-kernel.  Also here: the CUDA IPC export / import of the receive buffers.
//
// This replaces, per layer, the partial packing, the NCCL all-gather, the unpacking and the
// merge launch of the NCCL path (which stays available).  The reference decodes on one GPU
// and has no counterpart.
#include <cudaTypedefs.h>

#include <cmath>
#include <cstring>
#include <mutex>

#include "xrank.cuh"

namespace oq {
namespace {

struct XrankParams {
  const float* part_out;  // [rows, head_dim] this rank's partial
  const float* part_lse;  // [rows]
  XrankLayout L;
  XrankArgs x;
  void* out;              // [rows, head_dim] in `dtype`
  float* out_lse;         // [rows] or null
  int32_t* status;
};

template <typename T>
__global__ void __launch_bounds__(256) xrank_merge_kernel(XrankParams p) {
  const int row = blockIdx.x;
  const int D = p.L.head_dim;
  pdl_wait();  // (the previous call at this site may be the kernel just ahead of this one)
  const uint32_t e = xrank_epoch(p.L, p.x, row);
  for (int d = threadIdx.x; d < D; d += blockDim.x) xrank_put(p.L, p.x, row, e, d, p.part_out[int64_t(row) * D + d]);
  if (threadIdx.x == 0) xrank_put(p.L, p.x, row, e, D, p.part_lse[row]);
  pdl_allow_next();
  for (int d0 = 0; d0 < D; d0 += blockDim.x) {
    const int d = d0 + threadIdx.x;
    float lse;
    const float o = xrank_merge(p.L, p.x, row, e, d, p.status, &lse);
    if (d < D) static_cast<T*>(p.out)[int64_t(row) * D + d] = from_float<T>(o);
    if (p.out_lse != nullptr && d == 0) p.out_lse[row] = lse;
  }
}

using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

AddressRangeFn address_range_fn() {
  static AddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<AddressRangeFn>(ptr);
    }
  });
  return fn;
}

}  // namespace
}  // namespace oq

extern "C" size_t oq_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int oq_ipc_export(const void* ptr, void* handle, int64_t* offset) {
  using namespace oq;
  if (!ptr || !handle || !offset) return fail(OQ_ERR_INVALID_ARGUMENT, "ipc_export: null pointer");
  auto fn = address_range_fn();
  if (fn == nullptr) return fail(OQ_ERR_CUDA, "ipc_export: cuMemGetAddressRange is not available from the driver");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) {
    return fail(OQ_ERR_CUDA, "ipc_export: pointer is not in a device allocation");
  }
  cudaIpcMemHandle_t h;
  const cudaError_t err = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (err != cudaSuccess) return fail(OQ_ERR_CUDA, "ipc_export: cudaIpcGetMemHandle: %s", cudaGetErrorString(err));
  memcpy(handle, &h, sizeof(h));
  *offset = int64_t(reinterpret_cast<uintptr_t>(ptr) - uintptr_t(base));
  return ok();
}

extern "C" int oq_ipc_import(const void* handle, int64_t offset, void** ptr) {
  using namespace oq;
  if (!handle || !ptr || offset < 0) return fail(OQ_ERR_INVALID_ARGUMENT, "ipc_import: bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  const cudaError_t err = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (err != cudaSuccess) return fail(OQ_ERR_CUDA, "ipc_import: cudaIpcOpenMemHandle: %s", cudaGetErrorString(err));
  *ptr = static_cast<uint8_t*>(base) + offset;
  return ok();
}

extern "C" int oq_ipc_close(void* ptr, int64_t offset) {
  using namespace oq;
  if (!ptr || offset < 0) return fail(OQ_ERR_INVALID_ARGUMENT, "ipc_close: bad argument");
  const cudaError_t err = cudaIpcCloseMemHandle(static_cast<uint8_t*>(ptr) - offset);
  if (err != cudaSuccess) return fail(OQ_ERR_CUDA, "ipc_close: cudaIpcCloseMemHandle: %s", cudaGetErrorString(err));
  return ok();
}

extern "C" size_t oq_xrank_buffer_bytes(int64_t rows, int64_t head_dim, int64_t world) {
  if (rows <= 0 || head_dim <= 0 || world <= 0 || rows > (1 << 20) || head_dim > 4096 ||
      world > oq::kXrankMaxWorld) {
    return 0;
  }
  const oq::XrankLayout L{int(rows), int(head_dim), int(world)};
  return size_t((L.total_bytes() + 255) / 256 * 256);
}

extern "C" int oq_xrank_lse_merge(const float* part_out, const float* part_lse, int64_t rows, int64_t head_dim,
                                  float* const* peer_buffers, int rank, int world, void* out, int dtype,
                                  float* out_lse, int32_t* device_status, void* stream) {
  using namespace oq;
  if (!valid_dtype(dtype)) return fail(OQ_ERR_UNSUPPORTED, "xrank_lse_merge: unknown dtype %d", dtype);
  if (rows <= 0 || head_dim <= 0 || world <= 0 || rank < 0 || rank >= world || rows > (1 << 20) ||
      head_dim > 4096 || world > kXrankMaxWorld) {
    return fail(OQ_ERR_INVALID_ARGUMENT, "xrank_lse_merge: bad sizes");
  }
  if (!part_out || !part_lse || !peer_buffers || !out) {
    return fail(OQ_ERR_INVALID_ARGUMENT, "xrank_lse_merge: null pointer");
  }
  XrankParams p;
  p.part_out = part_out;
  p.part_lse = part_lse;
  p.L = XrankLayout{int(rows), int(head_dim), world};
  p.x = XrankArgs{peer_buffers, rank, world, xrank_polls()};
  p.out = out;
  p.out_lse = out_lse;
  p.status = device_status;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case OQ_F32: launch_pdl(xrank_merge_kernel<float>, dim3(unsigned(rows)), dim3(256), 0, s, p); break;
    case OQ_F16: launch_pdl(xrank_merge_kernel<__half>, dim3(unsigned(rows)), dim3(256), 0, s, p); break;
    default: launch_pdl(xrank_merge_kernel<__nv_bfloat16>, dim3(unsigned(rows)), dim3(256), 0, s, p); break;
  }
  return check_launch("xrank_lse_merge");
}
