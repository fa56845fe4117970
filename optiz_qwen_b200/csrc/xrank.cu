// Cross-GPU log-sum-exp merge over NVLink peer memory, for the long-context decode whose KV
// range is split across the GPUs of one box.
//
// Every rank holds a receive buffer in its own HBM, mapped into the other ranks' address
// space with CUDA IPC (oq_ipc_export / oq_ipc_import; no multicast object is involved).  One
// call of oq_xrank_lse_merge per (layer, step) runs one CTA per rank that
//   1. stores this rank's partial (normalised fp32 output rows, then their natural-log LSE)
//      into slot [rank] of every rank's buffer with plain 16-byte stores over NVLink,
//   2. after a system-scope fence, raises flag [rank] of every rank to the call's epoch
//      (a release store),
//   3. polls its own flags until every rank's epoch has arrived (acquire loads, bounded:
//      OQ_DEV_TIMEOUT in the status word if a peer never arrives), and
//   4. merges the partials from its own buffer: out = sum_r exp(lse_r - m) o_r /
//      sum_r exp(lse_r - m), m = max_r lse_r -- the arithmetic of oq_lse_merge, in the same
//      order, so both exchange paths give the same bits.
// The epoch is a per-call-site counter in device memory that the kernel advances itself, so
// a captured CUDA graph replays correctly.  Slots and flags are double-buffered by epoch
// parity: a rank can be at most one call ahead of another at the same call site (it waits
// for every rank's flag of the previous call first), so it never overwrites a slot that is
// still being read.  No TMA or bulk copy touches peer memory; every peer access is a plain
// load or store.
//
// This replaces, per layer, the partial packing, the NCCL all-gather, the unpacking and the
// merge launch of the NCCL path (which stays available).  The reference decodes on one GPU
// and has no counterpart.
#include <cudaTypedefs.h>

#include <cmath>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace oq {
namespace {

struct XrankParams {
  const float* part_out;  // [rows, head_dim] this rank's partial
  const float* part_lse;  // [rows]
  int rows, head_dim;
  float* const* peers;    // [world] device pointers to every rank's buffer for this call site
  int rank, world;
  uint32_t* epoch;        // this call site's counter (device, this rank)
  void* out;              // [rows, head_dim] in `dtype`
  float* out_lse;         // [rows] or null
  int32_t* status;
  int64_t polls;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Buffer of one call site: slots [2 parities][world], each rows x head_dim output floats
// followed by rows LSE floats (padded to 16 bytes), then flags [2 parities][world] uint32.
__host__ __device__ inline int64_t slot_floats(int rows, int head_dim) {
  return (int64_t(rows) * (head_dim + 1) + 3) / 4 * 4;
}
__host__ __device__ inline int64_t flags_offset(int rows, int head_dim, int world) {
  return 2 * int64_t(world) * slot_floats(rows, head_dim);
}

template <typename T>
__global__ void __launch_bounds__(256) xrank_merge_kernel(XrankParams p) {
  const int tid = threadIdx.x;
  pdl_wait();
  const uint32_t e = *p.epoch + 1;
  const int par = int(e & 1);
  const int D = p.head_dim;
  const int64_t n = slot_floats(p.rows, D);
  const int64_t nv = int64_t(p.rows) * D / 4;  // float4 of output rows (head_dim % 4 == 0)
  // 1. this rank's partial into slot [par][rank] of every rank's buffer
  const float4* src = reinterpret_cast<const float4*>(p.part_out);
  for (int64_t i = tid; i < nv * p.world; i += blockDim.x) {
    const int q = int(i / nv);
    const int64_t j = i - int64_t(q) * nv;
    float4* dst = reinterpret_cast<float4*>(p.peers[q] + (int64_t(par) * p.world + p.rank) * n);
    dst[j] = src[j];
  }
  for (int i = tid; i < p.rows * p.world; i += blockDim.x) {
    const int q = i / p.rows, r = i - q * p.rows;
    p.peers[q][(int64_t(par) * p.world + p.rank) * n + int64_t(p.rows) * D + r] = p.part_lse[r];
  }
  __threadfence_system();
  __syncthreads();
  // 2. flag [par][rank] of every rank := epoch
  if (tid < p.world) {
    uint32_t* flags = reinterpret_cast<uint32_t*>(p.peers[tid] + flags_offset(p.rows, D, p.world));
    st_release_sys(flags + par * p.world + p.rank, e);
  }
  // 3. every rank's flag in this rank's own buffer: spin briefly, then back off to ~1 us polls
  bool ok = true;
  if (tid < p.world) {
    const uint32_t* flags = reinterpret_cast<const uint32_t*>(p.peers[p.rank] + flags_offset(p.rows, D, p.world));
    const uint32_t* f = flags + par * p.world + tid;
    ok = false;
    for (int64_t i = 0; i < p.polls; ++i) {
      if (ld_acquire_sys(f) == e) {
        ok = true;
        break;
      }
      if (i >= 256) __nanosleep(1000);
    }
  }
  const bool timed_out = __syncthreads_or(!ok);
  if (timed_out && tid == 0) report(p.status, OQ_DEV_TIMEOUT);
  // 4. merge (a warp per row, as oq_lse_merge)
  const float* slots = p.peers[p.rank] + int64_t(par) * p.world * n;
  const float* lse = slots + int64_t(p.rows) * D;
  const int lane = tid & 31;
  for (int row = tid >> 5; row < p.rows; row += blockDim.x >> 5) {
    float m = -INFINITY;
    for (int i = 0; i < p.world; ++i) m = fmaxf(m, __ldcg(lse + i * n + row));
    float denom = 0.0f;
    for (int i = 0; i < p.world; ++i) {
      const float l = __ldcg(lse + i * n + row);
      denom += (m == -INFINITY || l == -INFINITY) ? 0.0f : expf(l - m);
    }
    for (int d = lane; d < D; d += 32) {
      float acc = 0.0f;
      for (int i = 0; i < p.world; ++i) {
        const float l = __ldcg(lse + i * n + row);
        if (m == -INFINITY || l == -INFINITY) continue;
        acc += expf(l - m) * __ldcg(slots + i * n + int64_t(row) * D + d);
      }
      static_cast<T*>(p.out)[int64_t(row) * D + d] = from_float<T>(denom > 0.0f ? acc / denom : 0.0f);
    }
    if (p.out_lse != nullptr && lane == 0) p.out_lse[row] = denom > 0.0f ? m + logf(denom) : -INFINITY;
  }
  pdl_allow_next();
  __syncthreads();
  if (tid == 0) *p.epoch = e;
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
  if (rows <= 0 || head_dim <= 0 || world <= 0 || rows > (1 << 20) || head_dim > 4096 || world > 64) return 0;
  const int64_t floats = oq::flags_offset(int(rows), int(head_dim), int(world));
  return size_t((floats * 4 + 2 * world * 4 + 255) / 256 * 256);
}

extern "C" int oq_xrank_lse_merge(const float* part_out, const float* part_lse, int64_t rows, int64_t head_dim,
                                  float* const* peer_buffers, int rank, int world, uint32_t* epoch, void* out,
                                  int dtype, float* out_lse, int32_t* device_status, void* stream) {
  using namespace oq;
  if (!valid_dtype(dtype)) return fail(OQ_ERR_UNSUPPORTED, "xrank_lse_merge: unknown dtype %d", dtype);
  if (rows <= 0 || head_dim <= 0 || world <= 0 || rank < 0 || rank >= world || rows > (1 << 20) ||
      head_dim > 4096 || world > 64) {
    return fail(OQ_ERR_INVALID_ARGUMENT, "xrank_lse_merge: bad sizes");
  }
  if (head_dim % 4 != 0) return fail(OQ_ERR_UNSUPPORTED, "xrank_lse_merge: head_dim must be a multiple of 4");
  if (!part_out || !part_lse || !peer_buffers || !epoch || !out) {
    return fail(OQ_ERR_INVALID_ARGUMENT, "xrank_lse_merge: null pointer");
  }
  if (reinterpret_cast<uintptr_t>(part_out) % 16 != 0) {
    return fail(OQ_ERR_MISALIGNED, "xrank_lse_merge: part_out must be 16-byte aligned");
  }
  XrankParams p;
  p.part_out = part_out;
  p.part_lse = part_lse;
  p.rows = int(rows);
  p.head_dim = int(head_dim);
  p.peers = peer_buffers;
  p.rank = rank;
  p.world = world;
  p.epoch = epoch;
  p.out = out;
  p.out_lse = out_lse;
  p.status = device_status;
  // ~1 us per poll after the first 256: the same ~2 s bound (and the same test hook) as the copy waits
  p.polls = int64_t(wait_polls()) * 20;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case OQ_F32: launch_pdl(xrank_merge_kernel<float>, dim3(1), dim3(256), 0, s, p); break;
    case OQ_F16: launch_pdl(xrank_merge_kernel<__half>, dim3(1), dim3(256), 0, s, p); break;
    default: launch_pdl(xrank_merge_kernel<__nv_bfloat16>, dim3(1), dim3(256), 0, s, p); break;
  }
  return check_launch("xrank_lse_merge");
}
