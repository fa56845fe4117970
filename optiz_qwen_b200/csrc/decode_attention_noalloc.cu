// Decode attention for callers that cannot allocate device memory.
//
// oq_decode_attn_int4_paged needs a caller-provided workspace for its split-KV
// partials and merge counters.  Some callers cannot call cudaMalloc to get
// one: a decode loop embedded in a host runtime whose own arena owns all of the
// device memory, or a foreign-language caller that only holds buffers somebody
// else allocated and has no allocator to ask.  This entry point takes its
// scratch from a fixed array compiled into the library instead.
//
// The array is kNoAllocScratchBytes (8 MiB) of device memory on every GPU that
// loads the library, held until the process exits.  All calls share it, and it
// keeps the last call's contents: the merge counters are cleared (with an
// asynchronous memset on the caller's stream) at the start of every call, and
// calls that overlap on the GPU -- on different streams, or from several host
// threads -- race on it.  The first call on a device looks up the array's
// device address (cudaGetSymbolAddress) with that device current; make that
// first call before any stream capture.
#include <algorithm>
#include <mutex>

#include "decode_attention.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (looked up once per device).
int scratch_for_current_device(void** out) {
  int dev = -1;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return oq::fail(OQ_ERR_CUDA, "decode_attn_noalloc: cudaGetDevice: %s", cudaGetErrorString(err));
  if (dev < 0 || dev >= kMaxDevices) return oq::fail(OQ_ERR_UNSUPPORTED, "decode_attn_noalloc: device %d", dev);
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (err != cudaSuccess || ptr == nullptr) {
      return oq::fail(OQ_ERR_CUDA, "decode_attn_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(err));
    }
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return OQ_OK;
}

}  // namespace

extern "C" int oq_decode_attn_int4_paged_noalloc(
    const void* query, int dtype, int64_t query_stride_b, int64_t query_stride_h,
    const uint8_t* kv_codes, const uint16_t* kv_meta, int64_t num_pages, int64_t page_size,
    const int32_t* block_table, int64_t block_table_stride, int64_t max_pages_per_seq,
    const int32_t* seq_lens,
    int64_t batch, int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
    float scaling,
    void* out, int64_t out_stride_b, int64_t out_stride_h,
    float* out_f32, float* out_lse,
    int num_splits, int32_t* device_status, void* stream) {
  using namespace oq;
  if (batch <= 0 || num_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || max_pages_per_seq <= 0 ||
      num_heads % num_kv_heads != 0) {
    // let the regular entry point report the precise problem (it launches nothing for these)
    return oq_decode_attn_int4_paged(query, dtype, query_stride_b, query_stride_h, kv_codes, kv_meta, num_pages,
                                     page_size, block_table, block_table_stride, max_pages_per_seq, seq_lens, batch,
                                     num_heads, num_kv_heads, head_dim, scaling, out, out_stride_b, out_stride_h,
                                     out_f32, out_lse, nullptr, 0, 1, device_status, stream);
  }
  // Split count: the one oq_decode_attn_int4_paged would launch with (the same heuristic and
  // clamps), so both entry points run the same partition whenever its scratch fits; in auto
  // mode a partition that does not fit is halved until it does.
  const int64_t group = num_heads / num_kv_heads;
  int splits = decode_attn_plan(4, dtype, group, batch, num_kv_heads, max_pages_per_seq, num_splits, nullptr);
  if (num_splits <= 0) {
    while (splits > 1 && oq_decode_attn_workspace_bytes(batch, num_heads, num_kv_heads, head_dim, splits) >
                             kNoAllocScratchBytes) {
      splits = decode_attn_plan(4, dtype, group, batch, num_kv_heads, max_pages_per_seq, std::max(1, splits / 2),
                                nullptr);
    }
  } else if (splits > 1) {
    const size_t need = oq_decode_attn_workspace_bytes(batch, num_heads, num_kv_heads, head_dim, splits);
    if (need > kNoAllocScratchBytes) {
      return fail(OQ_ERR_WORKSPACE,
                  "decode_attn_noalloc: %d splits need %zu bytes of scratch; the library's fixed scratch holds %zu "
                  "(use fewer splits, or oq_decode_attn_int4_paged with your own workspace)",
                  splits, need, kNoAllocScratchBytes);
    }
  }
  void* scratch = nullptr;
  int st = scratch_for_current_device(&scratch);
  if (st != OQ_OK) return st;
  // merge counters must start at zero: clear them on the caller's stream
  const size_t counters = size_t((batch * num_kv_heads * int64_t(sizeof(int)) + 255) / 256 * 256);
  cudaError_t err = cudaMemsetAsync(scratch, 0, std::min(counters, kNoAllocScratchBytes),
                                    static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return fail(OQ_ERR_CUDA, "decode_attn_noalloc: clearing scratch: %s", cudaGetErrorString(err));
  return oq_decode_attn_int4_paged(query, dtype, query_stride_b, query_stride_h, kv_codes, kv_meta, num_pages,
                                   page_size, block_table, block_table_stride, max_pages_per_seq, seq_lens, batch,
                                   num_heads, num_kv_heads, head_dim, scaling, out, out_stride_b, out_stride_h,
                                   out_f32, out_lse, scratch, kNoAllocScratchBytes, splits, device_status, stream);
}
