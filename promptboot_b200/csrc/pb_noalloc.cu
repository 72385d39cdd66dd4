// pb_qmatvec_device_noalloc: the block-scaled matvec operator without any
// device allocation.
//
// pb_qmatvec_device needs scratch for the Q8_0-quantized activations and the
// per-row stage-error words, and allocates it on every call.  Some callers
// cannot do that: a host that gives this library a fixed share of device
// memory owned by its own allocator (a framework's caching allocator, a
// serving runtime's arena), where an extra cudaMalloc can fail or fragment
// that budget; a latency-critical loop that must not pay cudaMalloc/cudaFree
// and the device-wide synchronisation they can imply; and integrations built
// the way promptboot itself is, whose firmware runtime only ever works out of
// fixed, pre-sized arenas and never allocates on the token path.  This entry
// point serves them from one file-scope device array instead.
//
// Limits and rules:
//  * at most kNoAllocMaxRows activation rows per call (columns <= 4864); larger
//    requests are rejected with PB_CAPACITY and a message in
//    pb_last_error_string(); nothing is launched for them;
//  * the array (192 KiB) is held by every GPU that loads the library until the
//    process exits;
//  * the first call on a device (with that device current) looks up the
//    array's device address and sets the kernels' shared-memory attribute;
//    make that first call before any stream capture;
//  * every call shares the one array and overwrites it: calls that overlap on
//    the GPU (other streams, other threads) race and must be serialised by the
//    caller.
// There is no counterpart in the reference (which has no GPU path).
#include "pb_common.cuh"
#include "pb_host.h"
#include "pb_kernels.cuh"

#include <mutex>

namespace {

constexpr uint32_t kNoAllocMaxRows = 32;
constexpr size_t kAqBytes = (size_t)kNoAllocMaxRows * pb::kActStride;         // int8 quants
constexpr size_t kAdBytes = (size_t)kNoAllocMaxRows * pb::kActBlocks * 4;     // f32 scales
constexpr size_t kAsumBytes = (size_t)kNoAllocMaxRows * pb::kActBlocks * 4;   // int32 block sums
constexpr size_t kErrBytes = (size_t)kNoAllocMaxRows * 8;                     // stage-error words
constexpr size_t kAdOffset = kAqBytes;
constexpr size_t kAsumOffset = kAdOffset + kAdBytes;
constexpr size_t kErrOffset = kAsumOffset + kAsumBytes;
constexpr size_t kScratchBytes = kErrOffset + kErrBytes;
static_assert(kAdOffset % 256 == 0 && kAsumOffset % 256 == 0 && kErrOffset % 256 == 0,
              "scratch regions stay 256-byte aligned");

// In host code this name is only a host-side stand-in for the array; kernels
// receive the device address obtained with cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_lock;
void* g_scratch_address[kMaxDevices] = {};

// Once per device, with that device current.
uint32_t scratch_for_current_device(uint8_t** out) {
  int device = 0;
  PB_CUDA(cudaGetDevice(&device));
  if (device < 0 || device >= kMaxDevices) {
    pb::set_last_error("pb_qmatvec_device_noalloc: device ordinal out of range");
    return PB_CAPACITY;
  }
  std::lock_guard<std::mutex> guard(g_setup_lock);
  if (!g_scratch_address[device]) {
    void* address = nullptr;
    PB_CUDA(cudaGetSymbolAddress(&address, g_noalloc_scratch));
    pb::init_kernel_attributes();
    PB_CUDA(cudaGetLastError());
    g_scratch_address[device] = address;
  }
  *out = static_cast<uint8_t*>(g_scratch_address[device]);
  return PB_OK;
}

}  // namespace

extern "C" uint32_t pb_qmatvec_device_noalloc(uint32_t wtype, const uint8_t* w, uint32_t rows,
                                              uint32_t cols, const float* x, uint32_t batch,
                                              float* y, void* stream) {
  const uint32_t nb = cols / 32;
  const uint32_t rt = nb > 64 ? 8 : 32;
  if (batch == 0 || batch > kNoAllocMaxRows) {
    pb::set_last_error("pb_qmatvec_device_noalloc: batch must be 1..32 rows (fixed scratch)");
    return PB_CAPACITY;
  }
  if ((wtype != pb::W_Q4_0 && wtype != pb::W_Q8_0) || cols == 0 || cols % 32 ||
      cols > (uint32_t)pb::kFfn || rows == 0 || rows % rt) {
    pb::set_last_error("pb_qmatvec_device_noalloc: unsupported weight type or shape");
    return PB_CAPACITY;
  }
  uint8_t* scratch = nullptr;
  uint32_t st = scratch_for_current_device(&scratch);
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto* err = reinterpret_cast<unsigned long long*>(scratch + kErrOffset);
  // The error words must start "clear" (all ones) on every call.
  PB_CUDA(cudaMemsetAsync(err, 0xff, (size_t)batch * 8, s));
  pb::Batch b{};
  b.rows = (int)batch;
  b.aq = reinterpret_cast<int8_t*>(scratch);
  b.ad = reinterpret_cast<float*>(scratch + kAdOffset);
  b.asum = reinterpret_cast<int*>(scratch + kAsumOffset);
  b.err = err;
  pb::launch_quant(b, x, cols, (int)cols, s);
  pb::Epilogue ep{pb::EPI_STORE, y, rows, nullptr, err, 0, 0};
  pb::launch_qgemv((int)wtype, w, (int)rows, (int)cols, b, ep, s);
  PB_CUDA(cudaGetLastError());
  return PB_OK;
}
