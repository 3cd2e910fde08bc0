// Allocation-free decode attention: jsx_attn_decode_noalloc.
//
// Some callers cannot call cudaMalloc at all: code that runs while a CUDA
// graph is being captured for a framework that forbids allocation inside
// capture, embedded runtimes with a fixed memory budget reserved at start-up,
// or FFI hosts (an XLA custom call without a scratch operand, for instance)
// that give a kernel only its inputs and outputs.  For them this entry point
// runs the same split-context attention kernel as jsx_attn_decode, with the
// split partials kept in a static device array of this file instead of a
// caller-provided workspace.
//
// Limits and sharing:
//  * the array holds kNoAllocScratchBytes (16 MiB); every GPU that loads the
//    library keeps it until the process exits.  A shape whose workspace would
//    exceed it is rejected with JSX_EINVAL (jsx_attn_decode_workspace_size
//    gives the requirement);
//  * every call on a device shares the one array and it keeps the previous
//    call's contents: each call clears the per-sequence counters the kernel
//    needs at zero (an async memset on the caller's stream, not an
//    allocation).  Calls that overlap on the GPU — on different streams, or
//    from several host threads without ordering — race on the array;
//  * the first call on each device looks up the array's device address with
//    cudaGetSymbolAddress (with that device current) and caches it; make that
//    first call before any stream capture begins.  The cached address belongs
//    to the device's primary context: after cudaDeviceReset (or anything else
//    that destroys and recreates that context) the module is loaded again, the
//    array may move, and this entry point must not be called again in the
//    process;
//  * a call whose arguments are rejected returns before it touches the array.
#include <mutex>

#include "attn_core.cuh"
#include "common.cuh"

namespace jsx {

int attn_decode_check(const void* q, const void* k_cache, const void* v_cache, const void* out,
                      const int32_t* positions, int B, int nq, int nkv, int head_dim, int max_seq);  // attention.cu

constexpr size_t kNoAllocScratchBytes = (size_t)16 << 20;
constexpr int kMaxDevices = 128;

static __device__ __align__(256) unsigned char g_attn_scratch[kNoAllocScratchBytes];

// Device address of g_attn_scratch on `dev` (the current device), looked up once.
static int scratch_address(int dev, void** out) {
  static std::mutex mu;
  static void* addr[kMaxDevices] = {};
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
    if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(g_attn_scratch)");
    addr[dev] = p;
  }
  *out = addr[dev];
  return JSX_OK;
}

}  // namespace jsx

using namespace jsx;

extern "C" int jsx_attn_decode_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                       void* out, const int32_t* positions, int B, int nq, int nkv,
                                       int head_dim, int max_seq, float scale, void* stream) {
  // every argument check of jsx_attn_decode runs before the shared array is cleared
  int st = attn_decode_check(q, k_cache, v_cache, out, positions, B, nq, nkv, head_dim, max_seq);
  if (st != JSX_OK) return st;
  size_t need = 0;
  st = jsx_attn_decode_workspace_size(B, nq, nkv, head_dim, max_seq, &need);
  if (st != JSX_OK) return st;
  JSX_REQUIRE(need <= kNoAllocScratchBytes,
              "this shape needs %zu bytes of attention scratch; the static scratch holds %zu "
              "(use jsx_attn_decode with a caller workspace)",
              need, kNoAllocScratchBytes);
  int dev = 0;
  JSX_CUDA(cudaGetDevice(&dev));
  JSX_REQUIRE(dev >= 0 && dev < kMaxDevices, "device %d out of range", dev);
  void* ws = nullptr;
  const int sa = scratch_address(dev, &ws);
  if (sa != JSX_OK) return sa;
  // The header and the per-item-group counters open the jsx_attn_decode
  // workspace (attn_layout); they must be zero when the kernel starts.
  const size_t counters = attn_layout(B, nq, nkv, head_dim, max_seq).counter_bytes;
  JSX_CUDA(cudaMemsetAsync(ws, 0, counters, (cudaStream_t)stream));
  return jsx_attn_decode(q, k_cache, v_cache, out, positions, B, nq, nkv, head_dim, max_seq, scale,
                         ws, kNoAllocScratchBytes, stream);
}
