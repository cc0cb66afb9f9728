// Allocation-free forward entry point.
//
// gdn2_fwd needs caller-allocated scratch: the residual buffer (scores, WY inverse, wp, per-chunk
// states, v_new) and the forward workspace (u, state-transition images).  Some callers cannot
// allocate device memory at the point where they run the operator: plugin and custom-call hooks of inference runtimes and
// compilers (TensorRT plugin enqueue, XLA custom calls declared without a scratch operand) run
// under an allocator that owns the device's memory plan, so a cudaMalloc there can fail, stall
// against that allocator or break the plan, and code that only receives a stream and its
// input/output pointers has nothing to put scratch in.  gdn2_fwd_noalloc serves them: the same
// three forward kernels, with the scratch in one file-scope device array of fixed size.
#include <mutex>

#include "gdn2_kernels.cuh"

namespace {

// Maximum scratch: 64 MiB, enough for the residual plus the forward workspace of B*H*L/128 <= 96
// chunk-heads in the default modes (e.g. B=1, H=6, L=2048).  Every GPU that loads the library
// holds this array until exit.
constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device, looked up once per device.  In host
// code the array's name is only a host-side stand-in, so the address must come from
// cudaGetSymbolAddress with the device current.  The cached address belongs to the device's
// primary context: after cudaDeviceReset (or any other teardown of that context) the module is
// loaded again at a new address, so this entry point must not be used across such a reset.
gdn2_status noalloc_scratch(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return GDN2_ERR_CUDA;
  std::lock_guard<std::mutex> g(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return GDN2_ERR_CUDA;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return GDN2_OK;
}

}  // namespace

extern "C" gdn2_status gdn2_fwd_noalloc(const gdn2_desc* d, const void* q, const void* k, const void* v,
                                        const void* w, const void* b, const void* g, const float* h0, float* o,
                                        float* h_final, uint32_t* dev_status, void* stream) {
  const gdn2_status ds = gdn2::check_desc(d);  // same answer as gdn2_fwd for a rejected descriptor
  if (ds != GDN2_OK) return ds;
  const size_t res_bytes = gdn2::align256(gdn2_residual_bytes(d));
  const size_t need = res_bytes + gdn2_fwd_workspace_bytes(d);
  if (res_bytes == 0 || need > kNoAllocScratchBytes) return GDN2_ERR_INVALID_ARGUMENT;
  void* scratch = nullptr;
  const gdn2_status s = noalloc_scratch(&scratch);
  if (s != GDN2_OK) return s;
  // Every scratch region is written by the kernels before it is read, so stale contents from a
  // previous call need no clearing.
  // The residual and the forward workspace both live in the scratch array (the residual first).
  return gdn2_fwd(d, q, k, v, w, b, g, h0, o, h_final, scratch, static_cast<uint8_t*>(scratch) + res_bytes,
                  dev_status, stream);
}
