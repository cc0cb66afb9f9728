// Allocation-free forward entry point.
//
// gdn2_fwd needs a caller-allocated residual buffer as scratch (scores, WY inverse, wp / u,
// state-transition images, per-chunk states).  Some callers cannot allocate device memory at the
// point where they run the operator: plugin and custom-call hooks of inference runtimes and
// compilers (TensorRT plugin enqueue, XLA custom calls declared without a scratch operand) run
// under an allocator that owns the device's memory plan, so a cudaMalloc there can fail, stall
// against that allocator or break the plan, and code that only receives a stream and its
// input/output pointers has nothing to put scratch in.  gdn2_fwd_noalloc serves them: the same
// three forward kernels, with the scratch in one file-scope device array of fixed size.
#include <mutex>

#include "gdn2_kernels.cuh"

namespace {

// Maximum scratch: 64 MiB, enough for B*H*L/128 <= 96 chunk-heads in the default modes
// (e.g. B=1, H=6, L=2048).  Every GPU that loads the library holds this array until exit.
constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device, looked up once per device.  In host
// code the array's name is only a host-side stand-in, so the address must come from
// cudaGetSymbolAddress with the device current.
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
  const size_t need = gdn2_residual_bytes(d);  // 0 for an invalid descriptor
  if (need == 0 || need > kNoAllocScratchBytes) return GDN2_ERR_INVALID_ARGUMENT;
  void* scratch = nullptr;
  const gdn2_status s = noalloc_scratch(&scratch);
  if (s != GDN2_OK) return s;
  // Every scratch region is written by the kernels before it is read, so stale contents from a
  // previous call need no clearing.
  return gdn2_fwd(d, q, k, v, w, b, g, h0, o, h_final, scratch, dev_status, stream);
}
