// Shared device primitives for the GDN-2 sm_100a kernels.
//
// Everything here is hand-written inline PTX for Blackwell (sm_100a):
//   * mbarrier waits that always terminate (bounded by a cycle budget and
//     recorded in a device status word instead of spinning forever),
//   * tcgen05 tensor-memory allocation, loads and stores,
//   * tcgen05.mma issue (kind::tf32 and kind::f16 with bf16 operands),
//   * shared-memory operand tiles in the canonical no-swizzle ("interleave")
//     UMMA layouts, K-major and MN-major, filled by threads from fp32 values
//     split into hi/lo parts for the multi-pass precision modes.
//
// Conventions used by every kernel in this directory:
//   * a CTA has 128 threads (4 warps); thread t owns TMEM lane t, i.e. row t of
//     every 128-row accumulator ("row owner");
//   * T (chunk length) = D (head dim) = 128;
//   * all accumulators are fp32 in TMEM, 128 lanes x N columns.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include "../../include/gdn2_b200.h"

namespace gdn2 {

constexpr int kT = 128;        // chunk length (tokens per chunk)
constexpr int kD = 128;        // head dimension (d_k = d_v)
constexpr int kThreads = 128;  // threads per CTA

// Device status bits (OR-ed into the caller's status word).
constexpr unsigned kStatusTimeout = 1u;      // an mbarrier wait hit its cycle budget
constexpr unsigned kStatusPositiveGate = 4u; // g > 0 seen (outside domain I-1)

// ~4 s at 2 GHz: far beyond any legitimate wait in these kernels.
constexpr long long kWaitCycles = 8LL * 1000 * 1000 * 1000;

// ---------------------------------------------------------------------------
// Precision modes (runtime): fmt = operand element type on the tensor core,
// passes = 1 (hi*hi) or 3 (hi*hi + hi*lo + lo*hi).
// ---------------------------------------------------------------------------
enum Fmt : int { kBF16 = 0, kTF32 = 1 };

struct Mode {
  int fmt;     // kBF16 / kTF32
  int passes;  // 1 or 3
};

__host__ __device__ inline Mode mode_from_enum(int m) {
  // gdn2_precision: HIGHEST = 3 x tf32, BF16X3 = 3 x bf16, DEFAULT = 1 x bf16, TF32 = 1 x tf32
  switch (m) {
    case GDN2_PREC_HIGHEST: return Mode{kTF32, 3};
    case GDN2_PREC_BF16X3: return Mode{kBF16, 3};
    case GDN2_PREC_TF32: return Mode{kTF32, 1};
    default: return Mode{kBF16, 1};
  }
}

// ---------------------------------------------------------------------------
// Small helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ float sanitize(float x, float clip) {
  // nan -> 0, +-inf -> +-clip, otherwise clamp to [-clip, clip]
  if (x != x) return 0.0f;
  return fminf(fmaxf(x, -clip), clip);
}

__device__ __forceinline__ float ex(float x) { return __expf(x); }

__device__ __forceinline__ uint32_t tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <class T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

// Load 4 consecutive input elements (16 B for fp32, 8 B for bf16) as fp32.
__device__ __forceinline__ void ld4(const float* p, float v[4]) {
  float4 x = __ldg(reinterpret_cast<const float4*>(p));
  v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
}
__device__ __forceinline__ void ld4(const __nv_bfloat16* p, float v[4]) {
  uint2 x = __ldg(reinterpret_cast<const uint2*>(p));
  __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&x.x);
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&x.y);
  float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
  v[0] = fa.x; v[1] = fa.y; v[2] = fb.x; v[3] = fb.y;
}
// 16-byte asynchronous copy global -> shared (no registers; completion by cp_async_wait_all).
__device__ __forceinline__ void cp_async16(void* dst_smem, const void* src_gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst_smem)), "l"(src_gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// Hint: bring `bytes` (a multiple of 16, 16-byte aligned start) of global memory into L2.
__device__ __forceinline__ void l2_prefetch(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
__device__ __forceinline__ float ld1(const float* p) { return __ldg(p); }
__device__ __forceinline__ float ld1(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ void st4(float* p, const float v[4]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
__device__ __forceinline__ void st4(__nv_bfloat16* p, const float v[4]) {
  uint2 x;
  x.x = pack_bf16(v[0], v[1]);
  x.y = pack_bf16(v[2], v[3]);
  *reinterpret_cast<uint2*>(p) = x;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for the phase with the given parity to complete; never spins forever: after `limit` SM
// cycles the wait gives up, sets the timeout bit of the caller's status word and returns false.
// Once any wait of the call has given up (the bit is set), later waits give up at once, so that a
// call whose waits cannot complete ends after one limit instead of one limit per wait.
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, unsigned* status, long long limit) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 1023u) == 0 && (*reinterpret_cast<volatile unsigned*>(status) & kStatusTimeout)) return false;
    if (clock64() - t0 > limit) {
      atomicOr(status, kStatusTimeout);
      return false;
    }
  }
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned* status) {
  return mbar_wait_for(bar, parity, status, kWaitCycles);
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// 1-D bulk copy global -> shared, completion signalled on an mbarrier (tx bytes).
// Both addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Make this thread's generic-proxy shared-memory writes visible to the async proxy
// (tensor core operand reads).
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM management, fences, loads/stores
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {  // whole warp
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Lane base address for the calling warp: warp w of the CTA reads lanes [32(w%4), 32(w%4)+32).
__device__ __forceinline__ uint32_t tmem_lane_base(uint32_t tbase) {
  const uint32_t w = (threadIdx.x >> 5) & 3;
  return tbase + ((w * 32u) << 16);
}

// Load 32 consecutive fp32 columns of this thread's lane (row) starting at column col.
__device__ __forceinline__ void tmem_ld32(uint32_t tbase, uint32_t col, float v[32]) {
  uint32_t r[32];
  const uint32_t a = tmem_lane_base(tbase) + col;
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(a));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Load 16 consecutive fp32 columns of this thread's lane (row) starting at column col.
__device__ __forceinline__ void tmem_ld16(uint32_t tbase, uint32_t col, float v[16]) {
  uint32_t r[16];
  const uint32_t a = tmem_lane_base(tbase) + col;
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(a));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Store 16 consecutive fp32 columns into this thread's lane.
__device__ __forceinline__ void tmem_st16(uint32_t tbase, uint32_t col, const float v[16]) {
  uint32_t r[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(v[i]);
  const uint32_t a = tmem_lane_base(tbase) + col;
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(a),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Store 32 consecutive fp32 columns into this thread's lane.
__device__ __forceinline__ void tmem_st32(uint32_t tbase, uint32_t col, const float v[32]) {
  uint32_t r[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(v[i]);
  const uint32_t a = tmem_lane_base(tbase) + col;
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(a),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Raise a kernel's dynamic shared-memory limit once per device (the attribute persists), so that
// launches made while a stream is being captured into a CUDA graph issue no attribute calls.
// `done` is a per-kernel bit mask of devices already set up.
template <class Kernel>
inline cudaError_t smem_attr_once(Kernel kernel, int bytes, unsigned long long& done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = 1ull << (dev & 63);
  if (done & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done |= bit;
  return e;
}

// ---------------------------------------------------------------------------
// UMMA descriptors and issue
// ---------------------------------------------------------------------------
// Shared-memory matrix descriptor, no swizzle (canonical "interleave" layout).
//   bits [0,14): start >> 4, [16,30): LBO >> 4, [32,46): SBO >> 4, [46,48): version 1 (sm_100),
//   [61,64): layout type 0 = SWIZZLE_NONE.
__device__ __forceinline__ uint64_t sdesc(uint32_t start, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((start >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  return d;
}

// Instruction descriptor for kind::tf32 / kind::f16(bf16), fp32 accumulate, M = 128.
__device__ __forceinline__ uint32_t idesc(int fmt, int N, bool a_mn, bool b_mn, bool neg_a) {
  const uint32_t f = (fmt == kTF32) ? 2u : 1u;  // operand format: TF32 = 2, BF16 = 1
  uint32_t d = 0;
  d |= 1u << 4;                       // D format f32
  d |= f << 7;                        // A format
  d |= f << 10;                       // B format
  d |= (neg_a ? 1u : 0u) << 13;       // negate A
  d |= (a_mn ? 1u : 0u) << 15;        // A major: 0 = K, 1 = MN
  d |= (b_mn ? 1u : 0u) << 16;        // B major
  d |= (uint32_t)(N >> 3) << 17;      // N / 8
  d |= (uint32_t)(128 >> 4) << 24;    // M / 16
  return d;
}

__device__ __forceinline__ void mma_issue(int fmt, uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t id,
                                          uint32_t accumulate) {
  if (fmt == kTF32) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(id), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(id), "r"(accumulate)
        : "memory");
  }
}

// Arrive on an mbarrier once all previously issued MMAs of this thread have completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// ---------------------------------------------------------------------------
// Operand tiles in shared memory
// ---------------------------------------------------------------------------
// An operand tile holds one precision part (hi or lo) of an MMA operand with MN rows
// (M of A or N of B) and a K extent, in one of the canonical UMMA layouts.
//
//  K-major, no swizzle (core matrix = 8 rows x 16 bytes, 128 contiguous bytes):
//      byte(mn, kb) = (mn>>3)*sbo + (kb>>4)*128 + (mn&7)*16 + (kb&15)
//      lbo = 128 (next core along K), sbo = 8 * row_bytes (next 8-row group along MN);
//      one MMA K-step = 32 bytes of K = 2 cores -> start advances by 256.
//  MN-major bf16, no swizzle (core = 8 k-rows x 16 bytes of MN):
//      byte(mnb, k) = (mnb>>4)*128 + (k>>3)*lbo + (k&7)*16 + (mnb&15)
//      sbo = 128 (next core along MN), lbo = 8 * mn_bytes (next group of 8 k);
//      one MMA K-step = 16 k = 2 groups -> start advances by 2*lbo.
//  MN-major tf32: the only MN-major layout the tensor core accepts for 32-bit operands is
//      SWIZZLE_128B_BASE32B (descriptor layout type 1): atoms of 4 k-rows x 128 bytes
//      (32 elements of MN), the 32-byte chunk index inside each 128-byte row XOR-ed with
//      the row index mod 4.  Atoms: lbo = 512 (next 32 elements of MN), sbo = (MN/32)*512
//      (next 4 k-rows); one MMA K-step = 8 k = 2 atoms -> start advances by 2*sbo.
//      byte(mn, k) = (mn>>5)*512 + (k>>2)*sbo + (k&3)*128 + ((((mn>>3)&3) ^ (k&3))<<5) + (mn&7)*4
//
// A bf16 K-major tile with rows of R bytes read as MN-major is its transpose: same bytes,
// sbo_mn = 128 and lbo_mn = sbo_k.
struct Tile {
  uint32_t addr;   // shared-memory address of the tile
  uint32_t lbo;
  uint32_t sbo;
  uint32_t step;   // start-address advance per MMA K-step
  bool mn;         // MN-major?
  uint32_t ltype;  // descriptor layout type: 0 = no swizzle, 1 = 128B_BASE32B
};

// K-major tile whose K extent is `kbytes` per row.
__device__ __forceinline__ Tile tile_k(uint32_t addr, uint32_t kbytes) {
  return Tile{addr, 128u, 8u * kbytes, 256u, false, 0u};
}
// MN-major tile with MN extent of `mnbytes` (elements * element size) per k row.
// For tf32, mnbytes must be a multiple of 128 (MN a multiple of 32).
__device__ __forceinline__ Tile tile_mn(uint32_t addr, uint32_t mnbytes, int fmt) {
  if (fmt == kTF32) {
    const uint32_t sbo = (mnbytes >> 7) * 512u;
    return Tile{addr, 512u, sbo, 2u * sbo, true, 1u};
  }
  const uint32_t lbo = 8u * mnbytes;
  return Tile{addr, lbo, 128u, 2u * lbo, true, 0u};
}
// bf16 only: the transpose of a K-major tile with rows of `kbytes` bytes.
__device__ __forceinline__ Tile tile_k_as_mn(uint32_t addr, uint32_t kbytes) {
  const uint32_t lbo = 8u * kbytes;
  return Tile{addr, lbo, 128u, 2u * lbo, true, 0u};
}

__device__ __forceinline__ uint64_t tdesc(const Tile& t, int kstep) {
  return sdesc(t.addr + (uint32_t)kstep * t.step, t.lbo, t.sbo) | ((uint64_t)t.ltype << 61);
}

// One MMA with a compile-time operand kind.
template <int FMT>
__device__ __forceinline__ void mma_t(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t id, uint32_t accumulate) {
  if constexpr (FMT == kTF32) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(id), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(id), "r"(accumulate)
        : "memory");
  }
}

// Issue D (+)= A * B over `nsteps` MMA K-steps with the given number of precision passes.
// a[0]/b[0] are the hi parts, a[1]/b[1] the lo parts (used only when passes == 3).
// Descriptors are formed once; a K-step advances the 14-bit start-address field by step/16
// (shared-memory addresses stay below 256 KB, so the field never carries).  Small cross terms
// are accumulated first.
template <int FMT>
__device__ __forceinline__ void mma_tiles_t(int passes, uint32_t d_tmem, const Tile a[2], const Tile b[2], int N,
                                            int nsteps, bool neg_a, bool accumulate) {
  const uint32_t id = idesc(FMT, N, a[0].mn, b[0].mn, neg_a);
  const uint64_t ah = tdesc(a[0], 0), bh = tdesc(b[0], 0);
  const uint64_t ia = a[0].step >> 4, ib = b[0].step >> 4;
  uint32_t acc = accumulate ? 1u : 0u;
  if (passes == 3) {
    const uint64_t al = tdesc(a[1], 0), bl = tdesc(b[1], 0);
#pragma unroll 4
    for (int s = 0; s < nsteps; ++s) {
      mma_t<FMT>(d_tmem, ah + s * ia, bl + s * ib, id, acc);
      acc = 1u;
      mma_t<FMT>(d_tmem, al + s * ia, bh + s * ib, id, 1u);
    }
  }
#pragma unroll 4
  for (int s = 0; s < nsteps; ++s) {
    mma_t<FMT>(d_tmem, ah + s * ia, bh + s * ib, id, acc);
    acc = 1u;
  }
}
__device__ __forceinline__ void mma_tiles(int fmt, int passes, uint32_t d_tmem, const Tile a[2], const Tile b[2], int N,
                                          int nsteps, bool neg_a, bool accumulate) {
  if (fmt == kTF32) mma_tiles_t<kTF32>(passes, d_tmem, a, b, N, nsteps, neg_a, accumulate);
  else mma_tiles_t<kBF16>(passes, d_tmem, a, b, N, nsteps, neg_a, accumulate);
}

// --- writing operand values (one 16-byte piece at a time) -------------------
// K-major piece: 4 consecutive k (tf32) or 8 consecutive k (bf16) of row mn.
// MN-major piece: 4 consecutive mn (tf32) or 8 consecutive mn (bf16) of row k.
// `v` holds 4 (tf32) or 8 (bf16) fp32 values; hi and (if lo_addr != 0) lo parts are written.
// The operand format is a template parameter so that every index into the value arrays is a
// compile-time constant (the arrays stay in registers).
template <int FMT>
__device__ __forceinline__ void put_piece_t(uint32_t hi_addr, uint32_t lo_addr, const float* v) {
  uint32_t h[4], l[4];
  if constexpr (FMT == kTF32) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      h[i] = tf32_rna(v[i]);
      l[i] = tf32_rna(v[i] - __uint_as_float(h[i]));
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 hv = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      float2 hf = __bfloat1622float2(hv);
      __nv_bfloat162 lv = __floats2bfloat162_rn(v[2 * i] - hf.x, v[2 * i + 1] - hf.y);
      h[i] = *reinterpret_cast<uint32_t*>(&hv);
      l[i] = *reinterpret_cast<uint32_t*>(&lv);
    }
  }
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(hi_addr), "r"(h[0]), "r"(h[1]), "r"(h[2]), "r"(h[3])
               : "memory");
  if (lo_addr)
    asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(lo_addr), "r"(l[0]), "r"(l[1]), "r"(l[2]),
                 "r"(l[3])
                 : "memory");
}

// Byte offset of piece p (16-byte unit index along K) of row mn in a K-major tile.
__device__ __forceinline__ uint32_t koff(uint32_t mn, uint32_t p, uint32_t sbo) {
  return (mn >> 3) * sbo + p * 128u + (mn & 7u) * 16u;
}
// Byte offset of piece p (16-byte unit index along MN) of k-row k in an MN-major tile.
__device__ __forceinline__ uint32_t mnoff(const Tile& t, uint32_t k, uint32_t p) {
  if (t.ltype == 1u) {  // tf32, 128B_BASE32B swizzle; piece p covers mn = 4p .. 4p+3
    const uint32_t r = k & 3u;
    return (p >> 3) * 512u + (k >> 2) * t.sbo + r * 128u + ((((p >> 1) & 3u) ^ r) << 5) + (p & 1u) * 16u;
  }
  return p * 128u + (k >> 3) * t.lbo + (k & 7u) * 16u;
}

// Stage N fp32 values (N a multiple of the piece width) of operand row `mn` (K-major), starting at
// element k0 of the tile's K range.
template <int FMT, int N>
__device__ __forceinline__ void stage_krow_t(const Tile& hi, const Tile& lo, bool with_lo, uint32_t mn, int k0,
                                             const float* v) {
  constexpr int W = (FMT == kTF32) ? 4 : 8;
#pragma unroll
  for (int i = 0; i < N; i += W) {
    const uint32_t pc = (uint32_t)((k0 + i) / W);
    const uint32_t o = koff(mn, pc, hi.sbo);
    put_piece_t<FMT>(hi.addr + o, with_lo ? lo.addr + o : 0u, v + i);
  }
}
// Stage N values of k-row `k` (MN-major), starting at MN element m0.
template <int FMT, int N>
__device__ __forceinline__ void stage_mnrow_t(const Tile& hi, const Tile& lo, bool with_lo, uint32_t k, int m0,
                                              const float* v) {
  constexpr int W = (FMT == kTF32) ? 4 : 8;
#pragma unroll
  for (int i = 0; i < N; i += W) {
    const uint32_t pc = (uint32_t)((m0 + i) / W);
    const uint32_t o = mnoff(hi, k, pc);
    put_piece_t<FMT>(hi.addr + o, with_lo ? lo.addr + o : 0u, v + i);
  }
}

// Runtime-format wrappers (the selftest and the scan use them with constant sizes).
__device__ __forceinline__ void stage_krow(const Tile& hi, const Tile& lo, bool with_lo, int fmt, uint32_t mn,
                                           int k0, const float* v, int nvals) {
  for (int i = 0; i < nvals; i += 8) {
    if (fmt == kTF32) stage_krow_t<kTF32, 8>(hi, lo, with_lo, mn, k0 + i, v + i);
    else stage_krow_t<kBF16, 8>(hi, lo, with_lo, mn, k0 + i, v + i);
  }
}
__device__ __forceinline__ void stage_mnrow(const Tile& hi, const Tile& lo, bool with_lo, int fmt, uint32_t k,
                                            int m0, const float* v, int nvals) {
  for (int i = 0; i < nvals; i += 8) {
    if (fmt == kTF32) stage_mnrow_t<kTF32, 8>(hi, lo, with_lo, k, m0 + i, v + i);
    else stage_mnrow_t<kBF16, 8>(hi, lo, with_lo, k, m0 + i, v + i);
  }
}

// True when `st` is not being captured into a CUDA graph.  A failed query (the legacy stream
// while another thread captures in global mode) counts as capturing, and its error is cleared so
// that the launch's own error check does not report it.
inline bool stream_eager(cudaStream_t st) {
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cap) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  return cap == cudaStreamCaptureStatusNone;
}

// Programmatic dependent launch: the chunk and scan kernels are launched with programmatic stream
// serialization, which lets the hardware begin a launch before its predecessor in the stream has
// fully retired; each kernel's first instruction waits until that predecessor has completed and its
// writes are visible, so nothing is read early.
// No kernel triggers its dependents early: CTAs parked at the wait would hold SMs that the other
// batch group's stream uses to fill this kernel's wave tail (measured 3 % slower).
__device__ __forceinline__ void pdl_enter() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Launch `kern` with programmatic stream serialization (its body must begin with pdl_enter()).
// The same, at the device's greatest scheduling priority when `urgent` (pending CTAs of urgent
// launches are dispatched ahead of other streams' pending CTAs).
template <class... KArgs, class... Args>
static inline cudaError_t launch_pdl_prio(void (*kern)(KArgs...), unsigned nblocks, unsigned nthreads, size_t smem,
                                          cudaStream_t st, bool urgent, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nblocks);
  cfg.blockDim = dim3(nthreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  if (urgent) {
    static const int greatest = [] {
      int least = 0, g = 0;
      return cudaDeviceGetStreamPriorityRange(&least, &g) == cudaSuccess ? g : 0;
    }();
    at[1].id = cudaLaunchAttributePriority;
    at[1].val.priority = greatest;
    cfg.numAttrs = 2;
  }
  return cudaLaunchKernelEx(&cfg, kern, args...);
}
template <class... KArgs, class... Args>
static inline cudaError_t launch_pdl(void (*kern)(KArgs...), unsigned nblocks, unsigned nthreads, size_t smem,
                                     cudaStream_t st, Args... args) {
  return launch_pdl_prio(kern, nblocks, nthreads, smem, st, false, args...);
}

}  // namespace gdn2
