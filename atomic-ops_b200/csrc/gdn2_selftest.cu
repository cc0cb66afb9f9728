// Self-test of the tensor-core operand path: one 128 x N x 128 GEMM staged through the
// same shared-memory tile writers, descriptors and MMA issue helpers the operator uses.
#include "gdn2_common.cuh"

namespace gdn2 {

// Shared memory: A region (whole-K tiles need 2 x 64 KB), B region (2 x N*128 B), barrier, TMEM slot.
constexpr uint32_t kSelftestA = 2 * 65536;
constexpr uint32_t kSelftestB = 2 * 32768;
constexpr uint32_t kSelftestSmem = kSelftestA + kSelftestB + 1024 + 64;

__global__ void __launch_bounds__(kThreads, 1)
    selftest_gemm_kernel(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ C, int N,
                         int prec, int a_mode, int b_mn, unsigned* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kSelftestA;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sB + kSelftestB);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sB + kSelftestB + 16);

  const int t = threadIdx.x;
  const Mode md = mode_from_enum(prec);
  const int e = md.fmt == kTF32 ? 4 : 2;
  const int KS = 128 / e;  // K elements per 128-byte slice
  const bool lo = md.passes == 3;

  if (t < 32) {
    tmem_alloc(tslot, 256);
    tmem_relinquish();
  }
  if (t == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;

  const uint32_t a_base = smem_u32(sA), b_base = smem_u32(sB);
  uint32_t phase = 0;

  if (a_mode >= 2) {
    // Whole-K K-major tile of A (row bytes = 128 * e), hi at a_base, lo at a_base + 64 KB.
    Tile ah = tile_k(a_base, 128 * e), al = tile_k(a_base + 65536, 128 * e);
    float v[8];
    for (int k0 = 0; k0 < 128; k0 += 8) {
      for (int i = 0; i < 8; ++i) v[i] = A[t * 128 + k0 + i];
      stage_krow(ah, al, lo, md.fmt, t, k0, v, 8);
    }
  }

  const int nslices = 128 / KS;
  for (int s = 0; s < nslices; ++s) {
    const int kbeg = s * KS;
    Tile at[2], bt[2];
    if (a_mode == 0) {
      at[0] = tile_k(a_base, 128);
      at[1] = tile_k(a_base + 16384, 128);
      float v[8];
      for (int i = 0; i < KS; i += 8) {
        for (int j = 0; j < 8; ++j) v[j] = A[t * 128 + kbeg + i + j];
        stage_krow(at[0], at[1], lo, md.fmt, t, i, v, 8);
      }
    } else if (a_mode == 1) {
      at[0] = tile_mn(a_base, 128 * e, md.fmt);
      at[1] = tile_mn(a_base + 16384, 128 * e, md.fmt);
      if (t >= kbeg && t < kbeg + KS) {
        float v[8];
        for (int m0 = 0; m0 < 128; m0 += 8) {
          for (int j = 0; j < 8; ++j) v[j] = A[(m0 + j) * 128 + t];
          stage_mnrow(at[0], at[1], lo, md.fmt, t - kbeg, m0, v, 8);
        }
      }
    } else if (a_mode == 2) {
      at[0] = tile_k(a_base, 128 * e);
      at[1] = tile_k(a_base + 65536, 128 * e);
      at[0].addr += (uint32_t)s * 4 * at[0].step;
      at[1].addr += (uint32_t)s * 4 * at[1].step;
    } else {
      // Transposed view of the whole-K K-major tile (bf16 only): MN-major with lbo = 8 * row bytes.
      at[0] = tile_k_as_mn(a_base, 128 * e);
      at[1] = tile_k_as_mn(a_base + 65536, 128 * e);
      at[0].addr += (uint32_t)s * 4 * at[0].step;
      at[1].addr += (uint32_t)s * 4 * at[1].step;
    }
    const uint32_t bhalf = (uint32_t)N * 128u;
    if (!b_mn) {
      bt[0] = tile_k(b_base, 128);
      bt[1] = tile_k(b_base + bhalf, 128);
      if (t < N) {
        float v[8];
        for (int i = 0; i < KS; i += 8) {
          for (int j = 0; j < 8; ++j) v[j] = B[(kbeg + i + j) * N + t];
          stage_krow(bt[0], bt[1], lo, md.fmt, t, i, v, 8);
        }
      }
      // second half of the rows for N = 256
      if (N > 128) {
        float v[8];
        for (int i = 0; i < KS; i += 8) {
          for (int j = 0; j < 8; ++j) v[j] = B[(kbeg + i + j) * N + t + 128];
          stage_krow(bt[0], bt[1], lo, md.fmt, t + 128, i, v, 8);
        }
      }
    } else {
      bt[0] = tile_mn(b_base, (uint32_t)N * e, md.fmt);
      bt[1] = tile_mn(b_base + bhalf, (uint32_t)N * e, md.fmt);
      if (t >= kbeg && t < kbeg + KS) {
        float v[8];
        for (int n0 = 0; n0 < N; n0 += 8) {
          for (int j = 0; j < 8; ++j) v[j] = B[t * N + n0 + j];
          stage_mnrow(bt[0], bt[1], lo, md.fmt, t - kbeg, n0, v, 8);
        }
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (t == 0) {
      tc_fence_after();
      mma_tiles(md.fmt, md.passes, tbase, at, bt, N, 4, false, s > 0);
      mma_commit(bar);
    }
    mbar_wait(bar, phase, status);
    phase ^= 1u;
    tc_fence_after();
  }

  for (int c0 = 0; c0 < N; c0 += 32) {
    float v[32];
    tmem_ld32(tbase, c0, v);
    for (int j = 0; j < 32; ++j) C[t * N + c0 + j] = v[j];
  }
  tc_fence_before();
  __syncthreads();
  if (t < 32) tmem_dealloc(tbase, 256);
}

}  // namespace gdn2

extern "C" gdn2_status gdn2_selftest_gemm(const float* A, const float* B, float* C, int32_t N, int32_t precision,
                                          int32_t a_mode, int32_t b_mn, uint32_t* dev_status, void* stream) {
  if (!A || !B || !C || !dev_status) return GDN2_ERR_INVALID_ARGUMENT;
  if (!(N == 32 || N == 64 || N == 128 || N == 256)) return GDN2_ERR_INVALID_ARGUMENT;
  if (precision < 0 || precision > 3 || a_mode < 0 || a_mode > 3 || b_mn < 0 || b_mn > 1)
    return GDN2_ERR_INVALID_ARGUMENT;
  if (a_mode == 3 && gdn2::mode_from_enum(precision).fmt == gdn2::kTF32) return GDN2_ERR_UNSUPPORTED;
  if (cudaFuncSetAttribute(gdn2::selftest_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           gdn2::kSelftestSmem) != cudaSuccess)
    return GDN2_ERR_CUDA;
  gdn2::selftest_gemm_kernel<<<1, gdn2::kThreads, gdn2::kSelftestSmem, (cudaStream_t)stream>>>(
      A, B, C, N, precision, a_mode, b_mn, dev_status);
  return cudaGetLastError() == cudaSuccess ? GDN2_OK : GDN2_ERR_CUDA;
}

// ---------------------------------------------------------------------------------------------
// Self-test of the chunk kernels' staging engine (swizzled pool tiles, operand kinds): one
// 128 x 128 x 128 product C = A B through gemm1, A and B taken from global memory as K-major
// own-row (kmaj), K-major coalesced (kany) or MN-major coalesced (mn_any) operands.
// ---------------------------------------------------------------------------------------------
#include "gdn2_kernels.cuh"

namespace gdn2 {

constexpr uint32_t kEngineSmem = 1024 + 4 * 16384 + 64;

template <int AK, int BK>
__global__ void __launch_bounds__(kCT, 1)
    selftest_engine_kernel(const float* __restrict__ A, const float* __restrict__ At, const float* __restrict__ B,
                           const float* __restrict__ Bt, float* __restrict__ C, int prec, unsigned* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t pool = smem_u32(sm);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + 4 * 16384);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);
  const int tid = threadIdx.x, warp = tid >> 5;
  if (warp == 0) {
    tmem_alloc(tslot, 128);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tb = *tslot;
  MmaBar mb{bar, 0u, status};
  const Mode m = mode_from_enum(prec);
  // operand rows: A row m = A[m][:], A^T row k = At[k][:], B^T row n = Bt[n][:], B row k = B[k][:]
  auto a16 = [&](int r, int c0, float* x) { ld16_f(A + r * 128 + c0, x); };
  auto a4 = [&](int r, int c0, float* x) { ld4_f(A + r * 128 + c0, x); };
  auto at4 = [&](int r, int c0, float* x) { ld4_f(At + r * 128 + c0, x); };
  auto b16 = [&](int r, int c0, float* x) { ld16_f(Bt + r * 128 + c0, x); };
  auto b4 = [&](int r, int c0, float* x) { ld4_f(Bt + r * 128 + c0, x); };
  auto bk4 = [&](int r, int c0, float* x) { ld4_f(B + r * 128 + c0, x); };
  auto run = [&](auto aop) {
    if constexpr (BK == 0) gemm1(m, pool, mb, tb, aop, kmaj(b16), false, false);
    else if constexpr (BK == 1) gemm1(m, pool, mb, tb, aop, kany(b4), false, false);
    else gemm1(m, pool, mb, tb, aop, mn_any(bk4), false, false);
  };
  if constexpr (AK == 0) run(kmaj(a16));
  else if constexpr (AK == 1) run(kany(a4));
  else run(mn_any(at4));
  const int t = crow(), cb = chalf() * 64;
  for (int c0 = cb; c0 < cb + 64; c0 += 16) {
    float x[16];
    tmem_ld16(tb, (uint32_t)c0, x);
    st16_f(C + t * 128 + c0, x);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tb, 128);
}

template <int AK, int BK>
static cudaError_t launch_engine(const float* A, const float* At, const float* B, const float* Bt, float* C, int prec,
                                 unsigned* st, cudaStream_t s) {
  cudaError_t e = cudaFuncSetAttribute(selftest_engine_kernel<AK, BK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kEngineSmem);
  if (e != cudaSuccess) return e;
  selftest_engine_kernel<AK, BK><<<1, kCT, kEngineSmem, s>>>(A, At, B, Bt, C, prec, st);
  return cudaGetLastError();
}
template <int AK>
static cudaError_t launch_engine_b(int bk, const float* A, const float* At, const float* B, const float* Bt, float* C,
                                   int prec, unsigned* st, cudaStream_t s) {
  if (bk == 0) return launch_engine<AK, 0>(A, At, B, Bt, C, prec, st, s);
  if (bk == 1) return launch_engine<AK, 1>(A, At, B, Bt, C, prec, st, s);
  return launch_engine<AK, 2>(A, At, B, Bt, C, prec, st, s);
}

// Failure-detection self-test: one warp waits on an mbarrier phase that nothing completes, with
// the same bounded wait every kernel of the library uses, so the wait must run out, set the
// timeout bit and return; the elapsed cycles are reported.  No fault, trap or endless loop.
__global__ void selftest_wait_kernel(unsigned* st, long long limit, long long* cycles) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncwarp();
  const long long t0 = clock64();
  const bool done = mbar_wait_for(&bar, 0u, st, limit);
  const long long dt = clock64() - t0;
  if (threadIdx.x == 0) *cycles = done ? -1 : dt;
}

}  // namespace gdn2

extern "C" gdn2_status gdn2_selftest_wait_timeout(uint32_t* dev_status, int64_t limit_cycles, int64_t* dev_cycles,
                                                  void* stream) {
  using namespace gdn2;
  if (!dev_status || !dev_cycles || limit_cycles <= 0 || limit_cycles > kWaitCycles) return GDN2_ERR_INVALID_ARGUMENT;
  selftest_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(dev_status, (long long)limit_cycles,
                                                            reinterpret_cast<long long*>(dev_cycles));
  return cudaGetLastError() == cudaSuccess ? GDN2_OK : GDN2_ERR_CUDA;
}

extern "C" gdn2_status gdn2_selftest_engine(const float* A, const float* At, const float* B, const float* Bt, float* C,
                                            int32_t precision, int32_t a_kind, int32_t b_kind, uint32_t* dev_status,
                                            void* stream) {
  using namespace gdn2;
  if (!A || !At || !B || !Bt || !C || !dev_status) return GDN2_ERR_INVALID_ARGUMENT;
  if (precision < 0 || precision > 3 || a_kind < 0 || a_kind > 2 || b_kind < 0 || b_kind > 2)
    return GDN2_ERR_INVALID_ARGUMENT;
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e;
  if (a_kind == 0) e = launch_engine_b<0>(b_kind, A, At, B, Bt, C, precision, dev_status, s);
  else if (a_kind == 1) e = launch_engine_b<1>(b_kind, A, At, B, Bt, C, precision, dev_status, s);
  else e = launch_engine_b<2>(b_kind, A, At, B, Bt, C, precision, dev_status, s);
  return e == cudaSuccess ? GDN2_OK : GDN2_ERR_CUDA;
}
