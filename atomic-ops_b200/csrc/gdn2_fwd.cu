// Chunk-parallel forward kernels of the GDN-2 operator (sm_100a).
//
//   fwd_intra  one CTA per (b, h, chunk): gate cumsum, gated scores Aqk / Akk, the WY inverse
//              A = (I + (1-eps) Akk)^-1, wp = A (b k e^gc), u = A (w v), and the chunk's
//              state-transition pair  M = diag(e^gl) - kg^T wp,  Bc = kg^T u  so that the
//              inter-chunk recurrence becomes h <- M h + Bc.
//   fwd_out    one CTA per (b, h, chunk), after the scan: v_new = u - wp h_pre,
//              o = scale qg h_pre + Aqk v_new.
//
// Reference: atomic_gdn2/pipeline.py:20-26 (_fwd), fwd/scores.py (build_scores),
// fwd/solve.py (wy_solve_leafbatched), fwd/cd_slim.py:8-31 (recompute + scan).
//
// Gated scores.  Aqk[i,j] = scale sum_d q[i,d] k[j,d] e^(gc[i,d]-gc[j,d]) (i >= j) and
// Akk[i,j] = sum_d b[i,d] k[i,d] k[j,d] e^(gc[i,d]-gc[j,d]) (i > j) are computed as plain
// 128x128x128 tensor-core products of rescaled operands q e^(gc-m), k e^(m-gc) with one
// reference point per channel, m = (max_t gc + min_t gc) / 2.  Every leg then lies in
// [e^(-span/2), e^(span/2)].  This is the balanced-leg idea of the reference's BTL diagonal
// (fwd/scores.py:16-28) applied to the whole chunk, which the B200's fp32 range allows for
// spans up to kSpanMax.  Channels whose span inside the chunk is larger ("wide" channels,
// strongly decaying gates) are left out of the tensor-core products (their legs are zero) and
// their contribution sum_d q[i,d] k[j,d] e^(gc[i,d]-gc[j,d]) is added exactly by the CUDA
// cores, with the exponent difference formed first (<= 0 on the causal entries); chunks
// without wide channels never run that code.
//
// WY inverse.  With N = I + Se (Se = (1-eps) Akk, strictly lower), Dg its four 32x32 diagonal
// blocks and R the strictly block-lower rest, N^-1 = (I - W)(I + W^2) Dg^-1 with W = Dg^-1 R
// (W^4 = 0).  Dg^-1 comes from warp-level forward substitution (one warp per block, lane =
// column, fp32); the four remaining products run on the tensor core in solve_dot_mode, as three
// dependent K-loops: W, then W^2 and W Dg^-1 together, then W^2 Q with Q = (I - W) Dg^-1, so that
// N^-1 = Q + W^2 Q.  This replaces the reference's leaf + block-doubling ladder (fwd/solve.py:9-43).
#include <type_traits>

#include "gdn2_kernels.cuh"

namespace gdn2 {

constexpr uint32_t kPoolBytes = 6 * 16384;                  // six 16 KB operand tiles
constexpr uint32_t kGcBytes = kT * kGcPitch * 4;             // 67,584
constexpr uint32_t kDsmFloats = 4 * 32 * 33;                 // four padded 32x32 blocks
constexpr uint32_t kIntraSmem = 1024 + kPoolBytes + kGcBytes + kDsmFloats * 4 + 4 * kD * 4 + 64;
constexpr uint32_t kOutSmem = 1024 + kPoolBytes + kGcBytes + 64;

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// ---------------------------------------------------------------------------------------
// fwd_intra
// ---------------------------------------------------------------------------------------
// Wide channels' exact contribution to row i of the raw scores, columns j = c0..c0+15:
//   aq[j] += sum_{d wide} q[i,d] k[j,d] e^(gc[i,d]-gc[j,d]),  ak[j] = sum_{d wide} (b k)[i,d] k[j,d] e^(...)
// (entries with j > i are masked by the caller; their exponent is clamped at 0).
template <class TIn>
__device__ __forceinline__ void wide_scores(const TIn* __restrict__ q, const TIn* __restrict__ k,
                                            const TIn* __restrict__ b, const float* gcs, const float* wide_s, int i,
                                            int c0, float* aq, float* ak) {
#pragma unroll
  for (int j = 0; j < 16; ++j) ak[j] = 0.f;
#pragma unroll 1
  for (int d = 0; d < kD; ++d) {
    if (wide_s[d] == 0.f) continue;
    const float gci = gcs[i * kGcPitch + d];
    const float qi = ld1(q + i * kD + d), bki = ld1(b + i * kD + d) * ld1(k + i * kD + d);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int jj = c0 + j;
      const float w = ld1(k + jj * kD + d) * ex(fminf(gci - gcs[jj * kGcPitch + d], 0.f));
      aq[j] = fmaf(qi, w, aq[j]);
      ak[j] = fmaf(bki, w, ak[j]);
    }
  }
}

// WIDE = false: the common path; it records in the residual whether the chunk has wide channels
// and hands such chunks to the WIDE = true path (an out-of-line call in the same launch).
template <class TIn>
__device__ __noinline__ void fwd_intra_wide(const OpParams& p, const int ch);

template <class TIn, int DOT, int SOLVE, bool WIDE>
__device__ __forceinline__ void fwd_intra_chunk(const OpParams& p, const int ch) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  const uint32_t pool = smem_u32(sm);
  float* gcs = reinterpret_cast<float*>(sm + kPoolBytes);
  float* dsm = reinterpret_cast<float*>(sm + kPoolBytes + kGcBytes);
  float* mzE_s = dsm + kDsmFloats;  // per-channel reference m of the E legs (+1e30: wide channel)
  float* gl_s = mzE_s + kD;
  float* mzF_s = gl_s + kD;          // reference of the F legs (-1e30: wide channel)
  float* wide_s = mzF_s + kD;        // 1 for a wide channel
  uint64_t* bar = reinterpret_cast<uint64_t*>(wide_s + kD);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t = crow(), half = chalf();
  const int cb = half * 64;  // this thread's 64 columns of its row
  const int bh = ch / p.NC, c = ch % p.NC;
  const long long off = chunk_off(p, bh, c);
  const TIn* q = reinterpret_cast<const TIn*>(p.q) + off;
  const TIn* k = reinterpret_cast<const TIn*>(p.k) + off;
  const TIn* v = reinterpret_cast<const TIn*>(p.v) + off;
  const TIn* w = reinterpret_cast<const TIn*>(p.w) + off;
  const TIn* b = reinterpret_cast<const TIn*>(p.b) + off;
  const TIn* g = reinterpret_cast<const TIn*>(p.g) + off;
  const size_t mat = (size_t)kT * kD;
  float* aqk_g = reinterpret_cast<float*>(p.res + p.rl.aqk) + (size_t)ch * mat;
  float* ainv_g = reinterpret_cast<float*>(p.res + p.rl.ainv) + (size_t)ch * mat;
  float* wp_g = reinterpret_cast<float*>(p.res + p.rl.wp) + (size_t)ch * mat;
  float* u_g = reinterpret_cast<float*>(p.fws + p.rl.u) + (size_t)ch * mat;
  float* bc_g = reinterpret_cast<float*>(p.fws + p.rl.bc) + (size_t)ch * mat;
  uint8_t* mf_g = p.fws + p.rl.mf + (size_t)ch * p.rl.mf_stride;

  const Mode md = mode_from_enum(DOT >= 0 ? DOT : p.dot_mode);
  const Mode ms = mode_from_enum(SOLVE >= 0 ? SOLVE : p.solve_mode);
  const float clip = p.clip;

  int* wide_flag = reinterpret_cast<int*>(p.res + p.rl.wide) + ch;
  if constexpr (WIDE) {
    if (*wide_flag == 0) return;
  }
  {
    float mx, mn;
    bool pos;
    chunk_cumsum(g, gcs, mx, mn, pos);
    if (tid < kD) {
      const bool wide = mx - mn > kSpanMax;
      const float mid = 0.5f * (mx + mn);
      mzE_s[tid] = wide ? 1e30f : mid;
      mzF_s[tid] = wide ? -1e30f : mid;
      wide_s[tid] = wide ? 1.f : 0.f;
      if (pos && !WIDE) atomicOr(p.status, kStatusPositiveGate);
    }
    const int any_wide = __syncthreads_or(tid < kD && mx - mn > kSpanMax);
    if constexpr (!WIDE) {
      if (tid == 0) *wide_flag = any_wide;
      if (any_wide) {
        __syncthreads();  // the flag is visible to the whole CTA
        fwd_intra_wide<TIn>(p, ch);
        return;
      }
    }
  }
  if (warp == 0) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid < kD) gl_s[tid] = gcs[(kT - 1) * kGcPitch + tid];
  const uint32_t tb = *tslot;
  const uint32_t S0 = tb, S1 = tb + 128, S2 = tb + 256, S3 = tb + 384;
  MmaBar mbar{bar, 0u, p.status};
  __syncthreads();

  // ---- global row sources (4 values of row r from column c0: kany / mn_any operands) -----------
  auto src_qE = [&](int r, int c0, float* x) {  // q e^(gc - m)
    ld4_in(q + r * kD + c0, x);
    const float* gr = gcs + r * kGcPitch + c0;
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] *= ex(gr[j] - mzE_s[c0 + j]);
  };
  auto src_bkE = [&](int r, int c0, float* x) {  // b k e^(gc - m)
    float kv[4];
    ld4_in(b + r * kD + c0, x);
    ld4_in(k + r * kD + c0, kv);
    const float* gr = gcs + r * kGcPitch + c0;
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = x[j] * kv[j] * ex(gr[j] - mzE_s[c0 + j]);
  };
  auto src_kF = [&](int r, int c0, float* x) {  // k e^(m - gc)
    ld4_in(k + r * kD + c0, x);
    const float* gr = gcs + r * kGcPitch + c0;
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] *= ex(mzF_s[c0 + j] - gr[j]);
  };
  auto src_kb = [&](int r, int c0, float* x) {  // b k e^min(gc, 0)
    float kv[4];
    ld4_in(b + r * kD + c0, x);
    ld4_in(k + r * kD + c0, kv);
    const float* gr = gcs + r * kGcPitch + c0;
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = x[j] * kv[j] * ex(fminf(gr[j], 0.f));
  };
  auto src_wv = [&](int r, int c0, float* x) {
    float vv[4];
    ld4_in(w + r * kD + c0, x);
    ld4_in(v + r * kD + c0, vv);
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] *= vv[j];
  };
  auto src_kg = [&](int r, int c0, float* x) {  // sanitize(k e^min(gl - gc, 0))
    ld4_in(k + r * kD + c0, x);
    const float* gr = gcs + r * kGcPitch + c0;
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = sanitize(x[j] * ex(fminf(gl_s[c0 + j] - gr[j], 0.f)), clip);
  };
  // ---- shared-memory / TMEM row sources (16 values: kmaj / mn_own operands) ---------------------
  auto src_dinv = [&](int r, int c0, float* x) {  // row r of the block-diagonal Dg^-1
    if ((c0 >> 5) == (r >> 5)) {
      const float* src = dsm + (r >> 5) * 1056 + (r & 31) * 33 + (c0 & 31);
#pragma unroll
      for (int j = 0; j < 16; ++j) x[j] = src[j];
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) x[j] = 0.f;
    }
  };
  auto src_R = [&](int r, int c0, float* x) {  // strictly block-lower part of Se (TMEM S1, owner)
    tmem_ld16(S1, (uint32_t)c0, x);
    const int lim = (r >> 5) << 5;
#pragma unroll
    for (int j = 0; j < 16; ++j) x[j] = (c0 + j < lim) ? x[j] : 0.f;
  };
  auto src_dinv4 = [&](int r, int c0, float* x) {  // 4 values of row r of Dg^-1 (mn_any operand)
    const bool in = (c0 >> 5) == (r >> 5);
    const float* src = dsm + (r >> 5) * 1056 + (r & 31) * 33 + (c0 & 31);
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = in ? src[j] : 0.f;
  };
  auto tm = [&](uint32_t slot) { return [=](int, int c0, float* x) { tmem_ld16(slot, (uint32_t)c0, x); }; };

  // ---- 1. scores: S0 = (q E)(k F)^T, S1 = (b k E)(k F)^T                      (dot mode) --------
  gemm2(md, pool, mbar, S0, kany(src_qE), kany(src_kF), false, false, S1, kany(src_bkE), kany(NoSrc()), false,
        false, false, true);

  // ---- 2. Aqk out (scale, causal, sanitize); Se = (1-eps) sanitize(Akk) strict, in place -----------
  // (the body is instantiated twice: chunks with wide channels add their exact terms)
  auto ep2 = [&](auto wide_tag) {
    constexpr bool kWide = decltype(wide_tag)::value;
    const float keep = 1.0f - p.eps;
    const int blk = t >> 5;
    float* xb = xbuf(sm);
    for (int c0 = cb; c0 < cb + 64; c0 += 16) {
      float x[16], wk[16];
      tmem_ld16(S0, c0, x);
      if constexpr (kWide) wide_scores(q, k, b, gcs, wide_s, t, c0, x, wk);
#pragma unroll
      for (int j = 0; j < 16; ++j) x[j] = (c0 + j <= t) ? sanitize(p.scale * x[j], clip) : 0.f;
      xb_put16(xb, c0 - cb, x);
      tmem_ld16(S1, c0, x);
      if constexpr (kWide) {
#pragma unroll
        for (int j = 0; j < 16; ++j) x[j] += wk[j];
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) x[j] = (c0 + j < t) ? keep * sanitize(x[j], clip) : 0.f;
      tmem_st16(S1, c0, x);
      if ((c0 >> 5) == blk) {
#pragma unroll
        for (int j = 0; j < 16; ++j) dsm[blk * 1056 + (t & 31) * 33 + (c0 & 31) + j] = x[j];
      }
    }
    xb_flush(xb, aqk_g, kT, cb);
  };
  ep2(std::integral_constant<bool, WIDE>{});
  if (tid == 0) {  // L2 hints for step 8's w and v, first read after the on-chip solve below
    constexpr uint32_t kInTile = kT * kD * sizeof(TIn);
    l2_prefetch(w, kInTile);
    l2_prefetch(v, kInTile);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  // ---- 3. diagonal-block inverses (forward substitution, warp = block, lane = column) ----------
  if (warp < 4) {
    const float* Sb = dsm + warp * 1056;
    float x[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      float acc = (i == lane) ? 1.f : 0.f;
#pragma unroll
      for (int j = 0; j < i; ++j) acc = fmaf(-Sb[i * 33 + j], x[j], acc);
      x[i] = acc;
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 32; ++i) dsm[warp * 1056 + i * 33 + lane] = x[i];
  }
  __syncthreads();

  // ---- 4.-7. A = (I + W^2)(I - W) Dg^-1 = Q + W^2 Q,  Q = Dg^-1 - W Dg^-1,  W = Dg^-1 R   (solve mode)
  //      three dependent K-loops: W; then W^2 and W Dg^-1 sharing the staged W; then W^2 Q
  gemm1(ms, pool, mbar, S0, kmaj(src_dinv), mn_own(src_R), false, false);   // W -> S0
  gemm2(ms, pool, mbar, S2, kmaj(tm(S0)), mn_own(tm(S0)), false, false, S3, kmaj(NoSrc()), mn_any(src_dinv4), false,
        false, true, false);                                                 // W^2 -> S2, W Dg^-1 -> S3
  for (int c0 = cb; c0 < cb + 64; c0 += 16) {                               // Q = Dg^-1 - W Dg^-1 -> S3
    float x[16], dv[16];
    tmem_ld16(S3, c0, x);
    src_dinv(t, c0, dv);
#pragma unroll
    for (int j = 0; j < 16; ++j) x[j] = dv[j] - x[j];
    tmem_st16(S3, c0, x);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  gemm1(ms, pool, mbar, S0, kmaj(tm(S2)), mn_own(tm(S3)), false, false);    // W^2 Q -> S0
  {
    float* xb = xbuf(sm);
    for (int c0 = cb; c0 < cb + 64; c0 += 16) {                             // A = sanitize(Q + W^2 Q)
      float x[16], y[16];
      tmem_ld16(S3, c0, x);
      tmem_ld16(S0, c0, y);
#pragma unroll
      for (int j = 0; j < 16; ++j) x[j] = (c0 + j <= t) ? sanitize(x[j] + y[j], clip) : 0.f;
      tmem_st16(S1, c0, x);
      xb_put16(xb, c0 - cb, x);
    }
    xb_flush(xb, ainv_g, kT, cb);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  // ---- 8. wp = A (b k e^gc) -> S0,  u = A (w v) -> S2                          (dot mode) --------
  gemm2(md, pool, mbar, S0, kmaj(tm(S1)), mn_any(src_kb), false, false, S2, kmaj(NoSrc()), mn_any(src_wv), false,
        false, true, false);
  {
    float* xb = xbuf(sm);
#pragma unroll 1
    for (int pass = 0; pass < 2; ++pass) {
      const uint32_t slot = pass ? S2 : S0;
      for (int c0 = cb; c0 < cb + 64; c0 += 16) {
        float x[16];
        tmem_ld16(slot, c0, x);
#pragma unroll
        for (int j = 0; j < 16; ++j) x[j] = sanitize(x[j], clip);
        xb_put16(xb, c0 - cb, x);
      }
      xb_flush(xb, pass ? u_g : wp_g, kD, cb);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  // ---- 9. M = diag(e^gl) - kg^T wp -> S1,  Bc = kg^T u -> S3                  (dot mode) --------
  //      wp and u are read back from the residual tiles just written (L2) rather than staged from
  //      TMEM: a TMEM-backed MN-major operand can only be staged by the two warps owning the slice's
  //      lanes, a global one by all eight
  auto src_wp_res = [&](int r, int c0, float* x) { ld4_cg(wp_g + r * kD + c0, x); };
  auto src_u_res = [&](int r, int c0, float* x) { ld4_cg(u_g + r * kD + c0, x); };
  gemm2(md, pool, mbar, S1, mn_any(src_kg), mn_any(src_wp_res), false, false, S3, mn_any(NoSrc()), mn_any(src_u_res),
        false, false, true, false);
  {
    const float dec = ex(fminf(gl_s[t], 0.f));
    for (int c0 = cb; c0 < cb + 64; c0 += 16) {
      float x[16];
      tmem_ld16(S1, c0, x);
#pragma unroll
      for (int j = 0; j < 16; ++j) x[j] = ((c0 + j) == t ? dec : 0.f) - x[j];
      image_store8(mf_g, md, t, c0, x);
      image_store8(mf_g, md, t, c0 + 8, x + 8);
      tmem_ld16(S3, c0, x);
      xb_put16(xbuf(sm), c0 - cb, x);
    }
    xb_flush(xbuf(sm), bc_g, kD, cb);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tb, 512);
}

// A chunk with wide channels, out of line: its exact CUDA-core terms need registers that the
// common path cannot spare, and its rare call costs the common path no launch of its own.
template <class TIn>
__device__ __noinline__ void fwd_intra_wide(const OpParams& p, const int ch) {
  fwd_intra_chunk<TIn, -1, -1, true>(p, ch);
}

template <class TIn, int DOT, int SOLVE>
__global__ void __launch_bounds__(kCT, 1) fwd_intra_kernel(const OpParams p) {
  pdl_enter();
  fwd_intra_chunk<TIn, DOT, SOLVE, false>(p, p.ch0 + (int)blockIdx.x);
}

// ---------------------------------------------------------------------------------------
// fwd_out: v_new = u - wp h_pre;  o = sanitize(scale qg h_pre + Aqk v_new)
// ---------------------------------------------------------------------------------------
template <class TIn, int DOT>
__global__ void __launch_bounds__(kCT, 1) fwd_out_kernel(const OpParams p, float* __restrict__ o_out) {
  pdl_enter();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  const uint32_t pool = smem_u32(sm);
  float* gcs = reinterpret_cast<float*>(sm + kPoolBytes);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kPoolBytes + kGcBytes);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int t = crow(), cb = chalf() * 64;
  const int ch = p.ch0 + (int)blockIdx.x, bh = ch / p.NC, c = ch % p.NC;
  const long long off = chunk_off(p, bh, c);
  const TIn* q = reinterpret_cast<const TIn*>(p.q) + off;
  const TIn* g = reinterpret_cast<const TIn*>(p.g) + off;
  const size_t mat = (size_t)kT * kD;
  const float* aqk_g = reinterpret_cast<const float*>(p.res + p.rl.aqk) + (size_t)ch * mat;
  const float* wp_g = reinterpret_cast<const float*>(p.res + p.rl.wp) + (size_t)ch * mat;
  const float* u_g = reinterpret_cast<const float*>(p.fws + p.rl.u) + (size_t)ch * mat;
  const float* h_g = reinterpret_cast<const float*>(p.res + p.rl.hs) + ((size_t)bh * p.NC + c) * mat;
  float* vn_g = reinterpret_cast<float*>(p.res + p.rl.vnew) + (size_t)ch * mat;
  float* o_g = o_out + off;
  const Mode md = mode_from_enum(DOT >= 0 ? DOT : p.dot_mode);
  const float clip = p.clip, scale = p.scale;

  if (warp == 0) {
    tmem_alloc(tslot, 256);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  {
    float mx, mn;
    bool pos;
    chunk_cumsum(g, gcs, mx, mn, pos);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tb = *tslot;
  const uint32_t S0 = tb, S1 = tb + 128;
  MmaBar mbar{bar, 0u, p.status};

  // global row sources: 4 values of row r from column c0 (kany / mn_any operands)
  auto src_wp = [&](int r, int c0, float* x) { ld4_f(wp_g + r * kD + c0, x); };
  auto src_qg = [&](int r, int c0, float* x) {  // scale sanitize(q e^min(gc, 0))
    ld4_in(q + r * kD + c0, x);
    const float* gr = gcs + r * kGcPitch + c0;
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = scale * sanitize(x[j] * ex(fminf(gr[j], 0.f)), clip);
  };
  auto src_h = [&](int r, int c0, float* x) { ld4_f(h_g + r * kD + c0, x); };
  auto src_aqk = [&](int r, int c0, float* x) { ld4_f(aqk_g + r * kT + c0, x); };

  // S0 = wp h_pre,  S1 = (scale qg) h_pre   (shared B = h_pre)
  gemm2(md, pool, mbar, S0, kany(src_wp), mn_any(src_h), false, false, S1, kany(src_qg), mn_any(NoSrc()), false,
        false, false, true);
  if (threadIdx.x == 0) l2_prefetch(aqk_g, kT * kT * 4);  // L2 hint for the Aqk v_new product below
  // v_new = u - S0 (kept in S0 and written as a residual)
  {
    float uv[64];
    float* xb = xbuf(sm);  // two 1024-float blocks, then the 32 x 64 output block
    xs_fill(xb, 0, u_g, kD, cb);
    xs_fill(xb, 1, u_g, kD, cb + 32);
    xs_wait();
#pragma unroll
    for (int j = 0; j < 4; ++j) xs_get16(xb, j >> 1, 16 * (j & 1), uv + 16 * j);
    __syncwarp();  // the buffer is reused for v_new below
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int c0 = cb + 16 * jj;
      float x[16];
      tmem_ld16(S0, c0, x);
#pragma unroll
      for (int j = 0; j < 16; ++j) x[j] = uv[16 * jj + j] - x[j];
      xb_put16(xb, c0 - cb, x);
    }
    xb_flush(xb, vn_g, kD, cb);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // S1 += Aqk v_new, v_new read back from the residual tile just written (L2): all warps stage it,
  // where a TMEM-backed MN-major operand is staged by the two warps owning each slice's lanes
  auto src_vn_res = [&](int r, int c0, float* x) { ld4_cg(vn_g + r * kD + c0, x); };
  gemm1(md, pool, mbar, S1, kany(src_aqk), mn_any(src_vn_res), false, true);
  {
    float* xb = xbuf(sm);
    for (int c0 = cb; c0 < cb + 64; c0 += 16) {
      float x[16];
      tmem_ld16(S1, c0, x);
#pragma unroll
      for (int j = 0; j < 16; ++j) x[j] = sanitize(x[j], clip);
      xb_put16(xb, c0 - cb, x);
    }
    xb_flush(xb, o_g, kD, cb);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tb, 256);
}

// ---------------------------------------------------------------------------------------
// Host-side launchers
// ---------------------------------------------------------------------------------------
// Kernels are compiled with compile-time precision modes for the configurations that matter
// (the reference's defaults and the all-bf16 mode), and with runtime modes for the rest (-1).
template <class TIn, int DOT, int SOLVE>
static cudaError_t launch_fwd_intra_t(const OpParams& p, int nblocks, cudaStream_t st) {
  static unsigned long long done = 0;
  cudaError_t e = smem_attr_once(fwd_intra_kernel<TIn, DOT, SOLVE>, (int)kIntraSmem, done);
  if (e != cudaSuccess) return e;
  e = launch_pdl(fwd_intra_kernel<TIn, DOT, SOLVE>, nblocks, kCT, kIntraSmem, st, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}
template <class TIn, int DOT>
static cudaError_t launch_fwd_out_t(const OpParams& p, float* o, int nblocks, cudaStream_t st) {
  static unsigned long long done = 0;
  cudaError_t e = smem_attr_once(fwd_out_kernel<TIn, DOT>, (int)kOutSmem, done);
  if (e != cudaSuccess) return e;
  e = launch_pdl(fwd_out_kernel<TIn, DOT>, nblocks, kCT, kOutSmem, st, p, o);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}
// One launch; chunks with wide channels take the out-of-line path (runtime modes) inside it.
template <class TIn>
static cudaError_t launch_fwd_intra_m(const OpParams& p, int nblocks, cudaStream_t st) {
  if (p.dot_mode == GDN2_PREC_HIGHEST && p.solve_mode == GDN2_PREC_BF16X3)
    return launch_fwd_intra_t<TIn, GDN2_PREC_HIGHEST, GDN2_PREC_BF16X3>(p, nblocks, st);
  if (p.dot_mode == GDN2_PREC_DEFAULT && p.solve_mode == GDN2_PREC_DEFAULT)
    return launch_fwd_intra_t<TIn, GDN2_PREC_DEFAULT, GDN2_PREC_DEFAULT>(p, nblocks, st);
  return launch_fwd_intra_t<TIn, -1, -1>(p, nblocks, st);
}
template <class TIn>
static cudaError_t launch_fwd_out_m(const OpParams& p, float* o, int nblocks, cudaStream_t st) {
  if (p.dot_mode == GDN2_PREC_HIGHEST) return launch_fwd_out_t<TIn, GDN2_PREC_HIGHEST>(p, o, nblocks, st);
  if (p.dot_mode == GDN2_PREC_DEFAULT) return launch_fwd_out_t<TIn, GDN2_PREC_DEFAULT>(p, o, nblocks, st);
  return launch_fwd_out_t<TIn, -1>(p, o, nblocks, st);
}

cudaError_t launch_fwd_intra(const OpParams& p, bool bf16, int nblocks, cudaStream_t st) {
  return bf16 ? launch_fwd_intra_m<__nv_bfloat16>(p, nblocks, st) : launch_fwd_intra_m<float>(p, nblocks, st);
}
cudaError_t launch_fwd_out(const OpParams& p, bool bf16, float* o, int nblocks, cudaStream_t st) {
  return bf16 ? launch_fwd_out_m<__nv_bfloat16>(p, o, nblocks, st) : launch_fwd_out_m<float>(p, o, nblocks, st);
}

}  // namespace gdn2
