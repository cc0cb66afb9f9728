// Chunk-parallel backward kernels of the GDN-2 operator (sm_100a).
//
// Reference: atomic_gdn2/bwd/mega.py:9-58 (B1 .. B5 per chunk, reverse loop) and bwd/b4.py
// (intra-chunk score backward).  The reverse dh recurrence of mega.py:31-34,
//     dh_c = qg^T (scale do) + dh_{c+1} e^gl - wp^T (Aqk^T do + kg dh_{c+1}),
// is rewritten as dh_c = M^T dh_{c+1} + Cc with the forward's transition M = diag(e^gl) - kg^T wp
// and the chunk-local Cc = scale qg^T do - wp^T (Aqk^T do), so that
//   bwd_pre    (chunk-parallel)  dvl = Aqk^T do and Cc,
//   scan       (gdn2_scan.cu)    the sequential dh recurrence, storing dh entering every chunk,
//   bwd_intra  (chunk-parallel)  everything else: dv_new, B3 (WY / inverse gradients), B4 and B5.
//
// bwd_intra folds the gate factors into the operands so that the six gradients accumulate in
// four tensor-memory accumulators.  B3's dA = dwp' kb^T + dv_new (w v)^T is evaluated as
// dv_new X^T with X = w v - kb h_pre (kb = b k e^gc), and A^T dwp' as -(A^T dv_new) h_pre^T, which
// saves one product; the two B4 products with k F share one staging of k F.  With m the chunk's per-channel reference point,
// E = e^(gc - m), F = e^(m - gc):
//   Dq  = E o [ do (scale e^m h_pre)^T          + scale dAqk (k F) ]            = dq
//   Dbk = E o [ A^T dwp'                        + dAkk (k F) ]                  = dL/d(b k)
//         with dwp' = -dv_new (e^m h_pre)^T  (so that A^T dwp' = dkb e^m)
//   Dk  = F o [ (E o Dbk o b) + v_new (e^(gl-m) dh_next)^T + scale dAqk^T (q E) + dAkk^T (b k E) ]
// and dgc = q o Dq + 2 (b k) o Dbk - k o Dk, plus, on the chunk's last row,
// sum_v dh_next[d, v] h_next[d, v] (the derivative through the chunk decay e^gl; it equals the
// reference's dgc_last + the last-row kg term, mega.py:43-49).  dg is the reverse cumsum of dgc
// (mega.py:51, B5).
#include <type_traits>

#include "gdn2_kernels.cuh"

namespace gdn2 {

constexpr uint32_t kPreSmem = 1024 + 6 * 16384 + kT * kGcPitch * 4 + 64;
constexpr uint32_t kBwdSmem = 1024 + 8 * 16384 + kT * kGcPitch * 4 + 7 * kD * 4 + 64;

__device__ __forceinline__ uint8_t* align1024b(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// ---------------------------------------------------------------------------------------
// bwd_pre: dvl = Aqk^T do,  Cc = scale qg^T do - wp^T dvl, and the transposed transition
// image M^T = diag(e^gl) - wp^T kg of the reverse scan      (b3_dot_mode, mega.py:31-34)
// ---------------------------------------------------------------------------------------
template <class TIn, int B3>
__global__ void __launch_bounds__(kCT, 1) bwd_pre_kernel(const BwdParams P) {
  pdl_enter();
  extern __shared__ uint8_t smem_raw[];
  const OpParams& p = P.op;
  uint8_t* sm = align1024b(smem_raw);
  const uint32_t pool = smem_u32(sm);
  float* gcs = reinterpret_cast<float*>(sm + 6 * 16384);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + 6 * 16384 + kT * kGcPitch * 4);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int t = crow(), cb = chalf() * 64;
  const int ch = p.ch0 + (int)blockIdx.x, bh = ch / p.NC, c = ch % p.NC;
  const long long off = chunk_off(p, bh, c);
  const TIn* q = reinterpret_cast<const TIn*>(p.q) + off;
  const TIn* k = reinterpret_cast<const TIn*>(p.k) + off;
  const TIn* g = reinterpret_cast<const TIn*>(p.g) + off;
  const float* do_ = P.d_o + off;
  const size_t mat = (size_t)kT * kD;
  const float* aqk_g = reinterpret_cast<const float*>(p.res + p.rl.aqk) + (size_t)ch * mat;
  const float* wp_g = reinterpret_cast<const float*>(p.res + p.rl.wp) + (size_t)ch * mat;
  float* dvl_g = reinterpret_cast<float*>(P.ws + P.wl.dvl) + (size_t)ch * mat;
  float* cc_g = reinterpret_cast<float*>(P.ws + P.wl.cc) + (size_t)ch * mat;
  uint8_t* mb_g = P.ws + P.wl.mb + (size_t)ch * P.wl.mb_stride;
  const Mode m3 = mode_from_enum(B3 >= 0 ? B3 : p.b3_mode);
  const float clip = p.clip, scale = p.scale;

  if (warp == 0) {
    tmem_alloc(tslot, 512);  // three accumulators (allocations are powers of two)
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
  const uint32_t S0 = tb, S1 = tb + 128, S2 = tb + 256;
  MmaBar mb{bar, 0u, p.status};

  // global row sources: 4 values of row r from column c0 (mn_any operands)
  auto src_aqk = [&](int r, int c0, float* x) { ld4_f(aqk_g + r * kT + c0, x); };
  auto src_do = [&](int r, int c0, float* x) { ld4_f(do_ + r * kD + c0, x); };
  auto src_qg = [&](int r, int c0, float* x) {
    ld4_in(q + r * kD + c0, x);
    const float* gr = gcs + r * kGcPitch + c0;
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = scale * sanitize(x[j] * ex(fminf(gr[j], 0.f)), clip);
  };
  auto src_kg = [&](int r, int c0, float* x) {  // sanitize(k e^min(gl - gc, 0))
    ld4_in(k + r * kD + c0, x);
    const float* gr = gcs + r * kGcPitch + c0;
    const float* gl = gcs + (kT - 1) * kGcPitch + c0;
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = sanitize(x[j] * ex(fminf(gl[j] - gr[j], 0.f)), clip);
  };
  auto src_wp = [&](int r, int c0, float* x) { ld4_f(wp_g + r * kD + c0, x); };

  // S0 = Aqk^T do, S1 = (scale qg)^T do   (shared B = do)
  gemm2(m3, pool, mb, S0, mn_any(src_aqk), mn_any(src_do), false, false, S1, mn_any(src_qg), mn_any(NoSrc()), false,
        false, false, true);
  if (threadIdx.x == 0) {  // L2 hints for the wp^T products below
    l2_prefetch(wp_g, kT * kD * 4);
    l2_prefetch(k, kT * kD * sizeof(TIn));
  }
  {
    float* xb = xbuf(sm);
    tmem_to_xbuf(S0, cb, xb);
    xb_flush(xb, dvl_g, kD, cb);
  }
  __syncthreads();  // the buffers live in the operand pool the next product stages into
  // S1 -= wp^T dvl  and  S2 = wp^T kg  (one staging of wp^T): Cc, and the transposed transition
  // of this chunk for the reverse scan, M^T = diag(e^gl) - wp^T kg.  dvl is read back from the tile
  // just written (L2), so that all warps stage it (from TMEM only the lane owners could)
  auto src_dvl_res = [&](int r, int c0, float* x) { ld4_cg(dvl_g + r * kD + c0, x); };
  gemm2(m3, pool, mb, S1, mn_any(src_wp), mn_any(src_dvl_res), true, true, S2, mn_any(NoSrc()), mn_any(src_kg), false,
        false, true, false);
  {
    float* xb = xbuf(sm);
    tmem_to_xbuf(S1, cb, xb);
    xb_flush(xb, cc_g, kD, cb);
  }
  {
    const float dec = ex(fminf(gcs[(kT - 1) * kGcPitch + t], 0.f));
    for (int c0 = cb; c0 < cb + 64; c0 += 16) {
      float x[16];
      tmem_ld16(S2, c0, x);
#pragma unroll
      for (int j = 0; j < 16; ++j) x[j] = ((c0 + j) == t ? dec : 0.f) - x[j];
      image_store8(mb_g, m3, t, c0, x);
      image_store8(mb_g, m3, t, c0 + 8, x + 8);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tb, 512);
}

// ---------------------------------------------------------------------------------------
// Wide channels (gate span inside the chunk > kSpanMax): exact B4 terms on the CUDA cores.
// ---------------------------------------------------------------------------------------
// Row i of  scale dAqk (k e^(gc_i - gc_j))  and  dAkk (k e^(gc_i - gc_j))  for the 16 channels
// c0..c0+15 (zero for channels that are not wide).  dAqk / dAkk rows come from TMEM (this
// thread's lane); every thread of the warp runs the same loads.
template <class TIn>
__device__ __forceinline__ void wide_dq_dbk(uint32_t aqk_slot, uint32_t akk_slot, const TIn* __restrict__ k,
                                            const float* gcs, const float* wide_s, int i, int c0, float scale,
                                            float* oq, float* ob) {
#pragma unroll
  for (int j = 0; j < 16; ++j) oq[j] = ob[j] = 0.f;
#pragma unroll 1
  for (int jc = 0; jc < kT; jc += 16) {
    float aq[16], ak[16];
    tmem_ld16(aqk_slot, (uint32_t)jc, aq);
    tmem_ld16(akk_slot, (uint32_t)jc, ak);
#pragma unroll 1
    for (int dd = 0; dd < 16; ++dd) {
      const int d = c0 + dd;
      if (wide_s[d] == 0.f) continue;
      const float gci = gcs[i * kGcPitch + d];
      float sq = 0.f, sb = 0.f;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int j = jc + e;
        const float w = (j <= i) ? ld1(k + j * kD + d) * ex(fminf(gci - gcs[j * kGcPitch + d], 0.f)) : 0.f;
        sq = fmaf(aq[e], w, sq);
        sb = fmaf(ak[e], w, sb);
      }
      oq[dd] += scale * sq;
      ob[dd] += sb;
    }
  }
}
// dk contribution of one wide channel d at row j (see step 13 of bwd_intra).
template <class TIn>
__device__ __forceinline__ float wide_dk(const float* dqT, const float* dkT, const TIn* __restrict__ q,
                                         const TIn* __restrict__ k, const TIn* __restrict__ b,
                                         const float* __restrict__ vnew_g, const float* __restrict__ dhn_g,
                                         const float* gcs, float gl, int j, int d, float scale) {
  float tv = 0.f;
#pragma unroll 4
  for (int v = 0; v < kD; ++v) tv = fmaf(vnew_g[j * kD + v], dhn_g[d * kD + v], tv);
  const float gcj = gcs[j * kGcPitch + d];
  float acc = ex(fminf(gl - gcj, 0.f)) * tv;
#pragma unroll 4
  for (int i = 0; i < kT; ++i) {
    if (i < j) continue;
    const float e = ex(fminf(gcs[i * kGcPitch + d] - gcj, 0.f));
    const float bk = ld1(b + i * kD + d) * ld1(k + i * kD + d);
    const float aq = dqT[j * kT + (i ^ (j & 31))], ak = dkT[j * kT + (i ^ (j & 31))];
    acc = fmaf((scale * aq * ld1(q + i * kD + d) + ak * bk), e, acc);
  }
  return acc;
}

// ---------------------------------------------------------------------------------------
// bwd_intra
// ---------------------------------------------------------------------------------------
// WIDE = false handles the chunks without wide channels, WIDE = true the others (flag written by
// the forward's fwd_intra); each launch returns at once in the other kind of chunk.
template <class TIn, int B3, bool WIDE>
__global__ void __launch_bounds__(kCT, 1) bwd_intra_kernel(const BwdParams P) {
  pdl_enter();
  extern __shared__ uint8_t smem_raw[];
  const OpParams& p = P.op;
  uint8_t* sm = align1024b(smem_raw);
  const uint32_t pool = smem_u32(sm);
  float* gcs = reinterpret_cast<float*>(sm + 8 * 16384);
  float* mid_s = gcs + kT * kGcPitch;  // per-channel reference m (0 for a wide channel)
  float* gl_s = mid_s + kD;
  float* extra_s = gl_s + kD;  // two halves of the last-row decay term
  float* mzE_s = extra_s + 2 * kD;  // m of the zeroed-when-wide E legs (+1e30: wide channel)
  float* mzF_s = mzE_s + kD;        // m of the F legs (-1e30: wide channel)
  float* wide_s = mzF_s + kD;       // 1 for a wide channel
  uint64_t* bar = reinterpret_cast<uint64_t*>(wide_s + kD);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int t = crow(), half = chalf(), cb = half * 64;
  const int ch = p.ch0 + (int)blockIdx.x, bh = ch / p.NC, c = ch % p.NC;
  if ((reinterpret_cast<const int*>(p.res + p.rl.wide)[ch] != 0) != WIDE) return;
  const long long off = chunk_off(p, bh, c);
  const TIn* q = reinterpret_cast<const TIn*>(p.q) + off;
  const TIn* k = reinterpret_cast<const TIn*>(p.k) + off;
  const TIn* v = reinterpret_cast<const TIn*>(p.v) + off;
  const TIn* w = reinterpret_cast<const TIn*>(p.w) + off;
  const TIn* b = reinterpret_cast<const TIn*>(p.b) + off;
  const TIn* g = reinterpret_cast<const TIn*>(p.g) + off;
  const float* do_ = P.d_o + off;
  TIn* dq = reinterpret_cast<TIn*>(P.dq) + off;
  TIn* dk = reinterpret_cast<TIn*>(P.dk) + off;
  TIn* dv = reinterpret_cast<TIn*>(P.dv) + off;
  TIn* dw = reinterpret_cast<TIn*>(P.dw) + off;
  TIn* db = reinterpret_cast<TIn*>(P.db) + off;
  TIn* dg = reinterpret_cast<TIn*>(P.dg) + off;
  const size_t mat = (size_t)kT * kD;
  const float* ainv_g = reinterpret_cast<const float*>(p.res + p.rl.ainv) + (size_t)ch * mat;
  const float* hpre_g = reinterpret_cast<const float*>(p.res + p.rl.hs) + ((size_t)bh * p.NC + c) * mat;
  // h after this chunk: the next chunk's stored entry state, or the call's final state
  const float* hnext_g = c + 1 < p.NC ? hpre_g + mat : P.h_final + (size_t)bh * mat;
  const float* vnew_g = reinterpret_cast<const float*>(p.res + p.rl.vnew) + (size_t)ch * mat;
  const float* dvl_g = reinterpret_cast<const float*>(P.ws + P.wl.dvl) + (size_t)ch * mat;
  const float* dhn_g = reinterpret_cast<const float*>(P.ws + P.wl.dhs) + (size_t)ch * mat;
  float* daqk_g = reinterpret_cast<float*>(P.ws + P.wl.daqk) + (size_t)ch * mat;
  float* dakk_g = reinterpret_cast<float*>(P.ws + P.wl.dakk) + (size_t)ch * mat;
  const Mode m3 = mode_from_enum(B3 >= 0 ? B3 : p.b3_mode);
  const Mode mh = mode_from_enum(GDN2_PREC_HIGHEST);  // B4 products are fixed at "highest" (mega.py:13)
  const float clip = p.clip, scale = p.scale;

  if (warp == 0) {
    tmem_alloc(tslot, 512);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  // L2 prefetch hints, about two products ahead of each chunk tile's first use (the kernel is
  // latency-bound; an L2 hit shortens the first K-slice of every product)
  constexpr uint32_t kInTile = kT * kD * sizeof(TIn), kF32Tile = kT * kD * 4;
  auto l2_ahead = [&](int stage) {
    if (tid != 0) return;
    if (stage == 0) {
      l2_prefetch(k, kInTile);
      l2_prefetch(dvl_g, kF32Tile);
      l2_prefetch(b, kInTile);
      l2_prefetch(hpre_g, kF32Tile);
    } else if (stage == 1) {
      l2_prefetch(w, kInTile);
      l2_prefetch(v, kInTile);
      l2_prefetch(ainv_g, kF32Tile);
    } else if (stage == 2) {
      l2_prefetch(do_, kF32Tile);
      l2_prefetch(vnew_g, kF32Tile);
    } else {
      l2_prefetch(q, kInTile);
    }
  };
  {
    float mx, mn;
    bool pos;
    chunk_cumsum(g, gcs, mx, mn, pos);
    l2_ahead(0);  // after the gate tile has landed: the hints would compete with its copies
    const bool wide = tid < kD && mx - mn > kSpanMax;
    if (tid < kD) {
      const float mid = 0.5f * (mx + mn);
      mid_s[tid] = wide ? 0.f : mid;
      mzE_s[tid] = wide ? 1e30f : mid;
      mzF_s[tid] = wide ? -1e30f : mid;
      wide_s[tid] = wide ? 1.f : 0.f;
    }
  }
  {
    // last-row decay term: sum_v dh_next[d, v] h_next[d, v] per channel d, one warp per row
    // (lane l reads columns 4l .. 4l+3: coalesced 512-byte row reads), stored in extra_s[d]
    // (extra_s[kD + d] stays 0).
    const int lane = tid & 31;
    float part[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int d = warp * 16 + i;
      float a[4], h[4];
      ld4_f(dhn_g + d * kD + 4 * lane, a);
      ld4_f(hnext_g + d * kD + 4 * lane, h);
      part[i] = a[0] * h[0] + a[1] * h[1] + a[2] * h[2] + a[3] * h[3];
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) part[i] += __shfl_xor_sync(0xffffffffu, part[i], o);
    }
    if (lane < 16) {
      float v = part[0];
#pragma unroll
      for (int i = 1; i < 16; ++i) v = (lane == i) ? part[i] : v;
      extra_s[warp * 16 + lane] = v;
      extra_s[kD + warp * 16 + lane] = 0.f;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid < kD) gl_s[tid] = gcs[(kT - 1) * kGcPitch + tid];
  __syncthreads();
  const uint32_t tb = *tslot;
  const uint32_t S0 = tb, S1 = tb + 128, S2 = tb + 256, S3 = tb + 384;
  MmaBar mb{bar, 0u, p.status};
  auto sync_all = [&]() {
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  };

  // ---- global row sources: 4 values of row r from column c0 (kany / mn_any operands) ----
  auto gcrow = [&](int r) { return gcs + r * kGcPitch; };
  auto src_kg = [&](int r, int c0, float* x) {
    ld4_in(k + r * kD + c0, x);
    const float* gr = gcrow(r) + c0;
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = sanitize(x[j] * ex(fminf(gl_s[c0 + j] - gr[j], 0.f)), clip);
  };
  auto src_dhn = [&](int r, int c0, float* x) { ld4_f(dhn_g + r * kD + c0, x); };
  auto src_h = [&](int r, int c0, float* x) { ld4_f(hpre_g + r * kD + c0, x); };
  auto src_kb = [&](int r, int c0, float* x) {  // b k e^min(gc, 0)
    float kv[4];
    ld4_in(b + r * kD + c0, x);
    ld4_in(k + r * kD + c0, kv);
    const float* gr = gcrow(r) + c0;
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = x[j] * kv[j] * ex(fminf(gr[j], 0.f));
  };
  auto src_hpre_em = [&](int r, int c0, float* x) {  // row d = r of e^m h_pre
    ld4_f(hpre_g + r * kD + c0, x);
    const float s = ex(mid_s[r]);
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] *= s;
  };
  auto src_dhn_gl = [&](int r, int c0, float* x) {  // row d = r of e^(gl-m) dh_next
    ld4_f(dhn_g + r * kD + c0, x);
    const float s = ex(gl_s[r] - mzE_s[r]);
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] *= s;
  };
  auto src_bkEz = [&](int r, int c0, float* x) {  // b k E, zero in wide channels (B4 operand)
    float kv[4];
    ld4_in(b + r * kD + c0, x);
    ld4_in(k + r * kD + c0, kv);
    const float* gr = gcrow(r) + c0;
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = x[j] * kv[j] * ex(gr[j] - mzE_s[c0 + j]);
  };
  auto src_qE = [&](int r, int c0, float* x) {  // scale q E, zero in wide channels
    ld4_in(q + r * kD + c0, x);
    const float* gr = gcrow(r) + c0;
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = scale * x[j] * ex(gr[j] - mzE_s[c0 + j]);
  };
  auto src_kF = [&](int r, int c0, float* x) {  // k F, zero in wide channels
    ld4_in(k + r * kD + c0, x);
    const float* gr = gcrow(r) + c0;
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = x[j] * ex(mzF_s[c0 + j] - gr[j]);
  };
  auto src_ainv = [&](int r, int c0, float* x) { ld4_f(ainv_g + r * kT + c0, x); };
  auto src_vnew = [&](int r, int c0, float* x) { ld4_f(vnew_g + r * kD + c0, x); };
  auto src_do = [&](int r, int c0, float* x) { ld4_f(do_ + r * kD + c0, x); };
  auto src_do_s = [&](int r, int c0, float* x) {
    ld4_f(do_ + r * kD + c0, x);
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] *= scale;
  };
  auto tm = [&](uint32_t slot) { return [=](int, int c0, float* x) { tmem_ld16(slot, (uint32_t)c0, x); }; };
  auto tm_scaled = [&](uint32_t slot) {
    return [=](int, int c0, float* x) {
      tmem_ld16(slot, (uint32_t)c0, x);
#pragma unroll
      for (int j = 0; j < 16; ++j) x[j] *= scale;
    };
  };

  l2_ahead(1);
  // 1. + 2. in one K-loop (independent products)                                    [B1, B3]
  //  1. S0 = dv_new = sanitize(dvl + kg dh_next)
  //  2. S1 = X = w v - kb h_pre  (kb = b k e^gc; X^T is v_new's pre-image under A: v_new = A X).
  //     With dwp' = -dv_new (h_pre)^T (the gate factors cancel), the reference's
  //     dA = dwp' kb^T + dv_new (w v)^T is dv_new X^T, and A^T dwp' (step 7) is -dwv h_pre^T.
  gemm2(m3, pool, mb, S0, kany(src_kg), mn_any(src_dhn), false, false, S1, kany(src_kb), mn_any(src_h), false, false,
        false, false);
  {
    float* xb = xbuf4(sm);
    xs_fill(xb, 0, w, kD, cb);
    xs_fill(xb, 1, w, kD, cb + 32);
    xs_fill(xb, 2, v, kD, cb);
    xs_fill(xb, 3, v, kD, cb + 32);
    xs_wait();
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float x[16], w4[16], v4[16];
      xs_get16(xb, j >> 1, 16 * (j & 1), w4);
      xs_get16(xb, 2 + (j >> 1), 16 * (j & 1), v4);
      tmem_ld16(S1, cb + 16 * j, x);
#pragma unroll
      for (int i = 0; i < 16; ++i) x[i] = w4[i] * v4[i] - x[i];
      tmem_st16(S1, cb + 16 * j, x);
    }
    __syncwarp();  // the warp's blocks are refilled below
    xs_fill(xb, 0, dvl_g, kD, cb);
    xs_fill(xb, 1, dvl_g, kD, cb + 32);
    xs_wait();
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float x[16], y[16];
      xs_get16(xb, j >> 1, 16 * (j & 1), y);
      tmem_ld16(S0, cb + 16 * j, x);
#pragma unroll
      for (int i = 0; i < 16; ++i) x[i] = sanitize(x[i] + y[i], clip);
      tmem_st16(S0, cb + 16 * j, x);
    }
  }
  sync_all();
  l2_ahead(2);
  // 3. + 4. in one K-loop (independent products):  S2 = dA = sanitize(dv_new X^T),
  //     S3 = dwv = A^T dv_new;  dw = dwv v, dv = dwv w  (dwv stays in S3 for step 7) [B3]
  gemm2(m3, pool, mb, S2, kmaj(tm(S0)), kmaj(tm(S1)), false, false, S3, mn_any(src_ainv), mn_own(tm(S0)), false,
        false, false, false);
  for (int c0 = cb; c0 < cb + 64; c0 += 16) {
    float x[16];
    tmem_ld16(S2, c0, x);
#pragma unroll
    for (int j = 0; j < 16; ++j) x[j] = sanitize(x[j], clip);
    tmem_st16(S2, c0, x);
  }
  {
    float* xb = xbuf(sm);
    tmem_to_xbuf(S3, cb, xb);
    const int r0 = (warp & 3) * 32;
#pragma unroll 8
    for (int i = 0; i < 16; ++i) {
      const int lr = xrow(i), c0 = cb + xcol();
      const float4 d4 = *reinterpret_cast<const float4*>(xb + lr * kXPitch + xcol());
      const float d[4] = {d4.x, d4.y, d4.z, d4.w};
      float vv[4], ww[4], y[4], z[4];
      ld4(v + (r0 + lr) * kD + c0, vv);
      ld4(w + (r0 + lr) * kD + c0, ww);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        y[e] = sanitize(d[e] * vv[e], clip);
        z[e] = sanitize(d[e] * ww[e], clip);
      }
      st4(dw + (r0 + lr) * kD + c0, y);
      st4(dv + (r0 + lr) * kD + c0, z);
    }
    sync_all();  // the buffers live in the operand pool the next product stages into
  }
  // 5. S0 = tmp = sanitize(dA A^T)                                                   [B3]
  gemm1(m3, pool, mb, S0, kmaj(tm(S2)), kany(src_ainv), false, false);
  for (int c0 = cb; c0 < cb + 64; c0 += 16) {
    float x[16];
    tmem_ld16(S0, c0, x);
#pragma unroll
    for (int j = 0; j < 16; ++j) x[j] = sanitize(x[j], clip);
    tmem_st16(S0, c0, x);
  }
  sync_all();
  l2_ahead(3);
  // 6. S2 = dAkk = sanitize(-(1-eps) A^T tmp) strict                                  [B3]
  gemm1(m3, pool, mb, S2, mn_any(src_ainv), mn_own(tm(S0)), true, false);
  {
    const float keep = 1.0f - p.eps;
    float* xb = xbuf(sm);
    for (int c0 = cb; c0 < cb + 64; c0 += 16) {
      float x[16];
      tmem_ld16(S2, c0, x);
#pragma unroll
      for (int j = 0; j < 16; ++j) x[j] = (c0 + j < t) ? sanitize(x[j] * keep, clip) : 0.f;
      tmem_st16(S2, c0, x);
      xb_put16(xb, c0 - cb, x);
    }
    xb_flush(xb, dakk_g, kT, cb);  // read back by step 12 (all warps stage it from there)
  }
  sync_all();
  // 7a + 9a (one staging of e^m h_pre):  S0 = A^T dwp' = -dwv (e^m h_pre)^T,
  //     S1 = scale do (e^m h_pre)^T  (the Dq accumulator from here on)                 [B3]
  gemm2(m3, pool, mb, S0, kmaj(tm(S3)), kany(src_hpre_em), true, false, S1, kany(src_do_s), kany(NoSrc()), false,
        false, false, true);
  // 8. S3 = dAqk = (do v_new^T) causal  (dwv, read by 7a, is no longer needed)       [B2]
  gemm1(m3, pool, mb, S3, kany(src_do), kany(src_vnew), false, false);
  {
    float* xb = xbuf(sm);
    for (int c0 = cb; c0 < cb + 64; c0 += 16) {
      float x[16];
      tmem_ld16(S3, c0, x);
#pragma unroll
      for (int j = 0; j < 16; ++j) x[j] = (c0 + j <= t) ? x[j] : 0.f;
      tmem_st16(S3, c0, x);
      xb_put16(xb, c0 - cb, x);
    }
    xb_flush(xb, daqk_g, kT, cb);  // read back by step 12
  }
  sync_all();
  // 7b + 9b. S0 += dAkk (k F),  S1 += scale dAqk (k F)    (one staging of k F)      [B4, highest]
  gemm2(mh, pool, mb, S0, kmaj(tm(S2)), mn_any(src_kF), false, true, S1, kmaj(tm_scaled(S3)), mn_any(NoSrc()),
        false, true, false, true);
  // 10.-11. finish dq and db;  S1 <- dgc partial;  S0 <- Dbk b E (pre-scaled dk partial).
  //     Wide channels (m = 0): their B4 terms were left out of the products above and are added
  //     exactly here, and S0 keeps Dbk b (their dk is finished without the F leg in step 13).
  auto ep1011 = [&](auto wide_tag) {
    constexpr bool kWide = decltype(wide_tag)::value;
    const float* gr = gcrow(t);
    float* xb = xbuf4(sm);
#pragma unroll 1
    for (int hh = 0; hh < 2; ++hh) {
      float q2[32], k2[32], b2[32];
      xs_fill(xb, 0, q, kD, cb + 32 * hh);
      xs_fill(xb, 1, k, kD, cb + 32 * hh);
      xs_fill(xb, 2, b, kD, cb + 32 * hh);
      xs_wait();
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        xs_get16(xb, 0, 16 * j, q2 + 16 * j);
        xs_get16(xb, 1, 16 * j, k2 + 16 * j);
        xs_get16(xb, 2, 16 * j, b2 + 16 * j);
      }
      __syncwarp();  // the blocks are reused for the outputs below
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int c0 = cb + 32 * hh + 16 * jj;
        const float* qv = q2 + 16 * jj;
        const float* kv = k2 + 16 * jj;
        const float* bv = b2 + 16 * jj;
        float x[16], y[16], E[16], dgcp[16], wq[16], wb[16];
        if constexpr (kWide) wide_dq_dbk(S3, S2, k, gcs, wide_s, t, c0, scale, wq, wb);
#pragma unroll
        for (int j = 0; j < 16; ++j) E[j] = ex(gr[c0 + j] - mid_s[c0 + j]);
        tmem_ld16(S1, c0, x);  // Dq / E
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          x[j] *= E[j];
          if constexpr (kWide) x[j] += wq[j];
          y[j] = sanitize(x[j], clip);
          dgcp[j] = qv[j] * x[j];
        }
        xb2_put16(xb, 0, 16 * jj, y);
        tmem_ld16(S0, c0, x);  // Dbk / E
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          x[j] *= E[j];
          if constexpr (kWide) x[j] += wb[j];
          y[j] = sanitize(x[j] * kv[j], clip);
          dgcp[j] += 2.f * bv[j] * kv[j] * x[j];
          if constexpr (kWide) x[j] = x[j] * bv[j] * (wide_s[c0 + j] != 0.f ? 1.f : E[j]);
          else x[j] = x[j] * bv[j] * E[j];
        }
        xb2_put16(xb, 1, 16 * jj, y);
        tmem_st16(S1, c0, dgcp);
        tmem_st16(S0, c0, x);
      }
      xb2_flush(xb, 0, dq, kD, cb + 32 * hh);
      xb2_flush(xb, 1, db, kD, cb + 32 * hh);
    }
  };
  ep1011(std::integral_constant<bool, WIDE>{});
  sync_all();
  // 12. S0 += v_new (e^(gl-m) dh_next)^T (B3)  +  scale dAqk^T (q E) + dAkk^T (bk E) (B4)
  gemm1(m3, pool, mb, S0, kany(src_vnew), kany(src_dhn_gl), false, true);
  //     dAqk^T and dAkk^T come back from the tiles steps 8 and 6 wrote (L2): all warps stage them, where
  //     from TMEM only the two warps owning a slice's lanes could
  auto src_daqk_res = [&](int r, int c0, float* x) { ld4_cg(daqk_g + r * kT + c0, x); };
  auto src_dakk_res = [&](int r, int c0, float* x) { ld4_cg(dakk_g + r * kT + c0, x); };
  gemm2(mh, pool, mb, S0, mn_any(src_daqk_res), mn_any(src_qE), false, true, S0, mn_any(src_dakk_res), mn_any(src_bkEz), false,
        true, false, false);
  // 13. dk = F o S0;  dgc = S1 - k o dk (+ decay term on the last row).  dgc overwrites this
  //     thread's own half-row of gcs (no other thread reads that row any more).
  if constexpr (!WIDE) {
    float* gr = gcs + t * kGcPitch;
    float k4[64];
    {
      float* xb = xbuf4(sm);
      xs_fill(xb, 0, k, kD, cb);
      xs_fill(xb, 1, k, kD, cb + 32);
      xs_wait();
#pragma unroll
      for (int j = 0; j < 4; ++j) xs_get16(xb, j >> 1, 16 * (j & 1), k4 + 16 * j);
      __syncwarp();  // the buffer is reused for dk below
    }
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int c0 = cb + 16 * jj;
      const float* kv = k4 + 16 * jj;
      float x[16], y[16], dgcp[16];
      tmem_ld16(S0, c0, x);
      tmem_ld16(S1, c0, dgcp);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        x[j] *= ex(mid_s[c0 + j] - gr[c0 + j]);
        y[j] = sanitize(x[j], clip);
        dgcp[j] -= kv[j] * x[j];
        if (t == kT - 1) dgcp[j] += extra_s[c0 + j] + extra_s[kD + c0 + j];
      }
      xb_put16(xbuf4(sm), c0 - cb, y);
#pragma unroll
      for (int j = 0; j < 16; ++j) gr[c0 + j] = dgcp[j];
    }
    xb_flush(xbuf4(sm), dk, kD, cb);
  } else {
    // Wide channels: dk[j,d] = (Dbk b)[j,d] + e^(gl-gc[j,d]) (v_new dh_next^T)[j,d]
    //   + sum_{i>=j} (scale dAqk[i,j] q[i,d] + dAkk[i,j] (b k)[i,d]) e^(gc[i,d]-gc[j,d]),
    // with dAqk / dAkk read by column from transposed copies in the (idle) operand pool.
    float* dqT = reinterpret_cast<float*>(sm);
    float* dkT = dqT + kT * kT;
#pragma unroll 1
    for (int c0 = cb; c0 < cb + 64; c0 += 16) {
      float a1[16], a2[16];
      tmem_ld16(S3, c0, a1);
      tmem_ld16(S2, c0, a2);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int col = c0 + j;
        dqT[col * kT + (t ^ (col & 31))] = a1[j];
        dkT[col * kT + (t ^ (col & 31))] = a2[j];
      }
    }
    __syncthreads();
    const float* gr = gcs + t * kGcPitch;
    float dgc_keep[64];
#pragma unroll 1
    for (int jj = 0; jj < 4; ++jj) {
      const int c0 = cb + 16 * jj;
      float x[16], y[16], dgcp[16], kv[16];
      ld16_in(k + t * kD + c0, kv);
      tmem_ld16(S0, c0, x);
      tmem_ld16(S1, c0, dgcp);
#pragma unroll 1
      for (int j = 0; j < 16; ++j) {
        const int d = c0 + j;
        if (wide_s[d] != 0.f) {
          x[j] += wide_dk(dqT, dkT, q, k, b, vnew_g, dhn_g, gcs, gl_s[d], t, d, scale);
        } else {
          x[j] *= ex(mid_s[d] - gr[d]);
        }
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        y[j] = sanitize(x[j], clip);
        dgcp[j] -= kv[j] * x[j];
        if (t == kT - 1) dgcp[j] += extra_s[c0 + j] + extra_s[kD + c0 + j];
        dgc_keep[16 * jj + j] = dgcp[j];
      }
      st16_out(dk + t * kD + c0, y);
    }
    __syncthreads();  // every thread has read all of gcs; dgc may now overwrite it
    float* gw = gcs + t * kGcPitch;
#pragma unroll
    for (int j = 0; j < 64; ++j) gw[cb + j] = dgc_keep[j];
  }
  __syncthreads();  // all rows of dgc are in gcs
  // 14. dg = reverse cumsum of dgc over the chunk (B5)
  if (tid < kD) {
    float acc = 0.f;
#pragma unroll 8
    for (int r = kT - 1; r >= 0; --r) {
      acc += gcs[r * kGcPitch + tid];
      const float val = sanitize(acc, clip);
      if constexpr (sizeof(TIn) == 4) {
        dg[r * kD + tid] = val;
      } else {
        dg[r * kD + tid] = __float2bfloat16_rn(val);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tb, 512);
}

template <class TIn, int B3>
static cudaError_t launch_bwd_pre_t(const BwdParams& p, int nblocks, cudaStream_t st) {
  static unsigned long long done = 0;
  cudaError_t e = smem_attr_once(bwd_pre_kernel<TIn, B3>, (int)kPreSmem, done);
  if (e != cudaSuccess) return e;
  e = launch_pdl(bwd_pre_kernel<TIn, B3>, nblocks, kCT, kPreSmem, st, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}
template <class TIn, int B3, bool WIDE>
static cudaError_t launch_bwd_intra_t(const BwdParams& p, int nblocks, cudaStream_t st) {
  static unsigned long long done = 0;
  cudaError_t e = smem_attr_once(bwd_intra_kernel<TIn, B3, WIDE>, (int)kBwdSmem, done);
  if (e != cudaSuccess) return e;
  e = launch_pdl(bwd_intra_kernel<TIn, B3, WIDE>, nblocks, kCT, kBwdSmem, st, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}
// Compile-time precision for the reference's default B3 mode (bf16x3) and the all-bf16 mode.
template <class TIn>
static cudaError_t launch_bwd_pre_m(const BwdParams& p, int nblocks, cudaStream_t st) {
  if (p.op.b3_mode == GDN2_PREC_BF16X3) return launch_bwd_pre_t<TIn, GDN2_PREC_BF16X3>(p, nblocks, st);
  if (p.op.b3_mode == GDN2_PREC_DEFAULT) return launch_bwd_pre_t<TIn, GDN2_PREC_DEFAULT>(p, nblocks, st);
  return launch_bwd_pre_t<TIn, -1>(p, nblocks, st);
}
template <class TIn>
static cudaError_t launch_bwd_intra_m(const BwdParams& p, int nblocks, cudaStream_t st) {
  cudaError_t e;
  if (p.op.b3_mode == GDN2_PREC_BF16X3) e = launch_bwd_intra_t<TIn, GDN2_PREC_BF16X3, false>(p, nblocks, st);
  else if (p.op.b3_mode == GDN2_PREC_DEFAULT) e = launch_bwd_intra_t<TIn, GDN2_PREC_DEFAULT, false>(p, nblocks, st);
  else e = launch_bwd_intra_t<TIn, -1, false>(p, nblocks, st);
  if (e != cudaSuccess) return e;
  return launch_bwd_intra_t<TIn, -1, true>(p, nblocks, st);  // chunks with wide channels
}

cudaError_t launch_bwd_pre(const BwdParams& p, bool bf16, int nblocks, cudaStream_t st) {
  return bf16 ? launch_bwd_pre_m<__nv_bfloat16>(p, nblocks, st) : launch_bwd_pre_m<float>(p, nblocks, st);
}
cudaError_t launch_bwd_intra(const BwdParams& p, bool bf16, int nblocks, cudaStream_t st) {
  return bf16 ? launch_bwd_intra_m<__nv_bfloat16>(p, nblocks, st) : launch_bwd_intra_m<float>(p, nblocks, st);
}

}  // namespace gdn2
