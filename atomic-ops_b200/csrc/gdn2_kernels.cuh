// Kernel parameter blocks, the residual / workspace layout, and the small CTA-level helpers
// shared by the forward and backward kernels.
#pragma once

#include "gdn2_common.cuh"

namespace gdn2 {

// Largest per-channel gate span (max_t gc - min_t gc inside one chunk) the single-reference
// factorisation accepts: every exponential leg stays within e^(+-kSpanMax/2), far inside the
// fp32 normal range, so hi/lo splits of the legs stay exact.
constexpr float kSpanMax = 128.0f;

// Bytes of one encoded 128x128 operand image (one precision part) for a mode.
__host__ __device__ inline uint32_t image_part_bytes(Mode m) { return m.fmt == kTF32 ? 65536u : 32768u; }
__host__ __device__ inline uint32_t image_bytes(Mode m) { return image_part_bytes(m) * (m.passes == 3 ? 2u : 1u); }

// Per-call residual layout (byte offsets from the residual base), all regions 256-byte aligned.
struct ResLayout {
  size_t aqk, ainv, wp, u, mf, bc, hs, vnew, total;
  uint32_t mf_stride;  // bytes per chunk-head of the forward state-transition image
};

__host__ __device__ inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

__host__ __device__ inline ResLayout res_layout(int BH, int NC, Mode fwd_scan) {
  ResLayout r{};
  const size_t nch = (size_t)BH * NC;
  const size_t mat = (size_t)kT * kD * 4;  // one 128x128 fp32 matrix
  size_t o = 0;
  r.aqk = o; o = align256(o + nch * mat);
  r.ainv = o; o = align256(o + nch * mat);
  r.wp = o; o = align256(o + nch * mat);
  r.u = o; o = align256(o + nch * mat);
  r.mf_stride = image_bytes(fwd_scan);
  r.mf = o; o = align256(o + nch * r.mf_stride);
  r.bc = o; o = align256(o + nch * mat);
  r.hs = o; o = align256(o + (size_t)BH * (NC + 1) * mat);  // h entering each chunk, then h_final
  r.vnew = o; o = align256(o + nch * mat);
  r.total = o;
  return r;
}

// Backward workspace layout.
struct WsLayout {
  size_t dvl, cc, dhs, mb, total;
  uint32_t mb_stride;  // bytes per chunk-head of the backward (transposed) transition image
};
__host__ __device__ inline WsLayout ws_layout(int BH, int NC, Mode bwd_scan) {
  WsLayout w{};
  const size_t nch = (size_t)BH * NC;
  const size_t mat = (size_t)kT * kD * 4;
  size_t o = 0;
  w.mb_stride = image_bytes(bwd_scan);
  w.mb = o; o = align256(o + nch * w.mb_stride);
  w.dvl = o; o = align256(o + nch * mat);
  w.cc = o; o = align256(o + nch * mat);
  w.dhs = o; o = align256(o + nch * mat);  // dh entering each chunk from the right
  w.total = o;
  return w;
}

struct OpParams {
  const void* q; const void* k; const void* v; const void* w; const void* b; const void* g;
  long long stride_b, stride_h;  // elements
  int H, NC;                     // heads, chunks in this call
  float scale, eps, clip;
  int dot_mode, solve_mode, b3_mode;
  unsigned* status;
  uint8_t* res;                  // residual base
  ResLayout rl;
};

// Element offset of chunk c of head (b, h) in a (B,H,L,D) tensor.
__device__ __forceinline__ long long chunk_off(const OpParams& p, int bh, int c) {
  const int b = bh / p.H, h = bh % p.H;
  return (long long)b * p.stride_b + (long long)h * p.stride_h + (long long)c * kT * kD;
}

// ---------------------------------------------------------------------------
// CTA helpers for the "stage -> issue -> wait" rhythm (single-buffered operand pool)
// ---------------------------------------------------------------------------
// Make the staged operands visible to the tensor core and order prior TMEM accesses.
__device__ __forceinline__ void staged_sync() {
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
}

struct MmaBar {
  uint64_t* bar;
  uint32_t phase;
  unsigned* status;
  __device__ __forceinline__ void commit_wait() {
    if (threadIdx.x == 0) mma_commit(bar);
    __syncwarp();
    mbar_wait(bar, phase, status);
    phase ^= 1u;
    tc_fence_after();
  }
};

// Element size in bytes and K elements per 128-byte slice.
__device__ __forceinline__ int esize(Mode m) { return m.fmt == kTF32 ? 4 : 2; }
__device__ __forceinline__ int kslice(Mode m) { return m.fmt == kTF32 ? 32 : 64; }

// Operand pool: tile i is 16 KB at base + i * 16 KB.
__device__ __forceinline__ Tile pool_k(uint32_t base, int i) { return tile_k(base + (uint32_t)i * 16384u, 128); }
__device__ __forceinline__ Tile pool_mn(uint32_t base, int i, Mode m) {
  return tile_mn(base + (uint32_t)i * 16384u, 128u * (uint32_t)esize(m), m.fmt);
}

// Issue one K-slice (4 MMA K-steps) for operand pairs stored in pool tiles.
__device__ __forceinline__ void issue_slice(Mode m, uint32_t dcol, const Tile a[2], const Tile b[2], int N,
                                            bool neg_a, bool accumulate) {
  mma_tiles(m.fmt, m.passes, dcol, a, b, N, 4, neg_a, accumulate);
}

// Write one value of an encoded image (hi/lo parts) of a 128x128 matrix in the K-major
// whole-K layout: element (row, col).  `dst` is the image base (hi part; lo part follows).
__device__ __forceinline__ uint32_t image_offset(Mode m, int row, int col) {
  const uint32_t e = (uint32_t)esize(m);
  const uint32_t kb = (uint32_t)col * e;
  const uint32_t sbo = 8u * 128u * e;
  return ((uint32_t)row >> 3) * sbo + (kb >> 4) * 128u + ((uint32_t)row & 7u) * 16u + (kb & 15u);
}

// Encode 8 consecutive values of row `row` (cols c0..c0+7) of a matrix into a K-major
// whole-K image in global memory (16-byte stores for bf16, two 16-byte stores for tf32).
__device__ __forceinline__ void image_store8(uint8_t* dst, Mode m, int row, int c0, const float v[8]) {
  const uint32_t part = image_part_bytes(m);
  if (m.fmt == kTF32) {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      uint4 hi, lo;
      uint32_t* ph = reinterpret_cast<uint32_t*>(&hi);
      uint32_t* pl = reinterpret_cast<uint32_t*>(&lo);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float x = v[4 * hh + i];
        ph[i] = tf32_rna(x);
        pl[i] = tf32_rna(x - __uint_as_float(ph[i]));
      }
      const uint32_t off = image_offset(m, row, c0 + 4 * hh);
      *reinterpret_cast<uint4*>(dst + off) = hi;
      if (m.passes == 3) *reinterpret_cast<uint4*>(dst + part + off) = lo;
    }
  } else {
    uint4 hi, lo;
    uint32_t* ph = reinterpret_cast<uint32_t*>(&hi);
    uint32_t* pl = reinterpret_cast<uint32_t*>(&lo);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 hv = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      float2 hf = __bfloat1622float2(hv);
      __nv_bfloat162 lv = __floats2bfloat162_rn(v[2 * i] - hf.x, v[2 * i + 1] - hf.y);
      ph[i] = *reinterpret_cast<uint32_t*>(&hv);
      pl[i] = *reinterpret_cast<uint32_t*>(&lv);
    }
    const uint32_t off = image_offset(m, row, c0);
    *reinterpret_cast<uint4*>(dst + off) = hi;
    if (m.passes == 3) *reinterpret_cast<uint4*>(dst + part + off) = lo;
  }
}

// Encode one scalar at (row, col) of an image (used to write a transpose from row owners).
__device__ __forceinline__ void image_store1(uint8_t* dst, Mode m, int row, int col, float x) {
  const uint32_t part = image_part_bytes(m);
  const uint32_t off = image_offset(m, row, col);
  if (m.fmt == kTF32) {
    const uint32_t h = tf32_rna(x);
    *reinterpret_cast<uint32_t*>(dst + off) = h;
    if (m.passes == 3) *reinterpret_cast<uint32_t*>(dst + part + off) = tf32_rna(x - __uint_as_float(h));
  } else {
    const __nv_bfloat16 h = __float2bfloat16_rn(x);
    *reinterpret_cast<__nv_bfloat16*>(dst + off) = h;
    if (m.passes == 3) *reinterpret_cast<__nv_bfloat16*>(dst + part + off) = __float2bfloat16_rn(x - __bfloat162float(h));
  }
}

// ---------------------------------------------------------------------------
// Chunk kernels run 256 threads: thread t owns row (t & 127) -- TMEM lane t & 127, reachable by
// warps w and w + 4 -- and half (t >> 7) of that row's columns.
// ---------------------------------------------------------------------------
constexpr int kCT = 256;
__device__ __forceinline__ int crow() { return threadIdx.x & 127; }
__device__ __forceinline__ int chalf() { return threadIdx.x >> 7; }

// Column-wise inclusive cumsum of the chunk's gate g (T x D) into shared memory
// gcs[t * kGcPitch + d].  The chunk is loaded cooperatively with coalesced 16-byte loads (all
// threads, many loads in flight), then thread d < 128 scans channel d in shared memory and
// returns the channel's max, min and whether a positive gate was seen.
// (pipeline.py:21 / ref.py:14: gc = cumsum(g) per chunk.)
constexpr int kGcPitch = 132;  // padded row pitch (floats): conflict-free row reads by row owners

template <class TIn>
__device__ __forceinline__ void chunk_cumsum(const TIn* __restrict__ g, float* gcs, float& mx, float& mn,
                                             bool& pos) {
  const int tid = threadIdx.x;
#pragma unroll 8
  for (int i = tid; i < kT * (kD / 4); i += kCT) {
    const int r = i >> 5, c4 = (i & 31) * 4;
    float v[4];
    ld4(g + r * kD + c4, v);
    *reinterpret_cast<float4*>(gcs + r * kGcPitch + c4) = make_float4(v[0], v[1], v[2], v[3]);
  }
  __syncthreads();
  mx = -3.0e38f;
  mn = 3.0e38f;
  pos = false;
  if (tid < kD) {
    float acc = 0.f;
#pragma unroll 8
    for (int t = 0; t < kT; ++t) {
      const float x = gcs[t * kGcPitch + tid];
      pos |= x > 0.f;
      acc += x;
      gcs[t * kGcPitch + tid] = acc;
      mx = fmaxf(mx, acc);
      mn = fminf(mn, acc);
    }
  }
}

// ---------------------------------------------------------------------------
// Generic K-loop over one or two operand pairs (all M = N = K = 128).
// Operands come from "row sources": src(row, c0, out16) returns 16 consecutive values of row
// `row` of the source matrix starting at column c0.
//   kmaj  : K-major; the source row is the operand's M/N row; every thread stages its own row
//           (its half of the slice's columns).  Works for TMEM-backed sources.
//   mn_any: MN-major; the source row is the operand's K row; any thread may fetch any row
//           (global- or shared-memory-backed sources): (row, 16-column group) items over all
//           threads.
//   mn_own: MN-major, TMEM-backed: the two warps owning the slice's lanes stage it, one half of
//           the MN columns each.
// ---------------------------------------------------------------------------
template <class Src>
struct Opnd {
  bool mn, any;
  Src src;
};
template <class Src>
__device__ __forceinline__ Opnd<Src> kmaj(Src s) { return Opnd<Src>{false, false, s}; }
template <class Src>
__device__ __forceinline__ Opnd<Src> mn_any(Src s) { return Opnd<Src>{true, true, s}; }
template <class Src>
__device__ __forceinline__ Opnd<Src> mn_own(Src s) { return Opnd<Src>{true, false, s}; }

// Work items of one operand slice (KS elements of K) for this thread: kmaj and mn_any operands
// both give every thread KS / 32 items of 16 values.
//   kmaj  : item p = columns [k0 + half * KS/2 + 16 p, +16) of the thread's own row
//   mn_any: item p = (row r, 16-column group) with it = tid + 256 p, r = it % KS, c0 = (it / KS) * 16
template <class Src>
__device__ __forceinline__ void fetch_item(const Opnd<Src>& op, int k0, int KS, int p, float* x) {
  if (!op.mn) {
    op.src(crow(), k0 + chalf() * (KS >> 1) + p * 16, x);
  } else if (op.any) {
    const int it = threadIdx.x + p * kCT;
    op.src(k0 + it % KS, (it / KS) * 16, x);
  }
}
template <int FMT, class Src>
__device__ __forceinline__ void store_item(const Tile tt[2], const Opnd<Src>& op, bool lo, int KS, int p,
                                           const float* x) {
  if (!op.mn) {
    stage_krow_t<FMT, 16>(tt[0], tt[1], lo, (uint32_t)crow(), chalf() * (KS >> 1) + p * 16, x);
  } else if (op.any) {
    const int it = threadIdx.x + p * kCT;
    stage_mnrow_t<FMT, 16>(tt[0], tt[1], lo, (uint32_t)(it % KS), (it / KS) * 16, x);
  }
}
// TMEM-backed MN-major operands: the two warps owning the slice's lanes, one half of MN each.
template <int FMT, class Src>
__device__ __forceinline__ void stage_own(const Tile tt[2], const Opnd<Src>& op, bool lo, int k0, int KS) {
  const int warp = threadIdx.x >> 5;
  if (op.mn && !op.any && (warp & 3) * 32 >= k0 && (warp & 3) * 32 < k0 + KS) {
    const int row = crow(), half = chalf();
#pragma unroll 1
    for (int c0 = half * 64; c0 < half * 64 + 64; c0 += 16) {
      float x[16];
      op.src(row, c0, x);
      stage_mnrow_t<FMT, 16>(tt[0], tt[1], lo, (uint32_t)(row - k0), c0, x);
    }
  }
}

// Register buffer for the prefetched items of one slice: up to two items (KS / 32) of two operands.
struct Prefetch {
  float x[2][2][16];
};
template <class S1, class S2>
__device__ __forceinline__ void prefetch2(Prefetch& pf, const Opnd<S1>& o1, const Opnd<S2>& o2, int k0, int KS) {
  const int np = KS / 32;
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    if (p < np) {
      fetch_item(o1, k0, KS, p, pf.x[0][p]);
      fetch_item(o2, k0, KS, p, pf.x[1][p]);
    }
  }
}
template <int FMT, class S1, class S2>
__device__ __forceinline__ void store2_t(const Prefetch& pf, const Tile* t1, const Opnd<S1>& o1, const Tile* t2,
                                         const Opnd<S2>& o2, bool lo, int KS) {
  const int np = KS / 32;
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    if (p < np) {
      store_item<FMT>(t1, o1, lo, KS, p, pf.x[0][p]);
      store_item<FMT>(t2, o2, lo, KS, p, pf.x[1][p]);
    }
  }
}
// Stage operands 3 and 4 (not prefetched) of one slice: loads of both issued before the stores.
template <int FMT, class S3, class S4>
__device__ __forceinline__ void stage34_t(const Tile* t3, const Opnd<S3>& o3, const Tile* t4, const Opnd<S4>& o4,
                                          int nops, bool lo, int k0, int KS) {
  const int np = KS / 32;
#pragma unroll 1
  for (int p = 0; p < np; ++p) {
    float x3[16], x4[16];
    if (nops > 2) fetch_item(o3, k0, KS, p, x3);
    if (nops > 3) fetch_item(o4, k0, KS, p, x4);
    if (nops > 2) store_item<FMT>(t3, o3, lo, KS, p, x3);
    if (nops > 3) store_item<FMT>(t4, o4, lo, KS, p, x4);
  }
}

// One K-loop of up to four operands (ops 1-2: pair 1's A and B, or A1 and the shared B; ops 3-4:
// the rest).  Software-pipelined: the global / shared loads of ops 1-2 for slice s+1 are issued
// right after slice s's MMAs, so their latency overlaps the tensor core; TMEM-backed MN-major
// operands are staged in the slice itself (TMEM loads are short).
template <int FMT, class S1, class S2, class S3, class S4, class Issue>
__device__ __forceinline__ void kloop_t(MmaBar& mb, const Tile* t1, const Opnd<S1>& o1, const Tile* t2,
                                        const Opnd<S2>& o2, const Tile* t3, const Opnd<S3>& o3, const Tile* t4,
                                        const Opnd<S4>& o4, int nops, bool lo, int KS, Issue issue) {
  const int ns = 128 / KS;
  Prefetch pf;
  prefetch2(pf, o1, o2, 0, KS);
  for (int s = 0; s < ns; ++s) {
    const int k0 = s * KS;
    store2_t<FMT>(pf, t1, o1, t2, o2, lo, KS);
    stage34_t<FMT>(t3, o3, t4, o4, nops, lo, k0, KS);
    stage_own<FMT>(t1, o1, lo, k0, KS);
    stage_own<FMT>(t2, o2, lo, k0, KS);
    if (nops > 2) stage_own<FMT>(t3, o3, lo, k0, KS);
    if (nops > 3) stage_own<FMT>(t4, o4, lo, k0, KS);
    staged_sync();
    if (threadIdx.x == 0) {
      tc_fence_after();
      issue(s);
      mma_commit(mb.bar);
    }
    __syncwarp();
    if (s + 1 < ns) prefetch2(pf, o1, o2, k0 + KS, KS);
    mbar_wait(mb.bar, mb.phase, mb.status);
    mb.phase ^= 1u;
    tc_fence_after();
  }
}

struct NoSrc {
  __device__ void operator()(int, int, float*) const {}
};

// D (+)= op(A) op(B), all M = N = K = 128, in K-slices of 128 bytes of mode m.
template <class SA, class SB>
__device__ __forceinline__ void gemm1(Mode m, uint32_t pool, MmaBar& mb, uint32_t d, const Opnd<SA>& a,
                                      const Opnd<SB>& b, bool neg, bool acc) {
  const int KS = kslice(m);
  Tile A[2], B[2];
  A[0] = a.mn ? pool_mn(pool, 0, m) : pool_k(pool, 0);
  A[1] = a.mn ? pool_mn(pool, 1, m) : pool_k(pool, 1);
  B[0] = b.mn ? pool_mn(pool, 2, m) : pool_k(pool, 2);
  B[1] = b.mn ? pool_mn(pool, 3, m) : pool_k(pool, 3);
  auto issue = [&](int s) { issue_slice(m, d, A, B, 128, neg, acc || s > 0); };
  const bool lo = m.passes == 3;
  if (m.fmt == kTF32) kloop_t<kTF32>(mb, A, a, B, b, A, a, B, b, 2, lo, KS, issue);
  else kloop_t<kBF16>(mb, A, a, B, b, A, a, B, b, 2, lo, KS, issue);
}

// Two products sharing the K-slicing: D1 (+)= A1 B1 and D2 (+)= A2 B2, where pair 2 reuses pair 1's
// staged A (share_a) or B (share_b) when set.  Tiles: A1 0-1, B1 2-3, then 4-5 (and 6-7).
template <class SA1, class SB1, class SA2, class SB2>
__device__ __forceinline__ void gemm2(Mode m, uint32_t pool, MmaBar& mb, uint32_t d1, const Opnd<SA1>& a1,
                                      const Opnd<SB1>& b1, bool neg1, bool acc1, uint32_t d2,
                                      const Opnd<SA2>& a2, const Opnd<SB2>& b2, bool neg2, bool acc2,
                                      bool share_a, bool share_b) {
  const int KS = kslice(m);
  auto tiles = [&](int i, bool mn, Tile out[2]) {
    out[0] = mn ? pool_mn(pool, i, m) : pool_k(pool, i);
    out[1] = mn ? pool_mn(pool, i + 1, m) : pool_k(pool, i + 1);
  };
  Tile A1[2], B1[2], A2[2], B2[2];
  tiles(0, a1.mn, A1);
  tiles(2, b1.mn, B1);
  int nt = 4;
  if (share_a) { A2[0] = A1[0]; A2[1] = A1[1]; } else { tiles(nt, a2.mn, A2); nt += 2; }
  if (share_b) { B2[0] = B1[0]; B2[1] = B1[1]; } else { tiles(nt, b2.mn, B2); nt += 2; }
  auto issue = [&](int s) {
    issue_slice(m, d1, A1, B1, 128, neg1, acc1 || s > 0);
    issue_slice(m, d2, A2, B2, 128, neg2, acc2 || s > 0);
  };
  const bool lo = m.passes == 3;
  if (m.fmt == kTF32) {
    if (share_a) kloop_t<kTF32>(mb, A1, a1, B1, b1, B2, b2, B2, b2, 3, lo, KS, issue);
    else if (share_b) kloop_t<kTF32>(mb, A1, a1, B1, b1, A2, a2, A2, a2, 3, lo, KS, issue);
    else kloop_t<kTF32>(mb, A1, a1, B1, b1, A2, a2, B2, b2, 4, lo, KS, issue);
  } else {
    if (share_a) kloop_t<kBF16>(mb, A1, a1, B1, b1, B2, b2, B2, b2, 3, lo, KS, issue);
    else if (share_b) kloop_t<kBF16>(mb, A1, a1, B1, b1, A2, a2, A2, a2, 3, lo, KS, issue);
    else kloop_t<kBF16>(mb, A1, a1, B1, b1, A2, a2, B2, b2, 4, lo, KS, issue);
  }
}

// ---------------------------------------------------------------------------
// Coalesced epilogues.  A thread's TMEM row (its lane) maps to one global row, so row-per-thread
// global accesses make every warp-wide 16-byte access touch 32 rows.  These helpers move a warp's
// 32 x 64 quarter of an accumulator through a warp-private buffer in the idle operand pool, after
// which lane l handles 4 consecutive columns of two rows per step (rows 2i + l / 16): each
// warp-wide access then covers two contiguous 256-byte row segments.
// ---------------------------------------------------------------------------
constexpr int kXPitch = 68;  // floats per buffered row (64 + 4: conflict-free 16-byte accesses)
__device__ __forceinline__ float* xbuf(uint8_t* pool_base) {
  return reinterpret_cast<float*>(pool_base) + (threadIdx.x >> 5) * 32 * kXPitch;
}
// This thread's 64-column half-row [cb, cb + 64) of TMEM slot `slot` -> the warp's buffer, row = lane.
__device__ __forceinline__ void tmem_to_xbuf(uint32_t slot, int cb, float* xb) {
  float* row = xb + (threadIdx.x & 31) * kXPitch;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float x[16];
    tmem_ld16(slot, (uint32_t)(cb + 16 * j), x);
#pragma unroll
    for (int i = 0; i < 16; i += 4)
      *reinterpret_cast<float4*>(row + 16 * j + i) = make_float4(x[i], x[i + 1], x[i + 2], x[i + 3]);
  }
  __syncwarp();
}
// Coalesced position of step i (0..15): the warp-local row (0..31) and column offset (0..60).
__device__ __forceinline__ int xrow(int i) { return 2 * i + ((threadIdx.x & 31) >> 4); }
__device__ __forceinline__ int xcol() { return 4 * (threadIdx.x & 15); }

// Row loaders (16 values)
template <class TIn>
__device__ __forceinline__ void ld16_in(const TIn* p, float* x) {
#pragma unroll
  for (int j = 0; j < 16; j += 4) ld4(p + j, x + j);
}
__device__ __forceinline__ void ld16_f(const float* p, float* x) {
#pragma unroll
  for (int j = 0; j < 16; j += 4) {
    float4 v = *reinterpret_cast<const float4*>(p + j);
    x[j] = v.x; x[j + 1] = v.y; x[j + 2] = v.z; x[j + 3] = v.w;
  }
}
__device__ __forceinline__ void st16_f(float* p, const float* x) {
#pragma unroll
  for (int j = 0; j < 16; j += 4) *reinterpret_cast<float4*>(p + j) = make_float4(x[j], x[j + 1], x[j + 2], x[j + 3]);
}
__device__ __forceinline__ void st16_out(float* p, const float* x) { st16_f(p, x); }
__device__ __forceinline__ void st16_out(__nv_bfloat16* p, const float* x) {
#pragma unroll
  for (int j = 0; j < 16; j += 4) st4(p + j, x + j);
}
// the 32-wide forms used by the scan / host-side helpers
__device__ __forceinline__ void ld32_f(const float* p, float* x) {
  ld16_f(p, x);
  ld16_f(p + 16, x + 16);
}

constexpr int kDV = 32;  // state columns per scan CTA

struct ScanParams {
  const uint8_t* img;      // per-chunk transition images, chunk-head stride img_stride bytes
  uint32_t img_stride;
  const float* add;        // per-chunk 128x128 additive term (Bc or Cc)
  const float* state_in;   // (BH, D, D) initial state, or nullptr for zeros
  float* states;           // per-chunk stored states: states[(bh * states_per_head + c) * D * D]
  int states_per_head;     // NC + 1 (forward) or NC (backward)
  int store_final_state;   // also store the final state at slot NC (forward)
  float* final_out;        // (BH, D, D)
  int NC;
  int mode;                // gdn2_precision of the products
  int reverse;
  float clip;
  unsigned* status;
};

cudaError_t launch_fwd_intra(const OpParams& p, bool bf16, int nblocks, cudaStream_t st);
cudaError_t launch_fwd_out(const OpParams& p, bool bf16, float* o, int nblocks, cudaStream_t st);
cudaError_t launch_scan(const ScanParams& sp, int BH, cudaStream_t st);

struct BwdParams {
  OpParams op;
  const float* d_o;        // (B,H,L,D) fp32 cotangent of o (same strides as the inputs)
  void* dq; void* dk; void* dv; void* dw; void* db; void* dg;  // (B,H,L,D) in the input dtype
  uint8_t* ws;             // backward workspace
  WsLayout wl;
};
cudaError_t launch_bwd_pre(const BwdParams& p, bool bf16, int nblocks, cudaStream_t st);
cudaError_t launch_bwd_intra(const BwdParams& p, bool bf16, int nblocks, cudaStream_t st);

}  // namespace gdn2
