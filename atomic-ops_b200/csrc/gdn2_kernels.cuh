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

// Per-call layouts of the forward's device memory (byte offsets), all regions 256-byte aligned.
// Residual (kept from the forward to the backward, read by bwd_pre / bwd_intra): the scores Aqk,
// the WY inverse A, wp = A (b k e^gc), the state entering every chunk (and h_final), v_new and
// the per-chunk-head wide-channel flags.  Forward workspace (dead once gdn2_fwd's launches have
// run): u = A (w v), the state-transition image M and the additive term Bc of the forward scan.
struct ResLayout {
  size_t aqk, ainv, wp, hs, vnew, wide, total;  // residual
  size_t u, mf, bc, ws_total;                   // forward workspace
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
  r.hs = o; o = align256(o + (size_t)BH * NC * mat);  // h entering each chunk (h_final is the output)
  r.vnew = o; o = align256(o + nch * mat);
  r.wide = o; o = align256(o + nch * sizeof(int));  // per chunk-head: 1 if it has wide channels
  r.total = o;
  o = 0;
  r.u = o; o = align256(o + nch * mat);
  r.mf_stride = image_bytes(fwd_scan);
  r.mf = o; o = align256(o + nch * r.mf_stride);
  r.bc = o; o = align256(o + nch * mat);
  r.ws_total = o;
  return r;
}

// Backward workspace layout.
struct WsLayout {
  size_t dvl, cc, dhs, daqk, dakk, mb, total;
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
  w.daqk = o; o = align256(o + nch * mat);  // bwd_intra's dAqk and dAkk, read back by its last product
  w.dakk = o; o = align256(o + nch * mat);
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
  uint8_t* fws;                  // forward workspace base (gdn2_fwd only)
  ResLayout rl;
  int ch0;                       // first chunk-head of this launch (batch groups split the heads)
};

// Element offset of chunk c of head bh = b * H + h in a (B,H,L,D) tensor.
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

// The MMA-completion barrier of a CTA and the parity of its next phase.  Every commit to it is
// preceded by a CTA barrier that all its waiters pass only after their previous wait, so no waiter
// can fall a whole phase behind.
struct MmaBar {
  uint64_t* bar;
  uint32_t phase;
  unsigned* status;
};

// Element size in bytes and K elements per 128-byte slice.
__device__ __forceinline__ int esize(Mode m) { return m.fmt == kTF32 ? 4 : 2; }
__device__ __forceinline__ int kslice(Mode m) { return m.fmt == kTF32 ? 32 : 64; }

// Operand pool: tile i is 16 KB at base + i * 16 KB (1024-byte aligned), swizzled layouts (see the
// staging engine below).  K-major: SWIZZLE_128B, SBO = 1024 (8 rows), one MMA K-step = 32 bytes.
// MN-major bf16: SWIZZLE_128B, LBO = 1024 (next 64 MN), SBO = 2048 (next 8 k), K-step = 16 k.
// MN-major tf32: SWIZZLE_128B_BASE32B (tile_mn).
__device__ __forceinline__ Tile pool_k(uint32_t base, int i) {
  return Tile{base + (uint32_t)i * 16384u, 16u, 1024u, 32u, false, 2u};
}
__device__ __forceinline__ Tile pool_mn(uint32_t base, int i, Mode m) {
  const uint32_t a = base + (uint32_t)i * 16384u;
  if (m.fmt == kTF32) return tile_mn(a, 512u, kTF32);
  return Tile{a, 1024u, 2048u, 4096u, true, 2u};
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
// gcs[t * kGcPitch + d].  The chunk is copied cooperatively (coalesced 16-byte copies, all
// threads, all in flight), then thread d < 128 scans channel d in shared memory and returns the
// channel's max, min and whether a positive gate was seen.
// (pipeline.py:21 / ref.py:14: gc = cumsum(g) per chunk.)
constexpr int kGcPitch = 132;  // padded row pitch (floats): conflict-free row reads by row owners

// The chunk's gate tile g (kT x kD) -> gcs (row pitch kGcPitch): fp32 by asynchronous copies
// (complete at chunk_cumsum_finish; the caller may issue other loads meanwhile), bf16 through
// registers.
__device__ __forceinline__ void chunk_gate_issue(const float* __restrict__ g, float* gcs) {
  const int tid = threadIdx.x;
#pragma unroll
  for (int i = tid; i < kT * (kD / 4); i += kCT) {
    const int r = i >> 5, c4 = (i & 31) * 4;
    cp_async16(gcs + r * kGcPitch + c4, g + r * kD + c4);
  }
}
__device__ __forceinline__ void chunk_gate_issue(const __nv_bfloat16* __restrict__ g, float* gcs) {
  const int tid = threadIdx.x;
#pragma unroll 8
  for (int i = tid; i < kT * (kD / 4); i += kCT) {
    const int r = i >> 5, c4 = (i & 31) * 4;
    float v[4];
    ld4(g + r * kD + c4, v);
    *reinterpret_cast<float4*>(gcs + r * kGcPitch + c4) = make_float4(v[0], v[1], v[2], v[3]);
  }
}
// In-place cumulative sum of gcs over the chunk's rows (one thread per channel), with the
// per-channel max / min of the cumsum and whether any gate is positive.
__device__ __forceinline__ void chunk_cumsum_finish(float* gcs, float& mx, float& mn, bool& pos) {
  const int tid = threadIdx.x;
  cp_async_wait_all();
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
template <class TIn>
__device__ __forceinline__ void chunk_cumsum(const TIn* __restrict__ g, float* gcs, float& mx, float& mn,
                                             bool& pos) {
  chunk_gate_issue(g, gcs);
  chunk_cumsum_finish(gcs, mx, mn, pos);
}

// ---------------------------------------------------------------------------
// Operand staging engine.  A product D (+)= A B (M = N = K = 128) runs in K-slices of 128 bytes
// per operand row (64 bf16 or 32 tf32 elements).  Every slice of every operand is written by the
// CTA's threads into 128-byte-swizzled tiles of the operand pool:
//   K-major tile (A, or B stored [n][k]): 128 rows of 128 bytes, 16-byte chunk j of row r at
//       chunk position j ^ (r & 7)                       (SWIZZLE_128B, SBO = 1024)
//   MN-major bf16 tile: atoms of 8 k-rows x 64 MN elements (128 bytes), chunk j of k-row r at
//       j ^ (r & 7); atoms along MN 1024 bytes apart, along K (8 rows) 2048  (SWIZZLE_128B)
//   MN-major tf32 tile: SWIZZLE_128B_BASE32B (the only MN-major tf32 layout; see Tile).
// Each 16-byte chunk position depends on the row, so a warp writing any 8 rows of one chunk
// column, or one row's 8 chunks, hits all 32 banks: conflict-free for both access patterns below.
//
// Operand kinds (all sources return consecutive values of one row of the source matrix):
//   kmaj  : K-major, TMEM- or shared-memory-backed; the source row is the operand's M/N row and
//           thread (row, half) stages its own row (src gives 16 values).
//   kany  : K-major, global-memory-backed; items of 4 consecutive K values laid out so that a
//           warp's 32 lanes read 512 contiguous bytes (two 256-byte row segments for bf16
//           slices, four 128-byte ones for tf32) -- fully coalesced (src gives 4 values).
//   mn_any: MN-major, global-backed; the source row is the operand's K row; a warp reads one
//           whole 128-element row per item (src gives 4 values).
//   mn_own: MN-major, TMEM-backed: the two warps owning the slice's K rows (TMEM lanes) stage
//           it, one half of the MN columns each (src gives 16 values).
// ---------------------------------------------------------------------------
enum OpKind { kKOwn = 0, kKAny = 1, kMnAny = 2, kMnOwn = 3 };
template <class Src>
struct Opnd {
  int kind;
  Src src;
  __device__ __forceinline__ bool mn() const { return kind >= kMnAny; }
};
template <class Src>
__device__ __forceinline__ Opnd<Src> kmaj(Src s) { return Opnd<Src>{kKOwn, s}; }
template <class Src>
__device__ __forceinline__ Opnd<Src> kany(Src s) { return Opnd<Src>{kKAny, s}; }
template <class Src>
__device__ __forceinline__ Opnd<Src> mn_any(Src s) { return Opnd<Src>{kMnAny, s}; }
template <class Src>
__device__ __forceinline__ Opnd<Src> mn_own(Src s) { return Opnd<Src>{kMnOwn, s}; }

template <int FMT>
struct SliceShape {
  static constexpr int KS = FMT == kTF32 ? 32 : 64;  // K elements per slice
  static constexpr int EB = FMT == kTF32 ? 4 : 2;    // element bytes
  static constexpr int NOWN = KS / 32;               // 16-value items per thread (kmaj)
  static constexpr int NANY = KS / 8;                // 4-value items per thread (kany, mn_any)
};

// Byte offset of element (mn, k) inside a K-major swizzled tile (k < KS).
template <int FMT>
__device__ __forceinline__ uint32_t off_k(uint32_t mn, uint32_t k) {
  const uint32_t kb = k * SliceShape<FMT>::EB;
  return mn * 128u + ((((kb >> 4) ^ mn) & 7u) << 4) + (kb & 15u);
}
// Byte offset of element (mn, k) inside an MN-major tile (MN = 128, k < KS).
template <int FMT>
__device__ __forceinline__ uint32_t off_mn(uint32_t mn, uint32_t k) {
  if constexpr (FMT == kTF32) {
    return (mn >> 5) * 512u + (k >> 2) * 2048u + (k & 3u) * 128u + (((((mn >> 3) ^ k) & 3u)) << 5) +
           (mn & 7u) * 4u;
  } else {
    return (k >> 3) * 2048u + (mn >> 6) * 1024u + (k & 7u) * 128u + (((((mn >> 3) ^ k) & 7u)) << 4) +
           (mn & 7u) * 2u;
  }
}

// Write 4 consecutive values (along the tile's contiguous axis) as hi (and lo) parts.
template <int FMT>
__device__ __forceinline__ void put4(uint32_t hi_addr, uint32_t lo_addr, bool lo, const float* v) {
  if constexpr (FMT == kTF32) {
    put_piece_t<kTF32>(hi_addr, lo ? lo_addr : 0u, v);
  } else {
    uint32_t h[2], l[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      __nv_bfloat162 hv = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      float2 hf = __bfloat1622float2(hv);
      __nv_bfloat162 lv = __floats2bfloat162_rn(v[2 * i] - hf.x, v[2 * i + 1] - hf.y);
      h[i] = *reinterpret_cast<uint32_t*>(&hv);
      l[i] = *reinterpret_cast<uint32_t*>(&lv);
    }
    asm volatile("st.shared.v2.b32 [%0], {%1,%2};" ::"r"(hi_addr), "r"(h[0]), "r"(h[1]) : "memory");
    if (lo) asm volatile("st.shared.v2.b32 [%0], {%1,%2};" ::"r"(lo_addr), "r"(l[0]), "r"(l[1]) : "memory");
  }
}
// Write 16 consecutive values (4 calls of put4 worth) along the contiguous axis.
template <int FMT>
__device__ __forceinline__ void put16_k(const Tile tt[2], bool lo, uint32_t mn, uint32_t k0, const float* v) {
  constexpr int W = FMT == kTF32 ? 4 : 8;
#pragma unroll
  for (int i = 0; i < 16; i += W) {
    const uint32_t o = off_k<FMT>(mn, k0 + i);
    put_piece_t<FMT>(tt[0].addr + o, lo ? tt[1].addr + o : 0u, v + i);
  }
}
template <int FMT>
__device__ __forceinline__ void put16_mn(const Tile tt[2], bool lo, uint32_t mn0, uint32_t k, const float* v) {
  constexpr int W = FMT == kTF32 ? 4 : 8;
#pragma unroll
  for (int i = 0; i < 16; i += W) {
    const uint32_t o = off_mn<FMT>(mn0 + i, k);
    put_piece_t<FMT>(tt[0].addr + o, lo ? tt[1].addr + o : 0u, v + i);
  }
}

// Coalesced item p of this thread: float index e of the slice's source block in row-major order.
__device__ __forceinline__ int any_e(int p) { return (p * kCT + (int)threadIdx.x) * 4; }

// Loads of one operand slice into registers (x holds 32 values: 2 x 16 or 8 x 4).
template <int FMT, class Src>
__device__ __forceinline__ void fetch_op(const Opnd<Src>& op, int k0, float* x) {
  using S = SliceShape<FMT>;
  if (op.kind == kKOwn) {
#pragma unroll
    for (int p = 0; p < S::NOWN; ++p) op.src(crow(), k0 + chalf() * (S::KS / 2) + 16 * p, x + 16 * p);
  } else if (op.kind == kKAny) {
#pragma unroll
    for (int p = 0; p < S::NANY; ++p) {
      const int e = any_e(p);
      op.src(e / S::KS, k0 + e % S::KS, x + 4 * p);
    }
  } else if (op.kind == kMnAny) {
#pragma unroll
    for (int p = 0; p < S::NANY; ++p) {
      const int e = any_e(p);
      op.src(k0 + (e >> 7), e & 127, x + 4 * p);
    }
  }
}
// Shared-memory stores of one operand slice from registers.
template <int FMT, class Src>
__device__ __forceinline__ void store_op(const Tile tt[2], const Opnd<Src>& op, bool lo, const float* x) {
  using S = SliceShape<FMT>;
  if (op.kind == kKOwn) {
#pragma unroll
    for (int p = 0; p < S::NOWN; ++p) put16_k<FMT>(tt, lo, (uint32_t)crow(), chalf() * (S::KS / 2) + 16 * p, x + 16 * p);
  } else if (op.kind == kKAny) {
#pragma unroll
    for (int p = 0; p < S::NANY; ++p) {
      const int e = any_e(p);
      const uint32_t o = off_k<FMT>((uint32_t)(e / S::KS), (uint32_t)(e % S::KS));
      put4<FMT>(tt[0].addr + o, tt[1].addr + o, lo, x + 4 * p);
    }
  } else if (op.kind == kMnAny) {
#pragma unroll
    for (int p = 0; p < S::NANY; ++p) {
      const int e = any_e(p);
      const uint32_t o = off_mn<FMT>((uint32_t)(e & 127), (uint32_t)(e >> 7));
      put4<FMT>(tt[0].addr + o, tt[1].addr + o, lo, x + 4 * p);
    }
  }
}
// TMEM-backed MN-major operands: the two warps owning the slice's lanes, one half of MN each.
template <int FMT, class Src>
__device__ __forceinline__ void stage_own(const Tile tt[2], const Opnd<Src>& op, bool lo, int k0) {
  const int warp = threadIdx.x >> 5;
  if (op.kind == kMnOwn && (warp & 3) * 32 >= k0 && (warp & 3) * 32 < k0 + SliceShape<FMT>::KS) {
    const int row = crow(), half = chalf();
#pragma unroll 1
    for (int c0 = half * 64; c0 < half * 64 + 64; c0 += 16) {
      float x[16];
      op.src(row, c0, x);
      put16_mn<FMT>(tt, lo, (uint32_t)c0, (uint32_t)(row - k0), x);
    }
  }
}

// One K-loop of up to four operands (ops 1-2: pair 1's A and B, or A1 and the shared B; ops 3-4:
// the rest).  Software-pipelined: the global loads of the next slice are issued right after a
// slice's MMAs, so their latency overlaps the tensor core.  A 64-value register buffer holds the
// prefetched slices of the first global operands (two for bf16 slices, four for tf32); TMEM- and
// shared-memory-backed operands, and global ones beyond the buffer, are staged inside the slice.
template <int FMT, class S1, class S2, class S3, class S4, class Issue>
__device__ __forceinline__ void kloop_t(MmaBar& mb, const Tile* t1, const Opnd<S1>& o1, const Tile* t2,
                                        const Opnd<S2>& o2, const Tile* t3, const Opnd<S3>& o3, const Tile* t4,
                                        const Opnd<S4>& o4, int nops, bool lo, Issue issue) {
  constexpr int KS = SliceShape<FMT>::KS;
  constexpr int ns = 128 / KS;
  constexpr int SLOT = FMT == kTF32 ? 16 : 32;  // values per operand slice and thread
  constexpr int NSLOT = 64 / SLOT;
  auto glob = [](int kind) { return kind == kKAny || kind == kMnAny; };
  int used = 0;
  const int p1 = (glob(o1.kind) && used < NSLOT) ? used++ : -1;
  const int p2 = (glob(o2.kind) && used < NSLOT) ? used++ : -1;
  const int p3 = (nops > 2 && glob(o3.kind) && used < NSLOT) ? used++ : -1;
  const int p4 = (nops > 3 && glob(o4.kind) && used < NSLOT) ? used++ : -1;
  float pf[64];
  auto prefetch = [&](int k0) {
    if (p1 >= 0) fetch_op<FMT>(o1, k0, pf + p1 * SLOT);
    if (p2 >= 0) fetch_op<FMT>(o2, k0, pf + p2 * SLOT);
    if (p3 >= 0) fetch_op<FMT>(o3, k0, pf + p3 * SLOT);
    if (p4 >= 0) fetch_op<FMT>(o4, k0, pf + p4 * SLOT);
  };
  auto stage_now = [&](const Tile* tt, const auto& op, int slot, int k0) {
    if (slot >= 0) {
      store_op<FMT>(tt, op, lo, pf + slot * SLOT);
    } else {
      float x[32];
      fetch_op<FMT>(op, k0, x);
      store_op<FMT>(tt, op, lo, x);
    }
  };
  prefetch(0);
  for (int s = 0; s < ns; ++s) {
    const int k0 = s * KS;
    stage_now(t1, o1, p1, k0);
    stage_now(t2, o2, p2, k0);
    if (nops > 2) stage_now(t3, o3, p3, k0);
    if (nops > 3) stage_now(t4, o4, p4, k0);
    stage_own<FMT>(t1, o1, lo, k0);
    stage_own<FMT>(t2, o2, lo, k0);
    if (nops > 2) stage_own<FMT>(t3, o3, lo, k0);
    if (nops > 3) stage_own<FMT>(t4, o4, lo, k0);
    staged_sync();
    if (threadIdx.x == 0) {
      tc_fence_after();
      issue(s);
      mma_commit(mb.bar);
    }
    __syncwarp();
    if (s + 1 < ns) prefetch(k0 + KS);
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
  Tile A[2], B[2];
  A[0] = a.mn() ? pool_mn(pool, 0, m) : pool_k(pool, 0);
  A[1] = a.mn() ? pool_mn(pool, 1, m) : pool_k(pool, 1);
  B[0] = b.mn() ? pool_mn(pool, 2, m) : pool_k(pool, 2);
  B[1] = b.mn() ? pool_mn(pool, 3, m) : pool_k(pool, 3);
  auto issue = [&](int s) { issue_slice(m, d, A, B, 128, neg, acc || s > 0); };
  const bool lo = m.passes == 3;
  if (m.fmt == kTF32) kloop_t<kTF32>(mb, A, a, B, b, A, a, B, b, 2, lo, issue);
  else kloop_t<kBF16>(mb, A, a, B, b, A, a, B, b, 2, lo, issue);
}

// Two products sharing the K-slicing: D1 (+)= A1 B1 and D2 (+)= A2 B2, where pair 2 reuses pair 1's
// staged A (share_a) or B (share_b) when set.  Tiles: A1 0-1, B1 2-3, then 4-5 (and 6-7).
template <class SA1, class SB1, class SA2, class SB2>
__device__ __forceinline__ void gemm2(Mode m, uint32_t pool, MmaBar& mb, uint32_t d1, const Opnd<SA1>& a1,
                                      const Opnd<SB1>& b1, bool neg1, bool acc1, uint32_t d2,
                                      const Opnd<SA2>& a2, const Opnd<SB2>& b2, bool neg2, bool acc2,
                                      bool share_a, bool share_b) {
  auto tiles = [&](int i, bool mn, Tile out[2]) {
    out[0] = mn ? pool_mn(pool, i, m) : pool_k(pool, i);
    out[1] = mn ? pool_mn(pool, i + 1, m) : pool_k(pool, i + 1);
  };
  Tile A1[2], B1[2], A2[2], B2[2];
  tiles(0, a1.mn(), A1);
  tiles(2, b1.mn(), B1);
  int nt = 4;
  if (share_a) { A2[0] = A1[0]; A2[1] = A1[1]; } else { tiles(nt, a2.mn(), A2); nt += 2; }
  if (share_b) { B2[0] = B1[0]; B2[1] = B1[1]; } else { tiles(nt, b2.mn(), B2); nt += 2; }
  auto issue = [&](int s) {
    issue_slice(m, d1, A1, B1, 128, neg1, acc1 || s > 0);
    issue_slice(m, d2, A2, B2, 128, neg2, acc2 || s > 0);
  };
  const bool lo = m.passes == 3;
  if (m.fmt == kTF32) {
    if (share_a) kloop_t<kTF32>(mb, A1, a1, B1, b1, B2, b2, B2, b2, 3, lo, issue);
    else if (share_b) kloop_t<kTF32>(mb, A1, a1, B1, b1, A2, a2, A2, a2, 3, lo, issue);
    else kloop_t<kTF32>(mb, A1, a1, B1, b1, A2, a2, B2, b2, 4, lo, issue);
  } else {
    if (share_a) kloop_t<kBF16>(mb, A1, a1, B1, b1, B2, b2, B2, b2, 3, lo, issue);
    else if (share_b) kloop_t<kBF16>(mb, A1, a1, B1, b1, A2, a2, A2, a2, 3, lo, issue);
    else kloop_t<kBF16>(mb, A1, a1, B1, b1, A2, a2, B2, b2, 4, lo, issue);
  }
}

// 4-value row loaders of the coalesced (kany / mn_any) sources
template <class TIn>
__device__ __forceinline__ void ld4_in(const TIn* p, float* x) { ld4(p, x); }
// 4 fp32 values written earlier by this kernel (L2, bypassing the incoherent read-only path)
__device__ __forceinline__ void ld4_cg(const float* p, float* x) {
  const float4 v = __ldcg(reinterpret_cast<const float4*>(p));
  x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
}
__device__ __forceinline__ void ld4_f(const float* p, float* x) {
  const float4 v = *reinterpret_cast<const float4*>(p);
  x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
}

// ---------------------------------------------------------------------------
// Coalesced epilogues.  A thread's TMEM row (its lane) maps to one global row, so row-per-thread
// global accesses make every warp-wide 16-byte access touch 32 rows.  These helpers move a warp's
// 32 x 64 quarter of an accumulator through a warp-private buffer in the idle operand pool, after
// which lane l handles 4 consecutive columns of two rows per step (rows 2i + l / 16): each
// warp-wide access then covers two contiguous 256-byte row segments.
// ---------------------------------------------------------------------------
constexpr int kXPitch = 68;   // floats per buffered row of a 32 x 64 block (conflict-free 16-byte accesses)
constexpr int kXPitch2 = 36;  // floats per buffered row of a 32 x 32 block
constexpr int kXSlot = 2304;  // floats per warp: one 32 x 64 block or two 32 x 32 blocks
__device__ __forceinline__ float* xbuf(uint8_t* pool_base) {
  return reinterpret_cast<float*>(pool_base) + (threadIdx.x >> 5) * kXSlot;
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
// Row-layout results into the buffer: this thread's row (its lane), 16 columns at local column c.
__device__ __forceinline__ void xb_put16(float* xb, int c, const float* x) {
  float* row = xb + (threadIdx.x & 31) * kXPitch + c;
#pragma unroll
  for (int i = 0; i < 16; i += 4) *reinterpret_cast<float4*>(row + i) = make_float4(x[i], x[i + 1], x[i + 2], x[i + 3]);
}
// 32-column variant: this thread's row, 16 columns at local column c (0 or 16) of block `blk` (0/1).
__device__ __forceinline__ void xb2_put16(float* xb, int blk, int c, const float* x) {
  float* row = xb + blk * 32 * kXPitch2 + (threadIdx.x & 31) * kXPitch2 + c;
#pragma unroll
  for (int i = 0; i < 16; i += 4) *reinterpret_cast<float4*>(row + i) = make_float4(x[i], x[i + 1], x[i + 2], x[i + 3]);
}
// Buffered 32 x 32 block `blk` -> global rows 32 (warp & 3) + r, columns c0..c0+31 (four 128-byte
// row segments per warp-wide store).
template <class TOut>
__device__ __forceinline__ void xb2_flush(float* xb, int blk, TOut* dst, int ld, int c0) {
  __syncwarp();
  const int r0 = ((threadIdx.x >> 5) & 3) * 32, lane = threadIdx.x & 31;
  const float* b = xb + blk * 32 * kXPitch2;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int lr = 4 * i + (lane >> 3), lc = 4 * (lane & 7);
    const float4 v4 = *reinterpret_cast<const float4*>(b + lr * kXPitch2 + lc);
    const float v[4] = {v4.x, v4.y, v4.z, v4.w};
    st4(dst + (size_t)(r0 + lr) * ld + c0 + lc, v);
  }
  __syncwarp();
}
// The warp's buffered 32 x 64 block -> global rows 32 (warp & 3) + r, columns cb..cb+63 of a
// matrix with row stride ld (coalesced: each warp-wide store covers two 256-byte row segments).
template <class TOut>
__device__ __forceinline__ void xb_flush(float* xb, TOut* dst, int ld, int cb) {
  __syncwarp();
  const int r0 = ((threadIdx.x >> 5) & 3) * 32;
#pragma unroll 8
  for (int i = 0; i < 16; ++i) {
    const int lr = xrow(i);
    const float4 v4 = *reinterpret_cast<const float4*>(xb + lr * kXPitch + xcol());
    const float v[4] = {v4.x, v4.y, v4.z, v4.w};
    st4(dst + (size_t)(r0 + lr) * ld + cb + xcol(), v);
  }
  __syncwarp();
}

// The reverse direction, for epilogues that combine an accumulator row with global operands:
// global rows 32 (warp & 3) + r, columns c0..c0+31 -> 32 x 32 block `blk` of a warp buffer (each
// warp-wide access covers four 128-byte row segments; fp32 by asynchronous copies), after which
// every lane reads its own row with xs_get16 (after xs_wait).  A thread's row read directly from
// global memory makes each warp-wide access touch 32 rows (32 L1 wavefronts), which made those
// loads the longest part of the epilogues.  Blocks are 1024 floats, 16-byte chunk j of row r at
// chunk position j ^ (r & 7): conflict-free for both access patterns.
__device__ __forceinline__ int xs_off(int r, int chunk) { return r * 32 + ((chunk ^ (r & 7)) << 2); }
__device__ __forceinline__ void xs_fill(float* xb, int blk, const float* src, int ld, int c0) {
  const int r0 = ((threadIdx.x >> 5) & 3) * 32, lane = threadIdx.x & 31;
  float* b = xb + blk * 1024;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int lr = 4 * i + (lane >> 3), ck = lane & 7;
    cp_async16(b + xs_off(lr, ck), src + (size_t)(r0 + lr) * ld + c0 + 4 * ck);
  }
}
__device__ __forceinline__ void xs_fill(float* xb, int blk, const __nv_bfloat16* src, int ld, int c0) {
  const int r0 = ((threadIdx.x >> 5) & 3) * 32, lane = threadIdx.x & 31;
  float* b = xb + blk * 1024;
  float v[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) ld4(src + (size_t)(r0 + 4 * i + (lane >> 3)) * ld + c0 + 4 * (lane & 7), v[i]);
#pragma unroll
  for (int i = 0; i < 8; ++i)
    *reinterpret_cast<float4*>(b + xs_off(4 * i + (lane >> 3), lane & 7)) = make_float4(v[i][0], v[i][1], v[i][2], v[i][3]);
}
__device__ __forceinline__ void xs_wait() {
  cp_async_wait_all();
  __syncwarp();
}
// This thread's row (its lane), 16 columns at local column c (0 or 16) of block `blk`.
__device__ __forceinline__ void xs_get16(const float* xb, int blk, int c, float* x) {
  const int r = threadIdx.x & 31;
  const float* b = xb + blk * 1024;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 v = *reinterpret_cast<const float4*>(b + xs_off(r, (c >> 2) + i));
    x[4 * i] = v.x; x[4 * i + 1] = v.y; x[4 * i + 2] = v.z; x[4 * i + 3] = v.w;
  }
}
// A warp buffer of four such blocks: warp w's region starts at w * 4096 floats of the operand pool.
__device__ __forceinline__ float* xbuf4(uint8_t* pool_base) {
  return reinterpret_cast<float*>(pool_base) + (threadIdx.x >> 5) * 4096;
}

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
  int states_per_head;     // NC
  float* final_out;        // (BH, D, D)
  int NC;
  int mode;                // gdn2_precision of the products
  int reverse;
  float clip;
  unsigned* status;
  int bh0;                 // first head of this launch
  int store_late;          // store each chunk's entering state under its MMA (launch runs alone)
};

// Descriptor validation shared by every C-ABI entry point (gdn2_api.cu).
gdn2_status check_desc(const gdn2_desc* d);

cudaError_t launch_fwd_intra(const OpParams& p, bool bf16, int nblocks, cudaStream_t st);
cudaError_t launch_fwd_out(const OpParams& p, bool bf16, float* o, int nblocks, cudaStream_t st);
cudaError_t launch_scan(const ScanParams& sp, int BH, cudaStream_t st);

struct BwdParams {
  OpParams op;
  const float* d_o;        // (B,H,L,D) fp32 cotangent of o (same strides as the inputs)
  void* dq; void* dk; void* dv; void* dw; void* db; void* dg;  // (B,H,L,D) in the input dtype
  uint8_t* ws;             // backward workspace
  WsLayout wl;
  const float* h_final;    // (BH, D, D) the forward's final state: h after the last chunk
};
cudaError_t launch_bwd_pre(const BwdParams& p, bool bf16, int nblocks, cudaStream_t st);
cudaError_t launch_bwd_intra(const BwdParams& p, bool bf16, int nblocks, cudaStream_t st);

}  // namespace gdn2
