// Sequential inter-chunk state scans (sm_100a), one CTA per (b, h, 32-column tile of d_v).
//
// Forward:   h_{c+1} = M_c h_c + Bc_c             (h_pre of every chunk and h_final stored)
// Backward:  dh_c    = M_c^T dh_{c+1} + Cc_c       (dh entering every chunk from the right stored)
//
// Both are the same loop: the 128x128 transition operand of chunk c is a pre-encoded image
// (hi/lo parts in the tensor core's K-major layout, written by fwd_intra) that one thread copies
// into shared memory with a single bulk async copy while the previous chunk finishes; the state
// tile (128 x 32, fp32 in registers: thread d owns row d) is the MMA's B operand.  Column tiles
// of the state are independent because the transition acts on the d_k side only
// (fwd/cd_slim.py:23-31, bwd/mega.py:31-34).
#include "gdn2_kernels.cuh"

namespace gdn2 {

constexpr uint32_t kScanImg = 2 * 65536;                 // largest image (tf32, 3 passes)
constexpr uint32_t kScanB = 2 * 16384;                   // state tile hi + lo
constexpr uint32_t kScanSmem = 1024 + kScanImg + kScanB + 64;

// Transition images arrive by bulk copy.  When two images fit in the image area (every mode but
// 3 x tf32, whose hi + lo image fills it), they are double-buffered: chunk c + 1's image is copied
// while chunk c is computed, instead of after chunk c's MMA has released the one buffer.
//
// The state entering a chunk is stored to HBM either before its B-operand staging or, when the
// launch runs alone on the GPU (one batch group: sp.store_late), after its MMA has been issued, so
// that the stores overlap the MMA.  Measured per launch: the late store makes a forward scan of
// B4 H6 L2048 (3 x tf32) 0.056 instead of 0.059 ms and a 3-head step 0.340 instead of 0.350 ms,
// while with the batch groups' kernels beside the scan it made the whole 24-head step 1 % slower.

__global__ void __launch_bounds__(kThreads, 1) scan_kernel(const ScanParams sp) {
  pdl_enter();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* img_s = sm;
  uint8_t* b_s = sm + kScanImg;
  uint64_t* bar_ld = reinterpret_cast<uint64_t*>(sm + kScanImg + kScanB);  // one per image buffer
  uint64_t* bar_mma = bar_ld + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bar_ld + 3);

  const int t = threadIdx.x, warp = t >> 5;
  const int tiles = kD / kDV;
  const int bh = sp.bh0 + (int)(blockIdx.x / tiles), v0 = (blockIdx.x % tiles) * kDV;
  const Mode m = mode_from_enum(sp.mode);
  const uint32_t part = image_part_bytes(m);
  const uint32_t ibytes = image_bytes(m);
  const int nbuf = 2 * ibytes <= kScanImg ? 2 : 1;
  const bool lo = m.passes == 3;
  const size_t mat = (size_t)kD * kD;

  if (warp == 0) {
    tmem_alloc(tslot, 32);
    tmem_relinquish();
  }
  if (t == 0) {
    mbar_init(&bar_ld[0], 1);
    mbar_init(&bar_ld[1], 1);
    mbar_init(bar_mma, 1);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tb = *tslot;

  auto chunk_of = [&](int it) { return sp.reverse ? sp.NC - 1 - it : it; };
  auto issue_load = [&](int it) {  // the image of iteration it into its buffer
    const int bf = nbuf == 2 ? (it & 1) : 0;
    const uint8_t* src = sp.img + ((size_t)bh * sp.NC + chunk_of(it)) * sp.img_stride;
    uint8_t* dst = img_s + (uint32_t)bf * ibytes;
    mbar_arrive_expect_tx(&bar_ld[bf], ibytes);
    for (uint32_t o = 0; o < ibytes; o += 32768u) bulk_g2s(dst + o, src + o, 32768u, &bar_ld[bf]);
  };
  if (t == 0) {
    issue_load(0);
    if (nbuf == 2 && sp.NC > 1) issue_load(1);
  }

  // State row t, columns v0 .. v0+31.
  float h[kDV];
  if (sp.state_in) {
    const float* src = sp.state_in + (size_t)bh * mat + (size_t)t * kD + v0;
#pragma unroll
    for (int j = 0; j < kDV; j += 4) {
      float4 x = *reinterpret_cast<const float4*>(src + j);
      h[j] = x.x; h[j + 1] = x.y; h[j + 2] = x.z; h[j + 3] = x.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < kDV; ++j) h[j] = 0.f;
  }

  const Tile A0[2] = {tile_k(smem_u32(img_s), 128u * (uint32_t)esize(m)),
                      tile_k(smem_u32(img_s) + part, 128u * (uint32_t)esize(m))};
  const Tile A1[2] = {tile_k(smem_u32(img_s) + ibytes, 128u * (uint32_t)esize(m)),
                      tile_k(smem_u32(img_s) + ibytes + part, 128u * (uint32_t)esize(m))};
  const uint32_t bpart = (m.fmt == kTF32) ? 16384u : 8192u;
  const Tile Bt[2] = {tile_mn(smem_u32(b_s), kDV * (uint32_t)esize(m), m.fmt),
                      tile_mn(smem_u32(b_s) + bpart, kDV * (uint32_t)esize(m), m.fmt)};
  const int nsteps = 128 * esize(m) / 32;
  uint32_t ph_ld[2] = {0u, 0u}, ph_mma = 0;

  for (int it = 0; it < sp.NC; ++it) {
    const int c = chunk_of(it);
    // the state entering this chunk
    auto store_state = [&] {
      float* dst = sp.states + ((size_t)bh * sp.states_per_head + c) * mat + (size_t)t * kD + v0;
#pragma unroll
      for (int j = 0; j < kDV; j += 4) *reinterpret_cast<float4*>(dst + j) = make_float4(h[j], h[j + 1], h[j + 2], h[j + 3]);
    };
    if (!sp.store_late) store_state();
    // stage the state as the B operand (row t of the state = k index t)
#pragma unroll
    for (int j = 0; j < kDV; j += 8) stage_mnrow(Bt[0], Bt[1], lo, m.fmt, t, j, h + j, 8);
    // prefetch the additive term
    float add[kDV];
    {
      const float* src = sp.add + ((size_t)bh * sp.NC + c) * mat + (size_t)t * kD + v0;
#pragma unroll
      for (int j = 0; j < kDV; j += 4) {
        float4 x = __ldg(reinterpret_cast<const float4*>(src + j));
        add[j] = x.x; add[j + 1] = x.y; add[j + 2] = x.z; add[j + 3] = x.w;
      }
    }
    // Every thread sees this chunk's image land BEFORE the CTA barrier; the buffer is refilled
    // only after that barrier, so no thread can still be waiting on a phase when the next one
    // completes (a thread that tested the parity after the refill had landed would see it come
    // round again and wait for a phase that never completes).  Waiting in every thread here is
    // also faster than letting the issuing thread wait alone (measured: 0.059 against 0.070 ms
    // per forward scan of B4 H6 L2048, fp32).
    const int bf = nbuf == 2 ? (it & 1) : 0;
    mbar_wait(&bar_ld[bf], ph_ld[bf], sp.status);
    ph_ld[bf] ^= 1u;
    staged_sync();
    if (t == 0) {
      tc_fence_after();
      mma_tiles(m.fmt, m.passes, tb, bf ? A1 : A0, Bt, kDV, nsteps, false, false);
      mma_commit(bar_mma);
    }
    __syncwarp();  // park warp 0's other lanes here while lane 0 issues, instead of polling the barrier
    if (sp.store_late) store_state();
    mbar_wait(bar_mma, ph_mma, sp.status);
    ph_mma ^= 1u;
    tc_fence_after();
    // the buffer this MMA read is free: the image nbuf iterations ahead goes into it
    if (t == 0 && it + nbuf < sp.NC) issue_load(it + nbuf);
    float acc[32];
    tmem_ld32(tb, 0, acc);
#pragma unroll
    for (int j = 0; j < kDV; ++j) h[j] = sanitize(acc[j] + add[j], sp.clip);
    tc_fence_before();
    __syncthreads();  // all TMEM reads and B-tile reads done before the next iteration rewrites them
    tc_fence_after();
  }
  {
    float* dst = sp.final_out + (size_t)bh * mat + (size_t)t * kD + v0;
#pragma unroll
    for (int j = 0; j < kDV; j += 4) *reinterpret_cast<float4*>(dst + j) = make_float4(h[j], h[j + 1], h[j + 2], h[j + 3]);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tb, 32);
}

cudaError_t launch_scan(const ScanParams& sp, int BH, cudaStream_t st) {
  static unsigned long long done = 0;
  cudaError_t e = smem_attr_once(scan_kernel, (int)kScanSmem, done);
  if (e != cudaSuccess) return e;
  // A scan is the short sequential link in each batch group's chain of launches.  Launched
  // eagerly, it is dispatched ahead of the other groups' pending chunk-kernel CTAs (measured: the
  // un-graphed fwd+bwd step of B4 H6 L2048 fp32 0.994 against 1.022 ms); captured into a CUDA graph
  // the same priority made the replayed step 3 % slower, so captured launches keep the default.
  const bool urgent = stream_eager(st);
  e = launch_pdl_prio(scan_kernel, (unsigned)(BH * (kD / kDV)), kThreads, kScanSmem, st, urgent, sp);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace gdn2
