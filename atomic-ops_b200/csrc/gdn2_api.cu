// C-ABI entry points: argument validation, residual / workspace layout and kernel orchestration.
#include <atomic>
#include <cstdlib>
#include <mutex>
#include <vector>

#include "gdn2_kernels.cuh"

using namespace gdn2;

extern "C" const char* gdn2_status_string(gdn2_status status) {
  switch (status) {
    case GDN2_OK: return "ok";
    case GDN2_ERR_INVALID_ARGUMENT: return "invalid argument";
    case GDN2_ERR_CUDA: return "CUDA error";
    case GDN2_ERR_UNSUPPORTED: return "unsupported configuration";
  }
  return "unknown status";
}

namespace {

bool mode_ok(int32_t m) { return m >= GDN2_PREC_HIGHEST && m <= GDN2_PREC_TF32; }

}  // namespace

namespace gdn2 {

// Shape / config validation shared by every entry point (the reference raises ValueError for a
// sequence length that is not a multiple of bt, pipeline.py:54-55, and for bad configs,
// config.py:52-65).
gdn2_status check_desc(const gdn2_desc* d) {
  if (!d) return GDN2_ERR_INVALID_ARGUMENT;
  if (d->B <= 0 || d->H <= 0 || d->L <= 0 || d->D <= 0 || d->bt <= 0) return GDN2_ERR_INVALID_ARGUMENT;
  if (d->L % d->bt) return GDN2_ERR_INVALID_ARGUMENT;
  if (!mode_ok(d->dot_mode) || !mode_ok(d->solve_dot_mode) || !mode_ok(d->b3_dot_mode))
    return GDN2_ERR_INVALID_ARGUMENT;
  if (d->in_dtype != GDN2_F32 && d->in_dtype != GDN2_BF16) return GDN2_ERR_INVALID_ARGUMENT;
  if (!(d->wy_eps >= 0.f && d->wy_eps < 1.f) || !(d->clip > 0.f)) return GDN2_ERR_INVALID_ARGUMENT;
  if (d->stride_h < (int64_t)d->L * d->D || d->stride_b < (int64_t)d->H * d->stride_h) {
    if (!(d->H == 1 && d->stride_h >= (int64_t)d->L * d->D)) return GDN2_ERR_INVALID_ARGUMENT;
  }
  if ((d->stride_h % 8) || (d->stride_b % 8)) return GDN2_ERR_INVALID_ARGUMENT;
  // This build implements the operator's production geometry: 128-token chunks, 128-wide heads.
  if (d->bt != kT || d->D != kD) return GDN2_ERR_UNSUPPORTED;
  return GDN2_OK;
}

}  // namespace gdn2

namespace {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool aligned256(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 255u) == 0; }

OpParams make_params(const gdn2_desc* d, const void* q, const void* k, const void* v, const void* w,
                     const void* b, const void* g, void* residual, uint32_t* status) {
  OpParams p{};
  p.q = q; p.k = k; p.v = v; p.w = w; p.b = b; p.g = g;
  p.stride_b = d->stride_b;
  p.stride_h = d->stride_h;
  p.H = d->H;
  p.NC = d->L / d->bt;
  p.scale = d->scale;
  p.eps = d->wy_eps;
  p.clip = d->clip;
  p.dot_mode = d->dot_mode;
  p.solve_mode = d->solve_dot_mode;
  p.b3_mode = d->b3_dot_mode;
  p.status = status;
  p.res = static_cast<uint8_t*>(residual);
  p.rl = res_layout(d->B * d->H, p.NC, mode_from_enum(d->dot_mode));
  return p;
}

// Optional per-kernel timing: CUDA events recorded on the launching stream around every kernel
// launch while enabled (gdn2_profile_enable), summed per kernel by gdn2_profile_collect.
struct KernelTimer {
  std::mutex mu;
  bool on = false;
  struct Rec { int id; cudaEvent_t a, b; };
  std::vector<Rec> recs;
  std::vector<cudaEvent_t> spare;
  cudaEvent_t get() {
    if (!spare.empty()) { cudaEvent_t e = spare.back(); spare.pop_back(); return e; }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
  }
};
KernelTimer& ktimer() { static KernelTimer t; return t; }

// Launch `f` (returns cudaError_t) bracketed by timing events when profiling is on.
template <class F>
cudaError_t timed(int id, cudaStream_t st, F f) {
  KernelTimer& kt = ktimer();
  if (!kt.on) return f();
  std::lock_guard<std::mutex> g(kt.mu);
  cudaEvent_t a = kt.get(), b = kt.get();
  cudaEventRecord(a, st);
  cudaError_t e = f();
  cudaEventRecord(b, st);
  kt.recs.push_back({id, a, b});
  return e;
}

}  // namespace

extern "C" void gdn2_profile_enable(int32_t enable) {
  KernelTimer& kt = ktimer();
  std::lock_guard<std::mutex> g(kt.mu);
  kt.on = enable != 0;
}

extern "C" int32_t gdn2_profile_collect(float* ms, int32_t* counts, int32_t n) {
  KernelTimer& kt = ktimer();
  std::lock_guard<std::mutex> g(kt.mu);
  for (int i = 0; i < n; ++i) { ms[i] = 0.f; counts[i] = 0; }
  int32_t total = 0;
  for (auto& r : kt.recs) {
    float t = 0.f;
    if (cudaEventSynchronize(r.b) == cudaSuccess && cudaEventElapsedTime(&t, r.a, r.b) == cudaSuccess &&
        r.id >= 0 && r.id < n) {
      ms[r.id] += t;
      counts[r.id] += 1;
      ++total;
    }
    kt.spare.push_back(r.a);
    kt.spare.push_back(r.b);
  }
  kt.recs.clear();
  return total;
}

namespace {

// ---------------------------------------------------------------------------------------------
// Batch groups.  The heads of a call are split into up to `groups` contiguous ranges whose launch
// sequences run on library-owned side streams, forked from and joined back to the caller's stream
// with events (so the call stays ordered on the caller's stream, and stream capture into a CUDA
// graph records the fork and the join).  One group's low-occupancy state scan and its chunk
// kernels' last-wave tails then overlap the other groups' chunk kernels (every head is an
// independent recurrence).
// ---------------------------------------------------------------------------------------------
constexpr int kMaxGroups = 8;
constexpr int kMaxDevs = 64;

int initial_groups() {
  const char* e = std::getenv("GDN2_STREAMS");
  int n = e ? std::atoi(e) : 6;
  return n < 1 ? 1 : (n > kMaxGroups ? kMaxGroups : n);
}
std::atomic<int> g_groups{initial_groups()};

struct DevStreams {
  std::mutex mu;
  bool ready = false;
  cudaStream_t side[kMaxGroups] = {};
  cudaEvent_t fork = nullptr;
  cudaEvent_t join[kMaxGroups] = {};
};
DevStreams g_dev_streams[kMaxDevs];

// Creates the side streams and events of the current device on first use (outside any capture).
DevStreams* dev_streams(cudaStream_t caller) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevs) return nullptr;
  DevStreams& ds = g_dev_streams[dev];
  std::lock_guard<std::mutex> g(ds.mu);
  if (ds.ready) return &ds;
  if (!stream_eager(caller)) return nullptr;
  bool ok = cudaEventCreateWithFlags(&ds.fork, cudaEventDisableTiming) == cudaSuccess;
  for (int i = 0; ok && i < kMaxGroups; ++i) {
    ok = cudaStreamCreateWithFlags(&ds.side[i], cudaStreamNonBlocking) == cudaSuccess &&
         cudaEventCreateWithFlags(&ds.join[i], cudaEventDisableTiming) == cudaSuccess;
  }
  ds.ready = ok;
  return ok ? &ds : nullptr;
}

// Streaming multiprocessors of the current device (looked up once per device).
int sm_count() {
  static std::atomic<int> cache[kMaxDevs];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevs) return 0;
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n == 0 && cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess) cache[dev].store(n);
  return n;
}

// Runs launch(first_head, n_heads, stream) for every group of the call's BH heads: on the caller's
// stream for a single group, else on forked side streams.  A call whose chunk-heads all fit in one
// wave of the GPU's SMs (the chunk kernels run one CTA per chunk-head and per SM) runs as one group:
// there is no wave tail for other groups to fill, and every group adds launches and events.
template <class F>
gdn2_status run_groups(int BH, int NC, cudaStream_t st, F launch) {
  int G = g_groups.load(std::memory_order_relaxed);
  if (G > BH) G = BH;
  if (G > 1 && (long long)BH * NC <= (long long)sm_count()) G = 1;
  DevStreams* ds = G > 1 ? dev_streams(st) : nullptr;
  if (!ds) G = 1;
  if (G == 1) return launch(0, BH, st) == cudaSuccess ? GDN2_OK : GDN2_ERR_CUDA;
  std::lock_guard<std::mutex> g(ds->mu);  // the fork / join events are shared by the device's calls
  if (cudaEventRecord(ds->fork, st) != cudaSuccess) return GDN2_ERR_CUDA;
  gdn2_status s = GDN2_OK;
  for (int i = 0; i < G; ++i) {
    const int h0 = (int)((long long)BH * i / G), h1 = (int)((long long)BH * (i + 1) / G);
    if (cudaStreamWaitEvent(ds->side[i], ds->fork, 0) != cudaSuccess) return GDN2_ERR_CUDA;
    if (s == GDN2_OK && launch(h0, h1 - h0, ds->side[i]) != cudaSuccess) s = GDN2_ERR_CUDA;
    // joined even after a failed launch, so that the caller's stream (and a capture) stays whole
    if (cudaEventRecord(ds->join[i], ds->side[i]) != cudaSuccess) return GDN2_ERR_CUDA;
    if (cudaStreamWaitEvent(st, ds->join[i], 0) != cudaSuccess) return GDN2_ERR_CUDA;
  }
  return s;
}

}  // namespace

extern "C" int32_t gdn2_set_batch_groups(int32_t n) {
  const int v = n < 1 ? 1 : (n > kMaxGroups ? kMaxGroups : n);
  return g_groups.exchange(v);
}

extern "C" int32_t gdn2_get_batch_groups(void) { return g_groups.load(); }

extern "C" size_t gdn2_residual_bytes(const gdn2_desc* d) {
  if (check_desc(d) != GDN2_OK) return 0;
  return res_layout(d->B * d->H, d->L / d->bt, mode_from_enum(d->dot_mode)).total;
}

extern "C" size_t gdn2_fwd_workspace_bytes(const gdn2_desc* d) {
  if (check_desc(d) != GDN2_OK) return 0;
  return res_layout(d->B * d->H, d->L / d->bt, mode_from_enum(d->dot_mode)).ws_total;
}

extern "C" size_t gdn2_bwd_workspace_bytes(const gdn2_desc* d) {
  if (check_desc(d) != GDN2_OK) return 0;
  return ws_layout(d->B * d->H, d->L / d->bt, mode_from_enum(d->b3_dot_mode)).total;
}

extern "C" gdn2_status gdn2_fwd(const gdn2_desc* d, const void* q, const void* k, const void* v, const void* w,
                                const void* b, const void* g, const float* h0, float* o, float* h_final,
                                void* residual, void* workspace, uint32_t* dev_status, void* stream) {
  gdn2_status s = check_desc(d);
  if (s != GDN2_OK) return s;
  const void* ins[] = {q, k, v, w, b, g, o, h_final};
  for (const void* x : ins)
    if (!x || !aligned16(x)) return GDN2_ERR_INVALID_ARGUMENT;
  if ((h0 && !aligned16(h0)) || !residual || !aligned256(residual) || !workspace || !aligned256(workspace) ||
      !dev_status)
    return GDN2_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf16 = d->in_dtype == GDN2_BF16;
  const OpParams base = make_params(d, q, k, v, w, b, g, residual, dev_status);
  const int BH = d->B * d->H, NC = base.NC;

  ScanParams sb{};
  sb.img = static_cast<uint8_t*>(workspace) + base.rl.mf;
  sb.img_stride = base.rl.mf_stride;
  sb.add = reinterpret_cast<const float*>(static_cast<uint8_t*>(workspace) + base.rl.bc);
  sb.state_in = h0;
  sb.states = reinterpret_cast<float*>(base.res + base.rl.hs);
  sb.states_per_head = NC;
  sb.final_out = h_final;
  sb.NC = NC;
  sb.mode = d->dot_mode;
  sb.reverse = 0;
  sb.clip = d->clip;
  sb.status = dev_status;

  return run_groups(BH, NC, st, [&](int h_first, int nh, cudaStream_t gs) -> cudaError_t {
    OpParams p = base;
    p.fws = static_cast<uint8_t*>(workspace);
    p.ch0 = h_first * NC;
    cudaError_t e = timed(GDN2_K_FWD_INTRA, gs, [&] { return launch_fwd_intra(p, bf16, nh * NC, gs); });
    if (e != cudaSuccess) return e;
    ScanParams sp = sb;
    sp.bh0 = h_first;
    sp.store_late = nh == BH;  // one batch group: the scan runs with no other group's kernels beside it
    e = timed(GDN2_K_FWD_SCAN, gs, [&] { return launch_scan(sp, nh, gs); });
    if (e != cudaSuccess) return e;
    return timed(GDN2_K_FWD_OUT, gs, [&] { return launch_fwd_out(p, bf16, o, nh * NC, gs); });
  });
}

extern "C" gdn2_status gdn2_bwd(const gdn2_desc* d, const void* q, const void* k, const void* v, const void* w,
                                const void* b, const void* g, const void* residual, const float* h_final,
                                const float* d_o, const float* d_hfinal, void* dq, void* dk, void* dv, void* dw,
                                void* db, void* dg, float* dh0, void* workspace, uint32_t* dev_status,
                                void* stream) {
  gdn2_status s = check_desc(d);
  if (s != GDN2_OK) return s;
  const void* ptrs[] = {q, k, v, w, b, g, h_final, d_o, dq, dk, dv, dw, db, dg, dh0};
  for (const void* x : ptrs)
    if (!x || !aligned16(x)) return GDN2_ERR_INVALID_ARGUMENT;
  if ((d_hfinal && !aligned16(d_hfinal)) || !residual || !aligned256(residual) || !workspace ||
      !aligned256(workspace) || !dev_status)
    return GDN2_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf16 = d->in_dtype == GDN2_BF16;
  BwdParams base{};
  base.op = make_params(d, q, k, v, w, b, g, const_cast<void*>(residual), dev_status);
  base.d_o = d_o;
  base.dq = dq; base.dk = dk; base.dv = dv; base.dw = dw; base.db = db; base.dg = dg;
  base.ws = static_cast<uint8_t*>(workspace);
  base.h_final = h_final;
  const int BH = d->B * d->H, NC = base.op.NC;
  base.wl = ws_layout(BH, NC, mode_from_enum(d->b3_dot_mode));

  ScanParams sb{};
  sb.img = base.ws + base.wl.mb;
  sb.img_stride = base.wl.mb_stride;
  sb.add = reinterpret_cast<const float*>(base.ws + base.wl.cc);
  sb.state_in = d_hfinal;
  sb.states = reinterpret_cast<float*>(base.ws + base.wl.dhs);
  sb.states_per_head = NC;
  sb.final_out = dh0;
  sb.NC = NC;
  sb.mode = d->b3_dot_mode;
  sb.reverse = 1;
  sb.clip = d->clip;
  sb.status = dev_status;

  return run_groups(BH, NC, st, [&](int h_first, int nh, cudaStream_t gs) -> cudaError_t {
    BwdParams bp = base;
    bp.op.ch0 = h_first * NC;
    cudaError_t e = timed(GDN2_K_BWD_PRE, gs, [&] { return launch_bwd_pre(bp, bf16, nh * NC, gs); });
    if (e != cudaSuccess) return e;
    ScanParams sp = sb;
    sp.bh0 = h_first;
    sp.store_late = nh == BH;
    e = timed(GDN2_K_BWD_SCAN, gs, [&] { return launch_scan(sp, nh, gs); });
    if (e != cudaSuccess) return e;
    return timed(GDN2_K_BWD_INTRA, gs, [&] { return launch_bwd_intra(bp, bf16, nh * NC, gs); });
  });
}
