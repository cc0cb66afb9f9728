// C-ABI entry points: argument validation, residual / workspace layout and kernel orchestration.
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

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool aligned256(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 255u) == 0; }
bool mode_ok(int32_t m) { return m >= GDN2_PREC_HIGHEST && m <= GDN2_PREC_TF32; }

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
  p.rl = res_layout(d->B * d->H, p.NC, mode_from_enum(d->dot_mode), mode_from_enum(d->b3_dot_mode));
  return p;
}

}  // namespace

extern "C" size_t gdn2_residual_bytes(const gdn2_desc* d) {
  if (check_desc(d) != GDN2_OK) return 0;
  return res_layout(d->B * d->H, d->L / d->bt, mode_from_enum(d->dot_mode), mode_from_enum(d->b3_dot_mode)).total;
}

extern "C" size_t gdn2_bwd_workspace_bytes(const gdn2_desc* d) {
  if (check_desc(d) != GDN2_OK) return 0;
  return ws_layout(d->B * d->H, d->L / d->bt).total;
}

extern "C" gdn2_status gdn2_fwd(const gdn2_desc* d, const void* q, const void* k, const void* v, const void* w,
                                const void* b, const void* g, const float* h0, float* o, float* h_final,
                                void* residual, uint32_t* dev_status, void* stream) {
  gdn2_status s = check_desc(d);
  if (s != GDN2_OK) return s;
  const void* ins[] = {q, k, v, w, b, g, o, h_final};
  for (const void* x : ins)
    if (!x || !aligned16(x)) return GDN2_ERR_INVALID_ARGUMENT;
  if ((h0 && !aligned16(h0)) || !residual || !aligned256(residual) || !dev_status) return GDN2_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf16 = d->in_dtype == GDN2_BF16;
  const OpParams p = make_params(d, q, k, v, w, b, g, residual, dev_status);
  const int BH = d->B * d->H, NC = p.NC;

  if (launch_fwd_intra(p, bf16, BH * NC, st) != cudaSuccess) return GDN2_ERR_CUDA;

  ScanParams sp{};
  sp.img = p.res + p.rl.mf;
  sp.img_stride = p.rl.mf_stride;
  sp.add = reinterpret_cast<const float*>(p.res + p.rl.bc);
  sp.state_in = h0;
  sp.states = reinterpret_cast<float*>(p.res + p.rl.hs);
  sp.states_per_head = NC + 1;
  sp.store_final_state = 1;
  sp.final_out = h_final;
  sp.NC = NC;
  sp.mode = d->dot_mode;
  sp.reverse = 0;
  sp.clip = d->clip;
  sp.status = dev_status;
  if (launch_scan(sp, BH, st) != cudaSuccess) return GDN2_ERR_CUDA;

  if (launch_fwd_out(p, bf16, o, BH * NC, st) != cudaSuccess) return GDN2_ERR_CUDA;
  return GDN2_OK;
}

extern "C" gdn2_status gdn2_bwd(const gdn2_desc* d, const void* q, const void* k, const void* v, const void* w,
                                const void* b, const void* g, const void* residual, const float* d_o,
                                const float* d_hfinal, void* dq, void* dk, void* dv, void* dw, void* db, void* dg,
                                float* dh0, void* workspace, uint32_t* dev_status, void* stream) {
  gdn2_status s = check_desc(d);
  if (s != GDN2_OK) return s;
  const void* ptrs[] = {q, k, v, w, b, g, d_o, dq, dk, dv, dw, db, dg, dh0};
  for (const void* x : ptrs)
    if (!x || !aligned16(x)) return GDN2_ERR_INVALID_ARGUMENT;
  if ((d_hfinal && !aligned16(d_hfinal)) || !residual || !aligned256(residual) || !workspace ||
      !aligned256(workspace) || !dev_status)
    return GDN2_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf16 = d->in_dtype == GDN2_BF16;
  BwdParams bp{};
  bp.op = make_params(d, q, k, v, w, b, g, const_cast<void*>(residual), dev_status);
  bp.d_o = d_o;
  bp.dq = dq; bp.dk = dk; bp.dv = dv; bp.dw = dw; bp.db = db; bp.dg = dg;
  bp.ws = static_cast<uint8_t*>(workspace);
  const int BH = d->B * d->H, NC = bp.op.NC;
  bp.wl = ws_layout(BH, NC);

  if (launch_bwd_pre(bp, bf16, BH * NC, st) != cudaSuccess) return GDN2_ERR_CUDA;

  ScanParams sp{};
  sp.img = bp.op.res + bp.op.rl.mb;
  sp.img_stride = bp.op.rl.mb_stride;
  sp.add = reinterpret_cast<const float*>(bp.ws + bp.wl.cc);
  sp.state_in = d_hfinal;
  sp.states = reinterpret_cast<float*>(bp.ws + bp.wl.dhs);
  sp.states_per_head = NC;
  sp.store_final_state = 0;
  sp.final_out = dh0;
  sp.NC = NC;
  sp.mode = d->b3_dot_mode;
  sp.reverse = 1;
  sp.clip = d->clip;
  sp.status = dev_status;
  if (launch_scan(sp, BH, st) != cudaSuccess) return GDN2_ERR_CUDA;

  if (launch_bwd_intra(bp, bf16, BH * NC, st) != cudaSuccess) return GDN2_ERR_CUDA;
  return GDN2_OK;
}
