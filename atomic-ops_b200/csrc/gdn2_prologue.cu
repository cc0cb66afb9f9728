// Fused GDN-2 layer prologue (sm_100a): the elementwise / per-row work between the layer's
// input projection and the operator (atomic_gdn2/layer.py:31-40), forward and backward.
//
//   y (B, L, 6, H, D) fp32, the six projections q | k | v | w | b | g side by side per token
//   q = y_q / sqrt(sum_d y_q^2 + 1e-6)     (if l2norm; else y_q)
//   k = y_k / sqrt(sum_d y_k^2 + 1e-6)     (if l2norm; else y_k)
//   v = y_v,  w = y_w
//   b = sigmoid(y_b)
//   g = -min(softplus(y_g), g_max)
// written as six (B, H, L, D) tensors (the operator's layout).  The backward recomputes the
// activations from y and writes dy in y's layout:
//   dy_q = (dq - q (q . dq)) / n_q,  dy_k likewise,  dy_v = dv,  dy_w = dw,
//   dy_b = db s (1 - s) with s = sigmoid(y_b),
//   dy_g = -dg sigmoid(y_g) where softplus(y_g) <= g_max, else 0.
//
// HBM-bound: one warp per (token, head) row; every lane moves one float4 of each of the six
// 512-byte rows, so all loads and stores are fully coalesced; the two L2 norms are warp
// reductions.  Bytes: forward 2 x 6 x 4 D per row, backward 3 x 6 x 4 D per row.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "gdn2_b200.h"

namespace gdn2 {
namespace {

constexpr int kPD = 128;  // head dimension handled (one float4 per lane)
constexpr int kPWarps = 8;

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}
__device__ __forceinline__ float dot4(float4 a, float4 b) { return a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w; }
__device__ __forceinline__ float4 scale4(float4 a, float s) { return make_float4(a.x * s, a.y * s, a.z * s, a.w * s); }
__device__ __forceinline__ float sigm(float x) { return 1.f / (1.f + expf(-x)); }
// softplus(x) = log(1 + e^x), evaluated without overflow: max(x, 0) + log1p(e^-|x|)
__device__ __forceinline__ float softplus_f(float x) { return fmaxf(x, 0.f) + log1pf(expf(-fabsf(x))); }
__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }

struct ProShape {
  long long rows;  // B * L * H
  int L, H;
  float g_max;
  int l2norm;
};

// Row r = (b * L + l) * H + h.  A token's y row holds the six projections, H * D values each.
__device__ __forceinline__ void row_index(const ProShape& s, long long r, long long& y_off, long long& o_off) {
  const long long h = r % s.H;
  const long long bl = r / s.H;
  const long long l = bl % s.L;
  const long long b = bl / s.L;
  y_off = bl * 6LL * s.H * kPD + h * kPD;                  // + t * H * D for projection t
  o_off = ((b * s.H + h) * (long long)s.L + l) * kPD;      // (B, H, L, D)
}

__global__ void __launch_bounds__(kPWarps * 32) prologue_fwd_kernel(const float* __restrict__ y, ProShape s,
                                                                   float* __restrict__ q, float* __restrict__ k,
                                                                   float* __restrict__ v, float* __restrict__ w,
                                                                   float* __restrict__ b, float* __restrict__ g) {
  const long long r = (long long)blockIdx.x * kPWarps + (threadIdx.x >> 5);
  if (r >= s.rows) return;
  const int lane = threadIdx.x & 31;
  long long yo, oo;
  row_index(s, r, yo, oo);
  const long long ts = (long long)s.H * kPD;
  const float* yr = y + yo + lane * 4;
  float4 yq = ldg4(yr), yk = ldg4(yr + ts), yv = ldg4(yr + 2 * ts), yw = ldg4(yr + 3 * ts);
  float4 yb = ldg4(yr + 4 * ts), yg = ldg4(yr + 5 * ts);
  if (s.l2norm) {
    const float nq = warp_sum(dot4(yq, yq)), nk = warp_sum(dot4(yk, yk));
    yq = scale4(yq, rsqrtf(nq + 1e-6f));
    yk = scale4(yk, rsqrtf(nk + 1e-6f));
  }
  const float gm = s.g_max;
  float4 bb = make_float4(sigm(yb.x), sigm(yb.y), sigm(yb.z), sigm(yb.w));
  float4 gg = make_float4(-fminf(softplus_f(yg.x), gm), -fminf(softplus_f(yg.y), gm), -fminf(softplus_f(yg.z), gm),
                          -fminf(softplus_f(yg.w), gm));
  const long long o = oo + lane * 4;
  st4(q + o, yq);
  st4(k + o, yk);
  st4(v + o, yv);
  st4(w + o, yw);
  st4(b + o, bb);
  st4(g + o, gg);
}

__global__ void __launch_bounds__(kPWarps * 32) prologue_bwd_kernel(
    const float* __restrict__ y, ProShape s, const float* __restrict__ dq, const float* __restrict__ dk,
    const float* __restrict__ dv, const float* __restrict__ dw, const float* __restrict__ db,
    const float* __restrict__ dg, float* __restrict__ dy) {
  const long long r = (long long)blockIdx.x * kPWarps + (threadIdx.x >> 5);
  if (r >= s.rows) return;
  const int lane = threadIdx.x & 31;
  long long yo, oo;
  row_index(s, r, yo, oo);
  const long long ts = (long long)s.H * kPD;
  const float* yr = y + yo + lane * 4;
  float* dyr = dy + yo + lane * 4;
  const long long o = oo + lane * 4;
  float4 gq = ldg4(dq + o), gk = ldg4(dk + o);
  st4(dyr + 2 * ts, ldg4(dv + o));
  st4(dyr + 3 * ts, ldg4(dw + o));
  float4 yq = ldg4(yr), yk = ldg4(yr + ts);
  if (s.l2norm) {
    // d(y / n)/dy applied to dx:  (dx - x (x . dx)) / n  with x = y / n
    const float iq = rsqrtf(warp_sum(dot4(yq, yq)) + 1e-6f), ik = rsqrtf(warp_sum(dot4(yk, yk)) + 1e-6f);
    const float4 xq = scale4(yq, iq), xk = scale4(yk, ik);
    const float pq = warp_sum(dot4(xq, gq)), pk = warp_sum(dot4(xk, gk));
    gq = make_float4((gq.x - xq.x * pq) * iq, (gq.y - xq.y * pq) * iq, (gq.z - xq.z * pq) * iq,
                     (gq.w - xq.w * pq) * iq);
    gk = make_float4((gk.x - xk.x * pk) * ik, (gk.y - xk.y * pk) * ik, (gk.z - xk.z * pk) * ik,
                     (gk.w - xk.w * pk) * ik);
  }
  st4(dyr, gq);
  st4(dyr + ts, gk);
  const float4 yb = ldg4(yr + 4 * ts), yg = ldg4(yr + 5 * ts);
  const float4 gb = ldg4(db + o), gg = ldg4(dg + o);
  auto dbf = [](float yv, float gv) {
    const float sv = sigm(yv);
    return gv * sv * (1.f - sv);
  };
  const float gm = s.g_max;
  auto dgf = [gm](float yv, float gv) { return softplus_f(yv) <= gm ? -gv * sigm(yv) : 0.f; };
  st4(dyr + 4 * ts, make_float4(dbf(yb.x, gb.x), dbf(yb.y, gb.y), dbf(yb.z, gb.z), dbf(yb.w, gb.w)));
  st4(dyr + 5 * ts, make_float4(dgf(yg.x, gg.x), dgf(yg.y, gg.y), dgf(yg.z, gg.z), dgf(yg.w, gg.w)));
}

bool pro_args_ok(int64_t B, int64_t L, int64_t H, int64_t D, float g_max) {
  return B > 0 && L > 0 && H > 0 && D == kPD && g_max > 0.f && B * L * H < (1LL << 33);  // grid < 2^30 blocks
}
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace gdn2

extern "C" gdn2_status gdn2_prologue_fwd(const float* y, int64_t B, int64_t L, int64_t H, int64_t D, float g_max,
                                         int32_t l2norm, float* q, float* k, float* v, float* w, float* b, float* g,
                                         void* stream) {
  using namespace gdn2;
  if (!pro_args_ok(B, L, H, D, g_max)) return D != kPD && D > 0 ? GDN2_ERR_UNSUPPORTED : GDN2_ERR_INVALID_ARGUMENT;
  const void* ptrs[] = {y, q, k, v, w, b, g};
  for (const void* p : ptrs)
    if (!p || !aligned16(p)) return GDN2_ERR_INVALID_ARGUMENT;
  ProShape s{B * L * H, (int)L, (int)H, g_max, l2norm};
  const long long blocks = (s.rows + kPWarps - 1) / kPWarps;
  prologue_fwd_kernel<<<(unsigned)blocks, kPWarps * 32, 0, (cudaStream_t)stream>>>(y, s, q, k, v, w, b, g);
  return cudaGetLastError() == cudaSuccess ? GDN2_OK : GDN2_ERR_CUDA;
}

extern "C" gdn2_status gdn2_prologue_bwd(const float* y, int64_t B, int64_t L, int64_t H, int64_t D, float g_max,
                                         int32_t l2norm, const float* dq, const float* dk, const float* dv,
                                         const float* dw, const float* db, const float* dg, float* dy,
                                         void* stream) {
  using namespace gdn2;
  if (!pro_args_ok(B, L, H, D, g_max)) return D != kPD && D > 0 ? GDN2_ERR_UNSUPPORTED : GDN2_ERR_INVALID_ARGUMENT;
  const void* ptrs[] = {y, dq, dk, dv, dw, db, dg, dy};
  for (const void* p : ptrs)
    if (!p || !aligned16(p)) return GDN2_ERR_INVALID_ARGUMENT;
  ProShape s{B * L * H, (int)L, (int)H, g_max, l2norm};
  const long long blocks = (s.rows + kPWarps - 1) / kPWarps;
  prologue_bwd_kernel<<<(unsigned)blocks, kPWarps * 32, 0, (cudaStream_t)stream>>>(y, s, dq, dk, dv, dw, db, dg,
                                                                                   dy);
  return cudaGetLastError() == cudaSuccess ? GDN2_OK : GDN2_ERR_CUDA;
}
