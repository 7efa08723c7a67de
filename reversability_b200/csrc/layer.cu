// One reversible Block step per call (rk_layer_*): the host-side sequence of
// librevk calls that the Python engine issues for a layer on a single stream,
// so a caller that binds only librevk.so can run the reversible forward and the
// reconstruction backward of reversible.py:21-69 / optimized.py:21-41.
//
// Every step below is one of the public entry points, called with the
// arguments and in the order of engine.py's single-stream path; the results
// are therefore bit-identical to it (and, through the engine's own tests, to
// the multi-stream pipelined sweep). Temporaries are carved out of the
// caller's workspace (256-byte aligned regions); nothing is allocated and the
// host never waits.
#include <cstdint>
#include "common.cuh"
#include "revk.h"

namespace {

// Bump allocator over the caller's workspace; with base == nullptr it only
// measures (rk_layer_workspace uses the same plan as the launches).
struct Arena {
  uint8_t* base;
  int64_t off = 0;
  template <typename T>
  T* take(int64_t n) {
    off = (off + 255) & ~int64_t(255);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += n * (int64_t)sizeof(T);
    return p;
  }
};

struct Shape {
  int64_t B, T, M, d, H, hd, ff, mt;
  int dt;
};

bool shape_of(const rk_layer_desc* L, Shape& s) {
  if (!L || L->batch < 0 || L->length < 0 || L->d_model <= 0 || L->n_heads <= 0 || L->d_ff <= 0 ||
      L->d_model % L->n_heads || L->mlp_tokens < 0)
    return false;
  s.B = L->batch;
  s.T = L->length;
  s.M = L->batch * L->length;
  s.d = L->d_model;
  s.H = L->n_heads;
  s.hd = L->d_model / L->n_heads;
  s.ff = L->d_ff;
  s.mt = (L->mlp_tokens > 0 && L->mlp_tokens < s.M) ? L->mlp_tokens : s.M;
  s.dt = L->dtype;
  return true;
}

// The fused epilogues the sequence relies on: SwiGLU in the up projection
// (ff a multiple of 128), SwiGLU backward in the down dgrad (ff % 64), the
// state update in the output projections (d % 32), 16-byte rows.
int shape_status(const rk_layer_desc* L, const Shape& s) {
  if (L->dtype != RK_BF16 && L->dtype != RK_F16) return RK_ERR_DTYPE;
  if (s.ff % 128 || s.d % 32 || (s.hd != 32 && s.hd != 64)) return RK_ERR_UNSUPPORTED;
  return RK_OK;
}

bool weights_ok(const rk_layer_desc* L) {
  return L->attn_norm && L->qkv && L->proj && L->mlp_norm && L->up && L->down;
}

bool grads_ok(const rk_layer_grads* G) {
  return G && G->attn_norm && G->qkv && G->proj && G->mlp_norm && G->up && G->down;
}

// Scratch of the attention sublayer forward (what its VJP keeps).
struct AttnBufs {
  void *n1, *qkv, *o;
  float *rstd1, *lse;
};

AttnBufs plan_attn(Arena& ar, const Shape& s, bool rstd) {
  AttnBufs b;
  b.n1 = ar.take<uint16_t>(s.M * s.d);
  b.rstd1 = rstd ? ar.take<float>(s.M) : nullptr;
  b.qkv = ar.take<uint16_t>(s.M * 3 * s.d);
  b.o = ar.take<uint16_t>(s.M * s.d);
  b.lse = ar.take<float>(s.B * s.H * s.T);
  return b;
}

// Scratch of the attention VJP.
struct AttnGradBufs {
  void *do_, *dqkv, *dn1;
  float* dsum;
};

AttnGradBufs plan_attn_grad(Arena& ar, const Shape& s) {
  AttnGradBufs b;
  b.do_ = ar.take<uint16_t>(s.M * s.d);
  b.dsum = ar.take<float>(s.B * s.H * s.T);
  b.dqkv = ar.take<uint16_t>(s.M * 3 * s.d);
  b.dn1 = ar.take<uint16_t>(s.M * s.d);
  return b;
}

// Workspaces of the weight-gradient GEMMs and the RMSNorm backward: the
// largest any call of the layer needs.
struct Scratch {
  float* wgrad;
  int64_t wgrad_bytes;
  float* norm;
  int64_t norm_bytes;
};

Scratch plan_scratch(Arena& ar, const Shape& s) {
  Scratch sc;
  int64_t w = rk_gemm_wgrad_workspace(s.M, s.d, s.d);
  const int64_t cands[3] = {rk_gemm_wgrad_workspace(s.M, 3 * s.d, s.d), rk_gemm_wgrad_workspace(s.mt, s.d, s.ff),
                            rk_gemm_wgrad_workspace(s.mt, 2 * s.ff, s.d)};
  for (int64_t c : cands) w = c > w ? c : w;
  int64_t n = rk_rmsnorm_bwd_workspace(s.M, s.d);
  const int64_t nt = rk_rmsnorm_bwd_workspace(s.mt, s.d);
  n = nt > n ? nt : n;
  sc.wgrad_bytes = w > 4 ? w : 4;
  sc.norm_bytes = n > 4 ? n : 4;
  sc.wgrad = ar.take<float>(sc.wgrad_bytes / 4 + 1);
  sc.norm = ar.take<float>(sc.norm_bytes / 4 + 1);
  return sc;
}

#define RK_TRY(call)              \
  do {                            \
    const int st_ = (call);       \
    if (st_ != RK_OK) return st_; \
  } while (0)

template <typename T>
T* at(T* p, int64_t elems, int64_t esz) {
  return reinterpret_cast<T*>(reinterpret_cast<uint8_t*>(const_cast<void*>(static_cast<const void*>(p))) +
                              elems * esz);
}

// rmsnorm(x) -> QKV -> causal attention (engine attn_forward up to o).
int attn_core(const rk_layer_desc* L, const Shape& s, const float* x, const AttnBufs& b, void* st) {
  RK_TRY(rk_rmsnorm_fwd(x, RK_F32, s.d, L->attn_norm, b.n1, s.dt, s.d, b.rstd1, s.M, s.d, L->eps_attn, st));
  RK_TRY(rk_gemm_fprop(b.n1, s.d, L->qkv, s.d, b.qkv, 3 * s.d, s.M, 3 * s.d, s.d, s.dt, s.dt, st));
  return rk_attn_fwd(b.qkv, 3 * s.d, b.o, s.d, b.lse, s.B, s.H, s.hd, s.T, s.dt, st);
}

// The attention VJP (engine attn_vjp, no side streams): da -> dx_out =
// residual + A^T da; lp_out (if not null) = round(round(dx_out) * lp_scale).
int attn_vjp(const rk_layer_desc* L, const rk_layer_grads* G, const Shape& s, const float* x, const AttnBufs& b,
             const AttnGradBufs& gb, const Scratch& sc, const void* da, const float* residual, float* dx_out,
             void* lp_out, float lp_scale, void* st) {
  RK_TRY(rk_gemm_dgrad(da, s.d, L->proj, s.d, gb.do_, s.d, s.M, s.d, s.d, s.dt, s.dt, st));
  RK_TRY(rk_gemm_wgrad(da, s.d, b.o, s.d, G->proj, s.d, s.M, s.d, s.d, s.dt, 1, sc.wgrad, sc.wgrad_bytes, st));
  RK_TRY(rk_attn_bwd(b.qkv, 3 * s.d, b.o, gb.do_, s.d, b.lse, gb.dsum, gb.dqkv, 3 * s.d, s.B, s.H, s.hd, s.T, s.dt,
                     st));
  RK_TRY(rk_gemm_wgrad(gb.dqkv, 3 * s.d, b.n1, s.d, G->qkv, s.d, s.M, 3 * s.d, s.d, s.dt, 1, sc.wgrad,
                       sc.wgrad_bytes, st));
  RK_TRY(rk_gemm_dgrad(gb.dqkv, 3 * s.d, L->qkv, s.d, gb.dn1, s.d, s.M, 3 * s.d, s.d, s.dt, s.dt, st));
  return rk_rmsnorm_bwd_fused(x, L->attn_norm, b.rstd1, gb.dn1, s.dt, residual, nullptr, lp_out, s.dt,
                              lp_out ? lp_scale : 1.f, dx_out, G->attn_norm, 1, sc.norm, sc.norm_bytes, s.M, s.d, st);
}

// MLP forward and VJP tile by tile (engine mlp_forward_vjp): for each tile the
// up projection with SwiGLU (u kept), the down projection with the state update
// out = state - round(coeff * round(m + addend)), the down dgrad with the
// SwiGLU backward, both weight gradients, the up dgrad and the RMSNorm backward
// (dx_out = residual + M^T gm; lp_out = round(lp_add + round(dx)) or
// round(round(dx_out)) without lp_add).
struct MlpBufs {
  void *hg, *u, *du, *dn2;
};

MlpBufs plan_mlp(Arena& ar, const Shape& s, bool vjp) {
  MlpBufs b;
  b.hg = ar.take<uint16_t>(s.mt * s.ff);
  b.u = vjp ? ar.take<uint16_t>(s.mt * 2 * s.ff) : nullptr;
  b.du = vjp ? ar.take<uint16_t>(s.mt * 2 * s.ff) : nullptr;
  b.dn2 = vjp ? ar.take<uint16_t>(s.mt * s.d) : nullptr;
  return b;
}

int mlp_forward_vjp(const rk_layer_desc* L, const rk_layer_grads* G, const Shape& s, const MlpBufs& b,
                    const Scratch& sc, const void* n2, const float* ysum, const float* rstd2, const float* state,
                    const void* addend, float coeff, float* out, const void* gm, const float* residual,
                    const void* lp_add, void* lp_out, float* dx_out, void* st) {
  const int64_t e2 = 2;
  for (int64_t r0 = 0; r0 < s.M; r0 += s.mt) {
    const int64_t rows = (s.M - r0) < s.mt ? (s.M - r0) : s.mt;
    const void* n2t = at(n2, r0 * s.d, e2);
    const void* gmt = at(gm, r0 * s.d, e2);
    RK_TRY(rk_gemm_fprop_swiglu(n2t, s.d, L->up, s.d, b.hg, s.ff, b.u, 2 * s.ff, rows, s.ff, s.d, s.dt, st));
    RK_TRY(rk_gemm_fprop_reconstruct(b.hg, s.ff, L->down, s.ff, state + r0 * s.d, s.d,
                                     addend ? at(addend, r0 * s.d, e2) : nullptr, s.d, coeff, out + r0 * s.d, s.d,
                                     rows, s.d, s.ff, s.dt, st));
    RK_TRY(rk_gemm_dgrad_swiglu(gmt, s.d, L->down, s.ff, b.u, 2 * s.ff, b.du, 2 * s.ff, rows, s.ff, s.d, s.dt, st));
    RK_TRY(rk_gemm_wgrad(gmt, s.d, b.hg, s.ff, G->down, s.ff, rows, s.d, s.ff, s.dt, 1, sc.wgrad, sc.wgrad_bytes,
                         st));
    RK_TRY(rk_gemm_wgrad(b.du, 2 * s.ff, n2t, s.d, G->up, s.d, rows, 2 * s.ff, s.d, s.dt, 1, sc.wgrad,
                         sc.wgrad_bytes, st));
    RK_TRY(rk_gemm_dgrad(b.du, 2 * s.ff, L->up, s.d, b.dn2, s.d, rows, 2 * s.ff, s.d, s.dt, s.dt, st));
    RK_TRY(rk_rmsnorm_bwd_fused(ysum + r0 * s.d, L->mlp_norm, rstd2 + r0, b.dn2, s.dt,
                                residual ? residual + r0 * s.d : nullptr, lp_add ? at(lp_add, r0 * s.d, e2) : nullptr,
                                at(lp_out, r0 * s.d, e2), s.dt, 1.f, dx_out + r0 * s.d, G->mlp_norm, 1, sc.norm,
                                sc.norm_bytes, rows, s.d, st));
  }
  return RK_OK;
}

// MLP forward only: up projection with SwiGLU, down projection with the
// state update (engine mlp_forward with recon).
int mlp_forward(const rk_layer_desc* L, const Shape& s, const MlpBufs& b, const void* n2, const float* state,
                const void* addend, float coeff, float* out, void* st) {
  const int64_t e2 = 2;
  for (int64_t r0 = 0; r0 < s.M; r0 += s.mt) {
    const int64_t rows = (s.M - r0) < s.mt ? (s.M - r0) : s.mt;
    RK_TRY(rk_gemm_fprop_swiglu(at(n2, r0 * s.d, e2), s.d, L->up, s.d, b.hg, s.ff, nullptr, 2 * s.ff, rows, s.ff,
                                s.d, s.dt, st));
    RK_TRY(rk_gemm_fprop_reconstruct(b.hg, s.ff, L->down, s.ff, state + r0 * s.d, s.d,
                                     addend ? at(addend, r0 * s.d, e2) : nullptr, s.d, coeff, out + r0 * s.d, s.d,
                                     rows, s.d, s.ff, s.dt, st));
  }
  return RK_OK;
}

// ---- per-entry plans (shared by the workspace query and the launches)
struct FwdPlan {
  AttnBufs at;
  void *a, *n2;
  MlpBufs mlp;
};

FwdPlan plan_fwd(Arena& ar, const Shape& s, int method) {
  FwdPlan p;
  p.at = plan_attn(ar, s, false);
  p.a = method == RK_METHOD_MIDPOINT ? ar.take<uint16_t>(s.M * s.d) : nullptr;
  p.n2 = ar.take<uint16_t>(s.M * s.d);
  p.mlp = plan_mlp(ar, s, false);
  return p;
}

struct BwdPlan {
  AttnBufs at;
  AttnGradBufs ag;
  Scratch sc;
  MlpBufs mlp;
  void *a, *g, *n2, *lp;
  float *ysum, *rstd2, *dxacc;
};

BwdPlan plan_bwd(Arena& ar, const Shape& s, int method) {
  BwdPlan p;
  p.at = plan_attn(ar, s, true);
  p.a = method == RK_METHOD_MIDPOINT ? ar.take<uint16_t>(s.M * s.d) : nullptr;
  p.g = ar.take<uint16_t>(s.M * s.d);  // gF / gm when the caller gave none
  p.n2 = ar.take<uint16_t>(s.M * s.d);
  p.ysum = method == RK_METHOD_MIDPOINT ? ar.take<float>(s.M * s.d) : nullptr;
  p.rstd2 = ar.take<float>(s.M);
  p.dxacc = method == RK_METHOD_MIDPOINT ? ar.take<float>(s.M * s.d) : nullptr;
  p.lp = ar.take<uint16_t>(s.M * s.d);  // da (midpoint) / ga (Euler)
  p.mlp = plan_mlp(ar, s, true);
  p.ag = plan_attn_grad(ar, s);
  p.sc = plan_scratch(ar, s);
  return p;
}

int begin(const rk_layer_desc* L, Shape& s, void* ws, int64_t ws_bytes, int64_t need) {
  if (!shape_of(L, s) || !weights_ok(L)) return RK_ERR_ARG;
  const int st = shape_status(L, s);
  if (st) return st;
  if (s.M == 0) return RK_OK;
  if (!ws || ws_bytes < need || (reinterpret_cast<uintptr_t>(ws) & 255)) return RK_ERR_WORKSPACE;
  return RK_OK;
}

}  // namespace

extern "C" int64_t rk_layer_workspace(const rk_layer_desc* desc, int method, int backward) {
  Shape s;
  if (!shape_of(desc, s) || (method != RK_METHOD_MIDPOINT && method != RK_METHOD_EULER)) return -1;
  Arena ar{nullptr};
  if (backward) plan_bwd(ar, s, method);
  else plan_fwd(ar, s, method);
  return (ar.off + 255) & ~int64_t(255);
}

extern "C" int rk_layer_fwd_midpoint(const rk_layer_desc* desc, const float* p, const float* q, float h,
                                     float* q_next, void* workspace, int64_t workspace_bytes, void* stream) {
  Shape s;
  if (!p || !q || !q_next) return RK_ERR_ARG;
  const int64_t need = rk_layer_workspace(desc, RK_METHOD_MIDPOINT, 0);
  if (const int st = begin(desc, s, workspace, workspace_bytes, need)) return st;
  if (s.M == 0) return RK_OK;
  Arena ar{static_cast<uint8_t*>(workspace)};
  const FwdPlan P = plan_fwd(ar, s, RK_METHOD_MIDPOINT);
  const rk_layer_desc* L = desc;
  RK_TRY(attn_core(L, s, q, P.at, stream));
  RK_TRY(rk_gemm_fprop(P.at.o, s.d, L->proj, s.d, P.a, s.d, s.M, s.d, s.d, s.dt, s.dt, stream));
  RK_TRY(rk_add_rmsnorm_fwd(q, P.a, s.dt, L->mlp_norm, P.n2, s.dt, nullptr, nullptr, s.M, s.d, L->eps_mlp, stream));
  return mlp_forward(L, s, P.mlp, P.n2, p, P.a, -2.f * h, q_next, stream);
}

extern "C" int rk_layer_fwd_euler(const rk_layer_desc* desc, const float* p, const float* q, float* p_next,
                                  float* q_next, void* workspace, int64_t workspace_bytes, void* stream) {
  Shape s;
  if (!p || !q || !p_next || !q_next) return RK_ERR_ARG;
  const int64_t need = rk_layer_workspace(desc, RK_METHOD_EULER, 0);
  if (const int st = begin(desc, s, workspace, workspace_bytes, need)) return st;
  if (s.M == 0) return RK_OK;
  Arena ar{static_cast<uint8_t*>(workspace)};
  const FwdPlan P = plan_fwd(ar, s, RK_METHOD_EULER);
  const rk_layer_desc* L = desc;
  RK_TRY(attn_core(L, s, p, P.at, stream));
  RK_TRY(rk_gemm_fprop_reconstruct(P.at.o, s.d, L->proj, s.d, q, s.d, nullptr, s.d, -1.f, q_next, s.d, s.M, s.d, s.d,
                                   s.dt, stream));
  RK_TRY(rk_rmsnorm_fwd(q_next, RK_F32, s.d, L->mlp_norm, P.n2, s.dt, s.d, nullptr, s.M, s.d, L->eps_mlp, stream));
  return mlp_forward(L, s, P.mlp, P.n2, p, nullptr, -1.f, p_next, stream);
}

extern "C" int rk_layer_bwd_midpoint(const rk_layer_desc* desc, const rk_layer_grads* grads, const float* p,
                                     const float* q, const float* dp, const float* dq, const void* gf_in, float h,
                                     float* p_prev, float* dq_prev, void* gf_out, void* workspace,
                                     int64_t workspace_bytes, void* stream) {
  Shape s;
  if (!p || !q || !dq || !p_prev || !dq_prev || !grads_ok(grads)) return RK_ERR_ARG;
  const int64_t need = rk_layer_workspace(desc, RK_METHOD_MIDPOINT, 1);
  if (const int st = begin(desc, s, workspace, workspace_bytes, need)) return st;
  if (s.M == 0) return RK_OK;
  Arena ar{static_cast<uint8_t*>(workspace)};
  const BwdPlan P = plan_bwd(ar, s, RK_METHOD_MIDPOINT);
  const rk_layer_desc* L = desc;
  const float* x = p;  // the force is evaluated at p_n (= q_{n-1})
  RK_TRY(attn_core(L, s, x, P.at, stream));
  RK_TRY(rk_gemm_fprop(P.at.o, s.d, L->proj, s.d, P.a, s.d, s.M, s.d, s.d, s.dt, s.dt, stream));
  const void* gf = gf_in;
  if (!gf) {  // gF = round(2h * round(dq))
    RK_TRY(rk_cast_scale(dq, P.g, s.dt, 2.f * h, s.M * s.d, stream));
    gf = P.g;
  }
  // MLP at y = x + a, its VJP for gF; p_{n-1} = q - round(2h round(a + m)) from
  // the down projection; dxacc = dp + M^T gF; da = round(gF + round(M^T gF))
  RK_TRY(rk_add_rmsnorm_fwd(x, P.a, s.dt, L->mlp_norm, P.n2, s.dt, P.ysum, P.rstd2, s.M, s.d, L->eps_mlp, stream));
  RK_TRY(mlp_forward_vjp(L, grads, s, P.mlp, P.sc, P.n2, P.ysum, P.rstd2, q, P.a, 2.f * h, p_prev, gf, dp, gf, P.lp,
                         P.dxacc, stream));
  // dq_{n-1} = dxacc + A^T da, and gF of the layer below in the same epilogue
  return attn_vjp(L, grads, s, x, P.at, P.ag, P.sc, P.lp, P.dxacc, dq_prev, gf_out, 2.f * h, stream);
}

extern "C" int rk_layer_bwd_euler(const rk_layer_desc* desc, const rk_layer_grads* grads, const float* p,
                                  const float* q, const float* dp, const float* dq, const void* gm_in, float* p_prev,
                                  float* q_prev, float* dp_prev, float* dq_prev, void* gm_out, void* workspace,
                                  int64_t workspace_bytes, void* stream) {
  Shape s;
  if (!p || !q || !dp || !p_prev || !q_prev || !dp_prev || !dq_prev || !grads_ok(grads)) return RK_ERR_ARG;
  const int64_t need = rk_layer_workspace(desc, RK_METHOD_EULER, 1);
  if (const int st = begin(desc, s, workspace, workspace_bytes, need)) return st;
  if (s.M == 0) return RK_OK;
  Arena ar{static_cast<uint8_t*>(workspace)};
  const BwdPlan P = plan_bwd(ar, s, RK_METHOD_EULER);
  const rk_layer_desc* L = desc;
  const void* gm = gm_in;
  if (!gm) {  // gm = round(dp)
    RK_TRY(rk_cast_scale(dp, P.g, s.dt, 1.f, s.M * s.d, stream));
    gm = P.g;
  }
  // M at q (its norm input is q itself); p_{n-1} = p - m from the down
  // projection; dq_{n-1} = dq + M^T gm; ga = round(dq_{n-1})
  RK_TRY(rk_rmsnorm_fwd(q, RK_F32, s.d, L->mlp_norm, P.n2, s.dt, s.d, P.rstd2, s.M, s.d, L->eps_mlp, stream));
  RK_TRY(mlp_forward_vjp(L, grads, s, P.mlp, P.sc, P.n2, q, P.rstd2, p, nullptr, 1.f, p_prev, gm, dq, nullptr, P.lp,
                         dq_prev, stream));
  // A at p_{n-1}; q_{n-1} = q - a from the output projection; its VJP for ga
  RK_TRY(attn_core(L, s, p_prev, P.at, stream));
  RK_TRY(rk_gemm_fprop_reconstruct(P.at.o, s.d, L->proj, s.d, q, s.d, nullptr, s.d, 1.f, q_prev, s.d, s.M, s.d, s.d,
                                   s.dt, stream));
  return attn_vjp(L, grads, s, p_prev, P.at, P.ag, P.sc, P.lp, dp, dp_prev, gm_out, 1.f, stream);
}
