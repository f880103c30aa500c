// torch_ops.cpp -- the estimators as PyTorch operators (namespace rl_triton).
//
// Each operator takes tensors, prepares them (one element type for the [N, T]
// streams: bf16 only when every stream is bf16, else fp32; contiguous; 16-byte
// aligned), allocates the fp32 outputs, takes the per-(device, stream)
// look-back workspace from the cache below and calls the C ABI of
// librlscan.so (include/rlscan.h) on the current CUDA stream.  Registering them
// with the dispatcher (CUDA kernels here, fake kernels in rl_triton/_native.py)
// lets torch.compile keep a call inside one graph and lets CUDA-graph capture
// record it, and moves the per-call host work out of Python.
//
// The Python functions of rl_triton keep the reference's argument checks and
// messages and its bootstrap-kind dispatch; these operators are what they
// call.  The reference has no counterpart: it launches Triton kernels from
// Python (src/rl_triton/ops/*.py).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <cstdint>
#include <map>
#include <mutex>
#include <optional>
#include <string>
#include <utility>
#include <vector>

#include "rlscan.h"

namespace {

using at::Tensor;
using OptT = std::optional<Tensor>;

// ---- per-(device, stream) workspace ------------------------------------------
// Zero-filled when allocated; the kernels keep it consistent from call to call
// (epoch-tagged records).  Grown by doubling; the old buffer is released to the
// caching allocator on the same stream, so work still queued on it is safe.
std::mutex g_ws_mu;
std::map<std::pair<int, cudaStream_t>, Tensor> g_ws;

Tensor workspace_for(const at::Device& dev, cudaStream_t s, int64_t num_elements) {
  const int64_t need = (int64_t)rls_workspace_bytes(num_elements < 1 ? 1 : num_elements);
  std::lock_guard<std::mutex> lock(g_ws_mu);
  auto key = std::make_pair((int)dev.index(), s);
  auto it = g_ws.find(key);
  if (it != g_ws.end() && it->second.numel() >= need) return it->second;
  int64_t size = need < (1 << 16) ? (1 << 16) : need;
  if (it != g_ws.end() && 2 * it->second.numel() > size) size = 2 * it->second.numel();
  Tensor buf = at::zeros({size}, at::TensorOptions().dtype(at::kByte).device(dev));
  g_ws[key] = buf;
  return buf;
}

cudaStream_t stream_of(const Tensor& t) { return c10::cuda::getCurrentCUDAStream(t.device().index()).stream(); }

void check(int st, const char* what) {
  TORCH_CHECK(st == RLS_OK, what, ": librlscan status ", st, " (", rls_status_string(st), ")");
}

// Contiguous and 16-byte aligned (the kernels use 16-byte vector accesses).
Tensor ready(const Tensor& t) {
  Tensor c = t.is_contiguous() ? t : t.contiguous();
  if (reinterpret_cast<uintptr_t>(c.data_ptr()) % 16 != 0) c = c.clone();
  return c;
}
OptT ready(const OptT& t) { return t ? OptT(ready(*t)) : OptT(); }

// One element type for the floating [N, T] streams of a call.
int unify(std::vector<OptT*> streams) {
  bool all_bf16 = true, any = false;
  for (OptT* s : streams)
    if (*s) {
      any = true;
      all_bf16 = all_bf16 && (*s)->scalar_type() == at::kBFloat16;
    }
  if (any && all_bf16) return RLS_BF16;
  for (OptT* s : streams)
    if (*s && (*s)->scalar_type() != at::kFloat) *s = (*s)->to(at::kFloat);
  return RLS_F32;
}

Tensor f32(const Tensor& t) { return ready(t.scalar_type() == at::kFloat ? t : t.to(at::kFloat)); }
OptT f32(const OptT& t) { return t ? OptT(f32(*t)) : OptT(); }

const void* P(const OptT& t) { return t ? t->data_ptr() : nullptr; }
const void* P(const Tensor& t) { return t.data_ptr(); }

// Optional time-split descriptor: t0 < 0 means whole rows.
struct Seg {
  rls_segment_t s;
  OptT halo;
  const rls_segment_t* ptr() const { return s.t0 < 0 ? nullptr : &s; }
};
Seg make_seg(int64_t t0, int64_t total, const OptT& halo) {
  Seg g;
  g.halo = f32(halo);
  g.s.t0 = t0;
  g.s.total_len = total;
  g.s.halo = g.halo ? static_cast<const float*>(g.halo->data_ptr()) : nullptr;
  return g;
}

Tensor empty_f32(const Tensor& like) { return at::empty(like.sizes(), like.options().dtype(at::kFloat)); }

// ---- operators ---------------------------------------------------------------
Tensor op_gae(const Tensor& rewards, const Tensor& values, const Tensor& terminateds, const OptT& truncateds,
              const OptT& bootstrap, int64_t boot_kind, double gamma, double lambda_, int64_t t0, int64_t total,
              const OptT& halo) {
  OptT r = rewards, v = values, term = terminateds, tr = truncateds;
  OptT full = boot_kind == RLS_BOOT_ROW ? OptT() : bootstrap;
  const int dt = unify({&r, &v, &term, &tr, &full});
  r = ready(r); v = ready(v); term = ready(term); tr = ready(tr); full = ready(full);
  OptT row = boot_kind == RLS_BOOT_ROW ? f32(bootstrap) : OptT();
  const Seg seg = make_seg(t0, total, halo);
  const int64_t n = rewards.size(0), t = rewards.size(1);
  Tensor out = empty_f32(*r);
  cudaStream_t s = stream_of(*r);
  Tensor ws = workspace_for(r->device(), s, n * t);
  check(rls_gae(P(r), P(v), P(term), P(tr), boot_kind == RLS_BOOT_ROW ? P(row) : P(full), (int)boot_kind,
                out.data_ptr<float>(), n, t, (float)gamma, (float)lambda_, dt, seg.ptr(), ws.data_ptr(),
                (size_t)ws.numel(), s),
        "rls_gae");
  return out;
}

// (normalized advantages, returns = A + V)
std::tuple<Tensor, Tensor> op_gae_normalized(const Tensor& rewards, const Tensor& values, const Tensor& terminateds,
                                             const OptT& truncateds, const OptT& bootstrap, int64_t boot_kind,
                                             double gamma, double lambda_, double eps) {
  OptT r = rewards, v = values, term = terminateds, tr = truncateds;
  OptT full = boot_kind == RLS_BOOT_ROW ? OptT() : bootstrap;
  const int dt = unify({&r, &v, &term, &tr, &full});
  r = ready(r); v = ready(v); term = ready(term); tr = ready(tr); full = ready(full);
  OptT row = boot_kind == RLS_BOOT_ROW ? f32(bootstrap) : OptT();
  const int64_t n = rewards.size(0), t = rewards.size(1);
  Tensor norm = empty_f32(*r), rets = empty_f32(*r);
  cudaStream_t s = stream_of(*r);
  Tensor ws = workspace_for(r->device(), s, n * t < (1 << 20) ? (1 << 20) : n * t);
  check(rls_gae_normalized(P(r), P(v), P(term), P(tr), boot_kind == RLS_BOOT_ROW ? P(row) : P(full), (int)boot_kind,
                           norm.data_ptr<float>(), rets.data_ptr<float>(), nullptr, nullptr, n, t, (float)gamma,
                           (float)lambda_, (float)eps, dt, ws.data_ptr(), (size_t)ws.numel(), s),
        "rls_gae_normalized");
  return {norm, rets};
}

// (advantages, returns, loss scalar, d loss / d new_values)
std::tuple<Tensor, Tensor, Tensor, Tensor> op_gae_value_loss(const Tensor& rewards, const Tensor& values,
                                                             const Tensor& terminateds, const OptT& truncateds,
                                                             const OptT& bootstrap, int64_t boot_kind,
                                                             const Tensor& new_values, double gamma, double lambda_,
                                                             int64_t loss_kind, double delta) {
  OptT r = rewards, v = values, term = terminateds, tr = truncateds;
  OptT full = boot_kind == RLS_BOOT_ROW ? OptT() : bootstrap;
  const int dt = unify({&r, &v, &term, &tr, &full});
  r = ready(r); v = ready(v); term = ready(term); tr = ready(tr); full = ready(full);
  OptT row = boot_kind == RLS_BOOT_ROW ? f32(bootstrap) : OptT();
  const Tensor nv = f32(new_values);
  const int64_t n = rewards.size(0), t = rewards.size(1);
  Tensor adv = empty_f32(*r), rets = empty_f32(*r), grad = empty_f32(*r);
  Tensor loss = at::empty({}, r->options().dtype(at::kFloat));
  cudaStream_t s = stream_of(*r);
  Tensor ws = workspace_for(r->device(), s, n * t < (1 << 20) ? (1 << 20) : n * t);
  check(rls_gae_value_loss(P(r), P(v), P(term), P(tr), boot_kind == RLS_BOOT_ROW ? P(row) : P(full), (int)boot_kind,
                           nv.data_ptr<float>(), adv.data_ptr<float>(), rets.data_ptr<float>(), grad.data_ptr<float>(),
                           loss.data_ptr<float>(), n, t, (float)gamma, (float)lambda_, (int)loss_kind, (float)delta, dt,
                           ws.data_ptr(), (size_t)ws.numel(), s),
        "rls_gae_value_loss");
  return {adv, rets, loss, grad};
}

// (advantages, returns) with observation-skip masking
std::tuple<Tensor, Tensor> op_gae_obs_skip(const Tensor& rewards, const Tensor& values, const Tensor& mask,
                                           double gamma, double lambda_) {
  OptT r = rewards, v = values, m = mask;
  const int dt = unify({&r, &v, &m});
  r = ready(r); v = ready(v); m = ready(m);
  const int64_t n = rewards.size(0), t = rewards.size(1);
  Tensor adv = empty_f32(*r), rets = empty_f32(*r);
  check(rls_gae_obs_skip(P(r), P(v), P(m), adv.data_ptr<float>(), rets.data_ptr<float>(), n, t, (float)gamma,
                         (float)lambda_, dt, stream_of(*r)),
        "rls_gae_obs_skip");
  return {adv, rets};
}

std::tuple<Tensor, Tensor> op_vtrace(const Tensor& lpt, const Tensor& lpb, const Tensor& values,
                                     const Tensor& rewards, const Tensor& terminateds, const OptT& truncateds,
                                     const OptT& bootstrap, int64_t boot_kind, double gamma, double rho_bar,
                                     double c_bar) {
  OptT a = lpt, b = lpb, v = values, r = rewards, term = terminateds, tr = truncateds;
  OptT full = boot_kind == RLS_BOOT_ROW ? OptT() : bootstrap;
  const int dt = unify({&a, &b, &v, &r, &term, &tr, &full});
  a = ready(a); b = ready(b); v = ready(v); r = ready(r); term = ready(term); tr = ready(tr); full = ready(full);
  OptT row = boot_kind == RLS_BOOT_ROW ? f32(bootstrap) : OptT();
  const int64_t n = rewards.size(0), t = rewards.size(1);
  Tensor vs = empty_f32(*r), adv = empty_f32(*r);
  cudaStream_t s = stream_of(*r);
  Tensor ws = workspace_for(r->device(), s, n * t);
  check(rls_vtrace(P(a), P(b), P(v), P(r), P(term), P(tr), boot_kind == RLS_BOOT_ROW ? P(row) : P(full),
                   (int)boot_kind, vs.data_ptr<float>(), adv.data_ptr<float>(), n, t, (float)gamma,
                   (float)rho_bar, (float)c_bar, dt, ws.data_ptr(), (size_t)ws.numel(), s),
        "rls_vtrace");
  return {vs, adv};
}

std::tuple<Tensor, Tensor> op_retrace(const Tensor& pi, const Tensor& mu, const Tensor& q, const Tensor& nq,
                                      const Tensor& actions, const Tensor& rewards, const Tensor& terminateds,
                                      const Tensor& truncateds, double gamma, double lambda_, double c_bar,
                                      double rho_bar) {
  const Tensor pi_ = f32(pi), mu_ = f32(mu), q_ = f32(q), nq_ = f32(nq), r = f32(rewards), term = f32(terminateds),
               tr = f32(truncateds);
  const Tensor act = ready(actions.scalar_type() == at::kLong ? actions : actions.to(at::kLong));
  const int64_t n = rewards.size(0), t = rewards.size(1), A = pi.size(2);
  Tensor tg = empty_f32(r), adv = empty_f32(r);
  cudaStream_t s = stream_of(r);
  Tensor ws = workspace_for(r.device(), s, n * t);
  check(rls_retrace(pi_.data_ptr<float>(), mu_.data_ptr<float>(), q_.data_ptr<float>(), nq_.data_ptr<float>(),
                    act.data_ptr<int64_t>(), r.data_ptr<float>(), term.data_ptr<float>(), tr.data_ptr<float>(),
                    tg.data_ptr<float>(), adv.data_ptr<float>(), n, t, A, (float)gamma, (float)lambda_,
                    (float)c_bar, (float)rho_bar, ws.data_ptr(), (size_t)ws.numel(), s),
        "rls_retrace");
  return {tg, adv};
}

Tensor op_lambda(const Tensor& rewards, const Tensor& next_values, const Tensor& terminateds, const OptT& truncateds,
                 const OptT& bootstrap, int64_t boot_kind, double gamma, double lambda_, int64_t t0, int64_t total,
                 const OptT& halo) {
  OptT r = rewards, nv = next_values, term = terminateds, tr = truncateds, bt = bootstrap;
  const int dt = unify({&r, &nv, &term, &tr, &bt});
  r = ready(r); nv = ready(nv); term = ready(term); tr = ready(tr); bt = ready(bt);
  const Seg seg = make_seg(t0, total, halo);
  const int64_t n = rewards.size(0), t = rewards.size(1);
  Tensor out = empty_f32(*r);
  cudaStream_t s = stream_of(*r);
  Tensor ws = workspace_for(r->device(), s, n * t);
  check(rls_lambda_returns(P(r), P(nv), P(term), P(tr), P(bt), (int)boot_kind, out.data_ptr<float>(), n, t,
                           (float)gamma, (float)lambda_, dt, seg.ptr(), ws.data_ptr(), (size_t)ws.numel(), s),
        "rls_lambda_returns");
  return out;
}

Tensor op_discounted(const Tensor& rewards, const Tensor& terminateds, const OptT& truncateds, const OptT& bootstrap,
                     int64_t boot_kind, double gamma, int64_t t0, int64_t total, const OptT& halo) {
  OptT r = rewards, term = terminateds, tr = truncateds, bt = bootstrap;
  const int dt = unify({&r, &term, &tr, &bt});
  r = ready(r); term = ready(term); tr = ready(tr); bt = ready(bt);
  const Seg seg = make_seg(t0, total, halo);
  const int64_t n = rewards.size(0), t = rewards.size(1);
  Tensor out = empty_f32(*r);
  cudaStream_t s = stream_of(*r);
  Tensor ws = workspace_for(r->device(), s, n * t);
  check(rls_discounted_returns(P(r), P(term), P(tr), P(bt), (int)boot_kind, out.data_ptr<float>(), n, t,
                               (float)gamma, dt, seg.ptr(), ws.data_ptr(), (size_t)ws.numel(), s),
        "rls_discounted_returns");
  return out;
}

Tensor op_eligibility(const Tensor& gradients, const Tensor& dones, const OptT& seed, double gamma, double lambda_,
                      int64_t t0, int64_t total, const OptT& halo) {
  OptT g = gradients, d = dones;
  const int dt = unify({&g, &d});
  g = ready(g); d = ready(d);
  const OptT sd = f32(seed);
  const Seg seg = make_seg(t0, total, halo);
  const int64_t n = gradients.size(0), t = gradients.size(1);
  Tensor out = empty_f32(*g);
  cudaStream_t s = stream_of(*g);
  Tensor ws = workspace_for(g->device(), s, n * t);
  check(rls_eligibility_traces(P(g), P(d), sd ? sd->data_ptr<float>() : nullptr, out.data_ptr<float>(), n, t,
                               (float)gamma, (float)lambda_, dt, seg.ptr(), ws.data_ptr(), (size_t)ws.numel(), s),
        "rls_eligibility_traces");
  return out;
}

Tensor op_prefix(const Tensor& inputs, const Tensor& dones, const OptT& seed, bool ends_at, int64_t t0,
                 int64_t total, const OptT& halo) {
  OptT x = inputs, d = dones;
  const int dt = unify({&x, &d});
  x = ready(x); d = ready(d);
  const OptT sd = f32(seed);
  const Seg seg = make_seg(t0, total, halo);
  const int64_t n = inputs.size(0), t = inputs.size(1);
  Tensor out = empty_f32(*x);
  cudaStream_t s = stream_of(*x);
  Tensor ws = workspace_for(x->device(), s, n * t);
  check(rls_prefix_sum(P(x), P(d), sd ? sd->data_ptr<float>() : nullptr, ends_at ? 1 : 0, out.data_ptr<float>(), n,
                       t, dt, seg.ptr(), ws.data_ptr(), (size_t)ws.numel(), s),
        "rls_prefix_sum");
  return out;
}

Tensor op_affine(const Tensor& u, const Tensor& v, const OptT& carry, int64_t direction, int64_t t0, int64_t total,
                 const OptT& halo) {
  const Tensor u_ = f32(u), v_ = f32(v);
  const OptT c = f32(carry);
  const Seg seg = make_seg(t0, total, halo);
  const int64_t n = u.size(0), t = u.size(1);
  Tensor out = empty_f32(u_);
  cudaStream_t s = stream_of(u_);
  Tensor ws = workspace_for(u_.device(), s, n * t);
  check(rls_affine_scan(u_.data_ptr<float>(), v_.data_ptr<float>(), c ? c->data_ptr<float>() : nullptr,
                        (int)direction, out.data_ptr<float>(), n, t, seg.ptr(), ws.data_ptr(), (size_t)ws.numel(), s),
        "rls_affine_scan");
  return out;
}

// The current stream's workspace on `like`'s device (for C-ABI callers that
// share it, and for reading its error latch).
Tensor op_workspace(const Tensor& like, int64_t num_elements) {
  return workspace_for(like.device(), stream_of(like), num_elements);
}

// Reads and clears the error latch of the current stream's workspace on
// `like`'s device (synchronises that stream); 0 when none exists yet.
int64_t op_workspace_error(const Tensor& like) {
  cudaStream_t s = stream_of(like);
  Tensor ws;
  {
    std::lock_guard<std::mutex> lock(g_ws_mu);
    auto it = g_ws.find(std::make_pair((int)like.device().index(), s));
    if (it == g_ws.end()) return 0;
    ws = it->second;
  }
  return rls_workspace_error(ws.data_ptr(), s);
}

}  // namespace

TORCH_LIBRARY(rl_triton, m) {
  m.def("gae(Tensor rewards, Tensor values, Tensor terminateds, Tensor? truncateds, Tensor? bootstrap, "
        "int boot_kind, float gamma, float lambda_, int t0=-1, int total=-1, Tensor? halo=None) -> Tensor");
  m.def("gae_normalized(Tensor rewards, Tensor values, Tensor terminateds, Tensor? truncateds, Tensor? bootstrap, "
        "int boot_kind, float gamma, float lambda_, float eps) -> (Tensor, Tensor)");
  m.def("gae_value_loss(Tensor rewards, Tensor values, Tensor terminateds, Tensor? truncateds, Tensor? bootstrap, "
        "int boot_kind, Tensor new_values, float gamma, float lambda_, int loss_kind, float delta) "
        "-> (Tensor, Tensor, Tensor, Tensor)");
  m.def("gae_obs_skip(Tensor rewards, Tensor values, Tensor mask, float gamma, float lambda_) -> (Tensor, Tensor)");
  m.def("vtrace(Tensor log_pi_target, Tensor log_pi_behavior, Tensor values, Tensor rewards, Tensor terminateds, "
        "Tensor? truncateds, Tensor? bootstrap, int boot_kind, float gamma, float rho_bar, float c_bar) "
        "-> (Tensor, Tensor)");
  m.def("retrace(Tensor action_probs_target, Tensor action_probs_behavior, Tensor q_values, "
        "Tensor next_q_values_all, Tensor actions, Tensor rewards, Tensor terminateds, Tensor truncateds, "
        "float gamma, float lambda_, float c_bar, float rho_bar) -> (Tensor, Tensor)");
  m.def("lambda_returns(Tensor rewards, Tensor next_values, Tensor terminateds, Tensor? truncateds, "
        "Tensor? bootstrap, int boot_kind, float gamma, float lambda_, int t0=-1, int total=-1, "
        "Tensor? halo=None) -> Tensor");
  m.def("discounted_returns(Tensor rewards, Tensor terminateds, Tensor? truncateds, Tensor? bootstrap, "
        "int boot_kind, float gamma, int t0=-1, int total=-1, Tensor? halo=None) -> Tensor");
  m.def("eligibility_traces(Tensor gradients, Tensor dones, Tensor? seed_values, float gamma, float lambda_, "
        "int t0=-1, int total=-1, Tensor? halo=None) -> Tensor");
  m.def("prefix_sum(Tensor inputs, Tensor dones, Tensor? seed_values, bool ends_at, int t0=-1, int total=-1, "
        "Tensor? halo=None) -> Tensor");
  m.def("affine_scan(Tensor u, Tensor v, Tensor? carry, int direction, int t0=-1, int total=-1, "
        "Tensor? halo=None) -> Tensor");
  m.def("workspace(Tensor like, int num_elements) -> Tensor");
  m.def("workspace_error(Tensor like) -> int");
}

TORCH_LIBRARY_IMPL(rl_triton, CUDA, m) {
  m.impl("gae", &op_gae);
  m.impl("gae_normalized", &op_gae_normalized);
  m.impl("gae_value_loss", &op_gae_value_loss);
  m.impl("gae_obs_skip", &op_gae_obs_skip);
  m.impl("vtrace", &op_vtrace);
  m.impl("retrace", &op_retrace);
  m.impl("lambda_returns", &op_lambda);
  m.impl("discounted_returns", &op_discounted);
  m.impl("eligibility_traces", &op_eligibility);
  m.impl("prefix_sum", &op_prefix);
  m.impl("affine_scan", &op_affine);
  m.impl("workspace", &op_workspace);
  m.impl("workspace_error", &op_workspace_error);
}
