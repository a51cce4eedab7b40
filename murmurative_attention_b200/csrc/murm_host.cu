// murm_host.cu — forward + backward over host buffers, copies overlapped with compute.
//
// murm_slot_murmurate_host_step is the drop-in for a caller whose tensors live in host
// memory (the reference's CPU path: reference.py:138-191 and its autograd backward).
// The (batch, head) pairs are independent, so the call splits them into groups and runs a
// three-stage pipeline: inputs are copied in on one stream, the groups' forwards and then
// their backwards run on the caller's stream, results are copied out on a third, so the
// host<->device copies (both directions at once) overlap the kernels. q and the slots of
// every group go in first and grad_out after them; the forwards' outputs (out, indices,
// weights: most of the bytes out) start copying out as soon as the first forward is done,
// and the gradients follow the backwards.
// No kernels of its own: each group goes through murm_slot_murmurate_fwd / _bwd.
#include <mutex>
#include <vector>

#include "murm_kernels.cuh"

namespace murm {
namespace {

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

size_t elem_bytes(int dtype) { return dtype == MURM_F32 ? 4 : 2; }

// One device's copy streams and events, created on first use and kept for the process.
struct HostPipe {
  cudaStream_t in = nullptr, out = nullptr;
  std::vector<cudaEvent_t> ev;  // [0] start, [1] copies out done, [2] copies in done, then 4 per group
};
std::mutex g_pipe_mu;
std::mutex g_call_mu;
std::vector<HostPipe> g_pipes;

cudaError_t pipe_for(int device, int groups, HostPipe** out) {
  std::lock_guard<std::mutex> lk(g_pipe_mu);
  if ((int)g_pipes.size() <= device) g_pipes.resize(device + 1);
  HostPipe& p = g_pipes[device];
  cudaError_t e = cudaSuccess;
  if (!p.in) e = cudaStreamCreateWithFlags(&p.in, cudaStreamNonBlocking);
  if (e == cudaSuccess && !p.out) e = cudaStreamCreateWithFlags(&p.out, cudaStreamNonBlocking);
  while (e == cudaSuccess && (int)p.ev.size() < 3 + 4 * groups) {
    cudaEvent_t ev;
    e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
    if (e == cudaSuccess) p.ev.push_back(ev);
  }
  *out = &p;
  return e;
}

constexpr int kMaxGroups = 64;
struct HostLayout {
  int groups;
  int64_t start[kMaxGroups + 1];    // group g holds the (b,h) pairs [start[g], start[g+1])
  size_t q, go, sk, sv, out, idx, w, gq, gsk, gsv;  // offsets of the full-size device copies
  size_t saved[kMaxGroups];         // each group's saved block (kept from its forward to its backward)
  size_t saved_bytes[kMaxGroups];
  size_t fws, bws, fws_bytes, bws_bytes, total;  // workspaces sized for the largest group
};

murm_status plan(const murm_shape* s, int32_t groups, HostLayout* L) {
  if (!s) return report_error(MURM_ERR_INVALID_ARGUMENT, "shape is NULL");
  const int64_t bh = (int64_t)s->batch * s->heads;
  if (bh < 1) return report_error(MURM_ERR_INVALID_ARGUMENT, "batch * heads must be >= 1");
  // automatic: groups of at least 4 (b,h) pairs (smaller ones leave the round kernels' grids
  // short of work), at least two groups so that copies overlap compute, at most 8. (Groups that
  // grow from a small first one, to start the copies out earlier, measured no faster.)
  int64_t want = groups > 0 ? groups : (bh / 4 > 8 ? 8 : (bh / 4 > 2 ? bh / 4 : 2));
  if (want > bh) want = bh;
  if (want > kMaxGroups) want = kMaxGroups;
  const int64_t per = (bh + want - 1) / want;
  int G = 0;
  L->start[0] = 0;
  for (int64_t p = 0; p < bh; p += per) L->start[++G] = p + per < bh ? p + per : bh;
  L->groups = G;
  size_t fws_max = 0, bws_max = 0;
  for (int g = 0; g < G; ++g) {
    murm_shape gs = *s;
    gs.batch = 1;
    gs.heads = (int32_t)(L->start[g + 1] - L->start[g]);
    size_t f = 0, b = 0;
    if (murm_status st = murm_slot_murmurate_sizes(&gs, &L->saved_bytes[g], &f, &b)) return st;
    fws_max = f > fws_max ? f : fws_max;
    bws_max = b > bws_max ? b : bws_max;
  }
  L->fws_bytes = fws_max;
  L->bws_bytes = bws_max;
  const size_t es = elem_bytes(s->dtype);
  const size_t tok = (size_t)bh * s->tokens, slot = (size_t)bh * s->slots;
  size_t o = 0;
  auto take = [&](size_t b) { const size_t at = o; o += align256(b); return at; };
  L->q = take(tok * s->head_dim * es);
  L->go = take(tok * s->head_dim * es);
  L->sk = take(slot * s->head_dim * es);
  L->sv = take(slot * s->head_dim * es);
  L->out = take(tok * s->head_dim * es);
  L->idx = take(tok * MURM_TOP_K * 8);
  L->w = take(tok * MURM_TOP_K * 4);
  L->gq = take(tok * s->head_dim * es);
  L->gsk = take(slot * s->head_dim * es);
  L->gsv = take(slot * s->head_dim * es);
  for (int g = 0; g < G; ++g) L->saved[g] = take(L->saved_bytes[g]);
  L->fws = take(L->fws_bytes);
  L->bws = take(L->bws_bytes);
  L->total = o;
  return MURM_OK;
}

}  // namespace
}  // namespace murm

using namespace murm;

extern "C" {

murm_status murm_host_step_sizes(const murm_shape* shape, int32_t groups, size_t* workspace_bytes) {
  HostLayout L;
  if (murm_status s = plan(shape, groups, &L)) return s;
  if (workspace_bytes) *workspace_bytes = L.total;
  return MURM_OK;
}

murm_status murm_slot_murmurate_host_step(const murm_host_step_args* a, void* stream) {
  if (!a) return report_error(MURM_ERR_INVALID_ARGUMENT, "args is NULL");
  HostLayout L;
  if (murm_status s = plan(&a->shape, a->groups, &L)) return s;
  if (!a->q || !a->slots_k || !a->slots_v || !a->grad_out || !a->out || !a->grad_q || !a->grad_slots_k ||
      !a->grad_slots_v)
    return report_error(MURM_ERR_INVALID_ARGUMENT, "q, slots, grad_out, out and the three gradients are required");
  if (!a->workspace || (reinterpret_cast<uintptr_t>(a->workspace) & 255) || a->workspace_bytes < L.total)
    return report_error(MURM_ERR_WORKSPACE, "host-step workspace too small or not 256-byte aligned");
  const murm_shape& s = a->shape;
  const size_t es = elem_bytes(s.dtype);
  const int64_t N = s.tokens, M = s.slots, D = s.head_dim;
  const size_t tokb = (size_t)N * D * es, slotb = (size_t)M * D * es;  // bytes per (b,h) pair
  const size_t recn = (size_t)N * MURM_TOP_K;
  char* ws = static_cast<char*>(a->workspace);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return report_error(MURM_ERR_CUDA, "cudaGetDevice failed");
  std::lock_guard<std::mutex> call_lk(g_call_mu);  // one device's streams and events: one call at a time
  HostPipe* pp = nullptr;
  if (cudaError_t e = pipe_for(dev, L.groups, &pp))
    return report_error(MURM_ERR_CUDA, cudaGetErrorString(e));
  HostPipe& P = *pp;
  const int64_t bh = (int64_t)s.batch * s.heads;
  auto H2D = [&](size_t dev_off, const void* host, size_t off, size_t bytes) {
    return cudaMemcpyAsync(ws + dev_off + off, static_cast<const char*>(host) + off, bytes, cudaMemcpyHostToDevice,
                           P.in);
  };
  auto D2H = [&](void* host, size_t dev_off, size_t off, size_t bytes) {
    return cudaMemcpyAsync(static_cast<char*>(host) + off, ws + dev_off + off, bytes, cudaMemcpyDeviceToHost, P.out);
  };
  cudaError_t e = cudaEventRecord(P.ev[0], st);  // the copies start after the caller's earlier work
  if (!e) e = cudaStreamWaitEvent(P.in, P.ev[0], 0);
  if (!e) e = cudaStreamWaitEvent(P.out, P.ev[0], 0);
  auto pairs = [&](int g, int64_t* p0, int64_t* np) {
    *p0 = L.start[g];
    *np = L.start[g + 1] - L.start[g];
  };
  // per group: q + slots copied in, grad_out copied in, forward done, backward done
  auto ev = [&](int g, int k) { return P.ev[3 + 4 * g + k]; };
  // every exit leaves the caller's stream behind both copy streams, so that work the caller
  // orders after this call (freeing the workspace, reading the host buffers) sees them finished
  auto join = [&]() {
    cudaError_t j = cudaEventRecord(P.ev[2], P.in);
    if (!j) j = cudaStreamWaitEvent(st, P.ev[2], 0);
    if (!j) j = cudaEventRecord(P.ev[1], P.out);
    if (!j) j = cudaStreamWaitEvent(st, P.ev[1], 0);
    return j;
  };
  auto fail_cuda = [&](cudaError_t err) {
    join();
    return report_error(MURM_ERR_CUDA, cudaGetErrorString(err));
  };
  // ---- copies in: q and slots of every group, then grad_out ----
  for (int g = 0; g < L.groups && !e; ++g) {
    int64_t p0, np;
    pairs(g, &p0, &np);
    e = H2D(L.q, a->q, p0 * tokb, np * tokb);
    if (!e) e = H2D(L.sk, a->slots_k, p0 * slotb, np * slotb);
    if (!e) e = H2D(L.sv, a->slots_v, p0 * slotb, np * slotb);
    if (!e) e = cudaEventRecord(ev(g, 0), P.in);
  }
  for (int g = 0; g < L.groups && !e; ++g) {
    int64_t p0, np;
    pairs(g, &p0, &np);
    e = H2D(L.go, a->grad_out, p0 * tokb, np * tokb);
    if (!e) e = cudaEventRecord(ev(g, 1), P.in);
  }
  if (e) return fail_cuda(e);
  // ---- forwards, then backwards, on the caller's stream ----
  const int64_t ts[3] = {bh * N * D, N * D, D}, ss[3] = {bh * M * D, M * D, D};  // batch stride unused (B = 1)
  auto group_shape = [&](int64_t np) {
    murm_shape gs = s;
    gs.batch = 1;
    gs.heads = (int32_t)np;
    return gs;
  };
  for (int g = 0; g < L.groups && !e; ++g) {
    int64_t p0, np;
    pairs(g, &p0, &np);
    if ((e = cudaStreamWaitEvent(st, ev(g, 0), 0))) break;
    murm_fwd_args f{};
    f.shape = group_shape(np);
    f.q = ws + L.q + p0 * tokb;
    f.slots_k = ws + L.sk + p0 * slotb;
    f.slots_v = ws + L.sv + p0 * slotb;
    f.out = ws + L.out + p0 * tokb;
    for (int i = 0; i < 3; ++i) {
      f.q_stride[i] = f.out_stride[i] = ts[i];
      f.sk_stride[i] = f.sv_stride[i] = ss[i];
    }
    f.indices = reinterpret_cast<int64_t*>(ws + L.idx) + p0 * recn;
    f.weights = reinterpret_cast<float*>(ws + L.w) + p0 * recn;
    f.saved = ws + L.saved[g];
    f.saved_bytes = L.saved_bytes[g];
    f.workspace = ws + L.fws;
    f.workspace_bytes = L.fws_bytes;
    if (murm_status ms = murm_slot_murmurate_fwd(&f, st)) {
      join();
      return ms;
    }
    e = cudaEventRecord(ev(g, 2), st);
  }
  for (int g = 0; g < L.groups && !e; ++g) {
    int64_t p0, np;
    pairs(g, &p0, &np);
    if ((e = cudaStreamWaitEvent(st, ev(g, 1), 0))) break;
    murm_bwd_args bw{};
    bw.shape = group_shape(np);
    bw.q = ws + L.q + p0 * tokb;
    bw.grad_out = ws + L.go + p0 * tokb;
    bw.saved = ws + L.saved[g];
    bw.saved_bytes = L.saved_bytes[g];
    bw.grad_q = ws + L.gq + p0 * tokb;
    bw.grad_slots_k = ws + L.gsk + p0 * slotb;
    bw.grad_slots_v = ws + L.gsv + p0 * slotb;
    for (int i = 0; i < 3; ++i) {
      bw.q_stride[i] = bw.go_stride[i] = bw.gq_stride[i] = ts[i];
      bw.gsk_stride[i] = bw.gsv_stride[i] = ss[i];
    }
    bw.workspace = ws + L.bws;
    bw.workspace_bytes = L.bws_bytes;
    if (murm_status ms = murm_slot_murmurate_bwd(&bw, st)) {
      join();
      return ms;
    }
    e = cudaEventRecord(ev(g, 3), st);
  }
  // ---- copies out: each forward's results, then each backward's gradients ----
  for (int g = 0; g < L.groups && !e; ++g) {
    int64_t p0, np;
    pairs(g, &p0, &np);
    e = cudaStreamWaitEvent(P.out, ev(g, 2), 0);
    if (!e) e = D2H(a->out, L.out, p0 * tokb, np * tokb);
    if (!e && a->indices) e = D2H(a->indices, L.idx, p0 * recn * 8, np * recn * 8);
    if (!e && a->weights) e = D2H(a->weights, L.w, p0 * recn * 4, np * recn * 4);
  }
  for (int g = 0; g < L.groups && !e; ++g) {
    int64_t p0, np;
    pairs(g, &p0, &np);
    e = cudaStreamWaitEvent(P.out, ev(g, 3), 0);
    if (!e) e = D2H(a->grad_q, L.gq, p0 * tokb, np * tokb);
    if (!e) e = D2H(a->grad_slots_k, L.gsk, p0 * slotb, np * slotb);
    if (!e) e = D2H(a->grad_slots_v, L.gsv, p0 * slotb, np * slotb);
  }
  if (e) return fail_cuda(e);
  // the caller's stream completes after the last copy out
  if ((e = join())) return report_error(MURM_ERR_CUDA, cudaGetErrorString(e));
  return MURM_OK;
}

}  // extern "C"
