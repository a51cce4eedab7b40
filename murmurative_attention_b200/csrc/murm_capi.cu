// murm_capi.cu — the C ABI (include/murm.h): argument checks, workspace
// layout, and dispatch to the kernels.
//
// Replaces the reference's torch-ext layer (torch-ext/torch_binding.cpp:6-43,
// torch-ext/wrappers.cpp:10-62) and its launchers' TORCH_CHECKs
// (src/murmurative/csrc/cuda/slot_select_attend.cu:474-490). Errors become
// status codes plus a per-thread message instead of c10::Error; no torch types
// cross this boundary.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "murm_kernels.cuh"

namespace murm {
namespace {

thread_local std::string g_last_error;

murm_status fail(murm_status s, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
murm_status fail(murm_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return s;
}

}  // namespace

// The per-phase entry points (murm_ops.cu) report through the same message.
murm_status report_error(murm_status s, const char* msg) {
  g_last_error = msg;
  return s;
}

namespace {

constexpr int kSmCount = 148;  // B200; fixes the chunking so sizes() is device-independent
static_assert(kSmCount == kMaxSplitCtas, "the forward split plans one CTA per SM");

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

murm_status check_shape(const murm_shape* s) {
  if (!s) return fail(MURM_ERR_INVALID_ARGUMENT, "shape is NULL");
  if (s->batch < 1 || s->heads < 1 || s->tokens < 1)
    return fail(MURM_ERR_INVALID_ARGUMENT, "batch, heads and tokens must be >= 1 (got %d, %d, %d)", s->batch,
                s->heads, s->tokens);
  if (s->top_k != kTopK)
    return fail(MURM_ERR_UNSUPPORTED, "top_k must be %d (the reference hard-codes k=7), got %d", kTopK, s->top_k);
  if (s->slots < kTopK)
    return fail(MURM_ERR_INVALID_ARGUMENT, "selected index k out of range: slots=%d < top_k=%d", s->slots, kTopK);
  if (s->slots > kMaxSlots) return fail(MURM_ERR_UNSUPPORTED, "slots=%d > %d not supported", s->slots, kMaxSlots);
  if (s->head_dim != 16 && s->head_dim != 32 && s->head_dim != 64)
    return fail(MURM_ERR_UNSUPPORTED, "head_dim must be 16, 32 or 64, got %d", s->head_dim);
  if (s->rounds < 0) return fail(MURM_ERR_INVALID_ARGUMENT, "rounds must be >= 0, got %d", s->rounds);
  if (s->dtype < MURM_F32 || s->dtype > MURM_BF16) return fail(MURM_ERR_DTYPE, "unsupported dtype code %d", s->dtype);
  if (!std::isfinite(s->alpha) || !std::isfinite(s->gamma) || !std::isfinite(s->scale))
    return fail(MURM_ERR_INVALID_ARGUMENT, "alpha, gamma and scale must be finite");
  const double bhn = (double)s->batch * s->heads * s->tokens;
  if (bhn * s->head_dim > 2147483647.0)
    return fail(MURM_ERR_UNSUPPORTED, "batch*heads*tokens*head_dim exceeds 2^31");
  return MURM_OK;
}

Geom make_geom(const murm_shape* s) {
  Geom g{};
  g.B = s->batch; g.H = s->heads; g.N = s->tokens; g.M = s->slots; g.D = s->head_dim; g.R = s->rounds;
  g.causal = s->causal ? 1 : 0;
  g.dtype = s->dtype;
  g.BH = g.B * g.H;
  // Python floats are doubles; the reference multiplies fp32 tensors by them,
  // which rounds each scalar to fp32 once (reference.py:112-113, 128-133).
  g.alpha = (float)s->alpha;
  g.one_minus_alpha = (float)(1.0 - s->alpha);
  g.gamma = (float)s->gamma;
  g.scale = (float)(s->scale > 0 ? s->scale : 1.0 / std::sqrt((double)s->head_dim));
  const int tiles = (g.N + kTile - 1) / kTile;
  // CUDA-core path's reduction kernels: one wave, at most one chunk per SM
  int red = kSmCount / g.BH;
  red = red < 1 ? 1 : (red > tiles ? tiles : red);
  const int tiles_per = (tiles + red - 1) / red;
  g.red_chunk_tokens = tiles_per * kTile;
  g.red_chunks = (g.N + g.red_chunk_tokens - 1) / g.red_chunk_tokens;
  // the backward token kernel splits each (b,h) at its own 64-token granularity: on 16 pairs of
  // 8192 tokens, 9 chunks of at most 15 tiles (144 CTAs) instead of 8 of 16
  const int btiles = (g.N + kBwdTile - 1) / kBwdTile;
  int bred = kSmCount / g.BH;
  bred = bred < 1 ? 1 : (bred > btiles ? btiles : bred);
  g.bwd_chunk_tokens = ((btiles + bred - 1) / bred) * kBwdTile;
  g.bwd_chunks = (g.N + g.bwd_chunk_tokens - 1) / g.bwd_chunk_tokens;
  TileSplit split;  // the plan of the forward launch (kMaxSplitCtas CTAs)
  plan_split(g.BH, g.N, kTile, kSmCount, &split);
  g.ft_parts = max_parts(split);
  return g;
}

struct Sizes {
  size_t saved, fwd_ws, bwd_ws;
  // offsets inside each block
  size_t sK, sV, sU, sW, sIdx, sw;
  size_t fS, fW, fImg, fCnt, fAmax, fExp;
  size_t bdK0, bdK1, bdV0, bdV1, bdS, bdW, bdKdir, bdVdir, bdKpart, bdVpart, bcoef, bdq, btab, bamax;
};

Sizes make_sizes(const Geom& g) {
  Sizes z{};
  const size_t R = (size_t)g.R, BH = (size_t)g.BH, M = (size_t)g.M, D = (size_t)g.D, N = (size_t)g.N;
  const size_t slot = BH * M * D * 4;
  size_t o = 0;
  auto take = [&o](size_t bytes) { const size_t at = o; o += align256(bytes); return at; };
  z.sK = take(R * slot);
  z.sV = take(R * slot);
  z.sU = take(R * slot);
  z.sW = take(R * BH * M * 4);
  z.sIdx = take(R * BH * N * 8);
  z.sw = take(R * BH * N * 8 * 4);
  z.saved = o;
  o = 0;
  const size_t fparts = (size_t)(g.ft_parts > g.red_chunks ? g.ft_parts : g.red_chunks);
  z.fS = take(BH * fparts * M * D * 4);
  z.fW = take(BH * fparts * M * 4);
  // operand images of the tensor-core path (16-bit dtypes, head_dim 64)
  z.fImg = take(tc_images_bytes(g));
  z.fCnt = take(2 * BH * sizeof(int));  // the multi-round tensor-core launch's counters per pair
  z.fAmax = take(BH * kAmaxBlocks * 3 * sizeof(float));
  z.fExp = take(BH * 4 * sizeof(int));
  z.fwd_ws = o;
  o = 0;
  z.bdK0 = take(slot); z.bdK1 = take(slot); z.bdV0 = take(slot); z.bdV1 = take(slot);
  z.bdS = take(slot); z.bdW = take(BH * M * 4); z.bdKdir = take(slot); z.bdVdir = take(slot);
  const size_t bparts = (size_t)(g.bwd_chunks > g.red_chunks ? g.bwd_chunks : g.red_chunks);
  z.bdKpart = take(BH * bparts * M * D * 4);
  z.bdVpart = take(BH * bparts * M * D * 4);
  z.bcoef = take(BH * N * 8 * 4);
  z.bdq = take(BH * N * D * 4);
  z.btab = take(tc_bwd_tables_bytes(g));
  z.bamax = take(BH * 64 * sizeof(float));
  z.bwd_ws = o;
  return z;
}

Saved saved_views(const Sizes& z, void* base) {
  char* p = static_cast<char*>(base);
  Saved s;
  s.K = reinterpret_cast<float*>(p + z.sK);
  s.V = reinterpret_cast<float*>(p + z.sV);
  s.U = reinterpret_cast<float*>(p + z.sU);
  s.W = reinterpret_cast<float*>(p + z.sW);
  s.idx = reinterpret_cast<uint8_t*>(p + z.sIdx);
  s.w = reinterpret_cast<float*>(p + z.sw);
  return s;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

murm_status check_tensor(const void* p, const int64_t* st, const char* name, bool allow_zero_batch) {
  if (!p) return fail(MURM_ERR_INVALID_ARGUMENT, "%s is NULL", name);
  if (!aligned(p, 16)) return fail(MURM_ERR_INVALID_ARGUMENT, "%s is not 16-byte aligned", name);
  for (int i = 0; i < 3; ++i) {
    if (st[i] < 0) return fail(MURM_ERR_INVALID_ARGUMENT, "%s stride[%d] is negative", name, i);
    if (st[i] == 0 && !(i == 0 && allow_zero_batch))
      return fail(MURM_ERR_INVALID_ARGUMENT, "%s stride[%d] is zero", name, i);
  }
  return MURM_OK;
}

murm_status cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return MURM_OK;
  return fail(MURM_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// Forward dispatch: tensor-core rounds for fp16/bf16 at head_dim 64, CUDA-core
// rounds otherwise (fp32 inputs keep exact fp32 selection arithmetic).
murm_status run_forward(const Geom& g, const FwdPtrs& p, const Saved& sv, const FwdScratch& fs, cudaStream_t st) {
  cudaError_t e = cudaSuccess;
  const bool tc = tc_forward_supported(g, g.dtype, p);
  switch (g.dtype) {
    case MURM_F32: e = fwd_simt<float>(g, p, sv, fs, st); break;
    case MURM_F16: e = tc ? fwd_tc<__half>(g, p, sv, fs, st) : fwd_simt<__half>(g, p, sv, fs, st); break;
    case MURM_BF16:
      e = tc ? fwd_tc<__nv_bfloat16>(g, p, sv, fs, st) : fwd_simt<__nv_bfloat16>(g, p, sv, fs, st);
      break;
  }
  return cuda_status(e, tc ? "slot_murmurate forward (tensor-core) launch" : "slot_murmurate forward launch");
}

}  // namespace
}  // namespace murm

using namespace murm;

extern "C" {

int32_t murm_abi_version(void) { return MURM_ABI_VERSION; }

const char* murm_status_string(murm_status s) {
  switch (s) {
    case MURM_OK: return "ok";
    case MURM_ERR_INVALID_ARGUMENT: return "invalid argument";
    case MURM_ERR_UNSUPPORTED: return "unsupported";
    case MURM_ERR_DTYPE: return "unsupported dtype";
    case MURM_ERR_WORKSPACE: return "workspace too small or misaligned";
    case MURM_ERR_CUDA: return "CUDA error";
    case MURM_ERR_DEVICE: return "device-side error";
  }
  return "unknown status";
}

const char* murm_last_error_message(void) { return g_last_error.c_str(); }

murm_status murm_device_status(void* stream) {
  int code = 0;
  cudaError_t e = read_and_clear_device_error(&code, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_status(e, "murm_device_status");
  if (code)
    return fail(MURM_ERR_DEVICE, "a kernel gave up waiting (error bits 0x%x: 1 operand copy, 2 token tile copy, "
                "4 tensor-core completion, 8 backward copy or MMA, 16 wait probe, 32 another CTA's round)", code);
  return MURM_OK;
}

murm_status murm_wait_probe(int32_t arrive, uint64_t limit_ns, void* stream) {
  if (limit_ns == 0 || limit_ns > 10000000000ull)
    return fail(MURM_ERR_INVALID_ARGUMENT, "limit_ns must be in (0, 10 s], got %llu", (unsigned long long)limit_ns);
  return cuda_status(launch_wait_probe(arrive ? 1 : 0, limit_ns, static_cast<cudaStream_t>(stream)),
                     "wait probe launch");
}

murm_status murm_slot_murmurate_sizes(const murm_shape* shape, size_t* saved, size_t* fwd_ws, size_t* bwd_ws) {
  if (murm_status s = check_shape(shape)) return s;
  const Sizes z = make_sizes(make_geom(shape));
  if (saved) *saved = z.saved;
  if (fwd_ws) *fwd_ws = z.fwd_ws;
  if (bwd_ws) *bwd_ws = z.bwd_ws;
  return MURM_OK;
}

}  // extern "C"

namespace murm {
namespace {
murm_status forward_entry(const murm_fwd_args* a, void* stream, int slots_f32) {
  if (!a) return fail(MURM_ERR_INVALID_ARGUMENT, "args is NULL");
  if (murm_status s = check_shape(&a->shape)) return s;
  const Geom g = make_geom(&a->shape);
  const Sizes z = make_sizes(g);
  if (murm_status s = check_tensor(a->q, a->q_stride, "q", false)) return s;
  if (murm_status s = check_tensor(a->slots_k, a->sk_stride, "slots_k", true)) return s;
  if (murm_status s = check_tensor(a->slots_v, a->sv_stride, "slots_v", true)) return s;
  if (murm_status s = check_tensor(a->out, a->out_stride, "out", false)) return s;
  if (z.saved && (!a->saved || !aligned(a->saved, 256) || a->saved_bytes < z.saved))
    return fail(MURM_ERR_WORKSPACE, "saved block needs %zu bytes, 256-byte aligned (got %zu)", z.saved,
                a->saved_bytes);
  if (z.fwd_ws && (!a->workspace || !aligned(a->workspace, 256) || a->workspace_bytes < z.fwd_ws))
    return fail(MURM_ERR_WORKSPACE, "forward workspace needs %zu bytes, 256-byte aligned (got %zu)", z.fwd_ws,
                a->workspace_bytes);
  FwdPtrs p;
  p.q = a->q; p.sk = a->slots_k; p.sv = a->slots_v; p.out = a->out;
  for (int i = 0; i < 3; ++i) {
    p.qs.s[i] = a->q_stride[i]; p.sks.s[i] = a->sk_stride[i]; p.svs.s[i] = a->sv_stride[i];
    p.os.s[i] = a->out_stride[i];
  }
  p.indices = a->indices;
  p.weights = a->weights;
  p.slots_f32 = slots_f32;
  const Saved sv = saved_views(z, a->saved);
  FwdScratch fs;
  fs.Spart = reinterpret_cast<float*>(static_cast<char*>(a->workspace) + z.fS);
  fs.Wpart = reinterpret_cast<float*>(static_cast<char*>(a->workspace) + z.fW);
  fs.images = reinterpret_cast<uint8_t*>(static_cast<char*>(a->workspace) + z.fImg);
  fs.counters = reinterpret_cast<int*>(static_cast<char*>(a->workspace) + z.fCnt);
  fs.amax = reinterpret_cast<float*>(static_cast<char*>(a->workspace) + z.fAmax);
  fs.fexp = reinterpret_cast<int*>(static_cast<char*>(a->workspace) + z.fExp);
  return run_forward(g, p, sv, fs, static_cast<cudaStream_t>(stream));
}
}  // namespace
}  // namespace murm

extern "C" {

murm_status murm_slot_murmurate_fwd(const murm_fwd_args* a, void* stream) { return forward_entry(a, stream, 0); }

murm_status murm_slot_murmurate_fwd_f32_slots(const murm_fwd_args* a, void* stream) {
  return forward_entry(a, stream, 1);
}

murm_status murm_slot_murmurate_bwd(const murm_bwd_args* a, void* stream) {
  if (!a) return fail(MURM_ERR_INVALID_ARGUMENT, "args is NULL");
  if (murm_status s = check_shape(&a->shape)) return s;
  const Geom g = make_geom(&a->shape);
  const Sizes z = make_sizes(g);
  if (murm_status s = check_tensor(a->q, a->q_stride, "q", false)) return s;
  if (murm_status s = check_tensor(a->grad_out, a->go_stride, "grad_out", false)) return s;
  if (murm_status s = check_tensor(a->grad_q, a->gq_stride, "grad_q", false)) return s;
  if (murm_status s = check_tensor(a->grad_slots_k, a->gsk_stride, "grad_slots_k", false)) return s;
  if (murm_status s = check_tensor(a->grad_slots_v, a->gsv_stride, "grad_slots_v", false)) return s;
  if (a->grad_weights && !aligned(a->grad_weights, 16))
    return fail(MURM_ERR_INVALID_ARGUMENT, "grad_weights is not 16-byte aligned");
  if (z.saved && (!a->saved || !aligned(a->saved, 256) || a->saved_bytes < z.saved))
    return fail(MURM_ERR_WORKSPACE, "saved block needs %zu bytes (got %zu)", z.saved, a->saved_bytes);
  if (!a->workspace || !aligned(a->workspace, 256) || a->workspace_bytes < z.bwd_ws)
    return fail(MURM_ERR_WORKSPACE, "backward workspace needs %zu bytes, 256-byte aligned (got %zu)", z.bwd_ws,
                a->workspace_bytes);
  BwdPtrs p;
  p.q = a->q; p.go = a->grad_out; p.gw = a->grad_weights; p.gq = a->grad_q;
  p.gsk = a->grad_slots_k; p.gsv = a->grad_slots_v;
  for (int i = 0; i < 3; ++i) {
    p.qs.s[i] = a->q_stride[i]; p.gos.s[i] = a->go_stride[i]; p.gqs.s[i] = a->gq_stride[i];
    p.gsks.s[i] = a->gsk_stride[i]; p.gsvs.s[i] = a->gsv_stride[i];
  }
  const Saved sv = saved_views(z, const_cast<void*>(a->saved));
  char* w = static_cast<char*>(a->workspace);
  BwdScratch bs;
  bs.dK[0] = reinterpret_cast<float*>(w + z.bdK0); bs.dK[1] = reinterpret_cast<float*>(w + z.bdK1);
  bs.dV[0] = reinterpret_cast<float*>(w + z.bdV0); bs.dV[1] = reinterpret_cast<float*>(w + z.bdV1);
  bs.dS = reinterpret_cast<float*>(w + z.bdS); bs.dW = reinterpret_cast<float*>(w + z.bdW);
  bs.dKdir = reinterpret_cast<float*>(w + z.bdKdir); bs.dVdir = reinterpret_cast<float*>(w + z.bdVdir);
  bs.dKpart = reinterpret_cast<float*>(w + z.bdKpart); bs.dVpart = reinterpret_cast<float*>(w + z.bdVpart);
  bs.coef = reinterpret_cast<float*>(w + z.bcoef); bs.dq = reinterpret_cast<float*>(w + z.bdq);
  bs.tables = reinterpret_cast<uint8_t*>(w + z.btab);
  bs.amax = reinterpret_cast<float*>(w + z.bamax);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
  const bool tc = tc_backward_supported(g, g.dtype, p);
  switch (a->shape.dtype) {
    case MURM_F32: e = bwd_simt<float>(g, p, sv, bs, st); break;
    case MURM_F16: e = tc ? bwd_tc<__half>(g, p, sv, bs, st) : bwd_simt<__half>(g, p, sv, bs, st); break;
    case MURM_BF16:
      e = tc ? bwd_tc<__nv_bfloat16>(g, p, sv, bs, st) : bwd_simt<__nv_bfloat16>(g, p, sv, bs, st);
      break;
  }
  return cuda_status(e, tc ? "slot_murmurate backward (tensor-core) launch" : "slot_murmurate backward launch");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Forward without caller scratch (murm_slot_murmurate_fwd_noscratch)
// ---------------------------------------------------------------------------
namespace murm {
namespace {

constexpr size_t kNoScratchBytes = MURM_NOSCRATCH_BYTES;
constexpr int kMaxDevices = 64;

// The scratch of murm_slot_murmurate_fwd_noscratch: round records + partial
// sums. In host code `g_noscratch` is only a host-side stand-in for the
// symbol; kernels get the device address looked up below.
static __device__ __align__(256) unsigned char g_noscratch[kNoScratchBytes];

std::mutex g_noscratch_mu;
void* g_noscratch_addr[kMaxDevices] = {};

// Device address of g_noscratch on the current device (looked up once per device).
murm_status noscratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(MURM_ERR_UNSUPPORTED, "device ordinal %d >= %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> lk(g_noscratch_mu);
  if (!g_noscratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noscratch);
    if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(built-in scratch)");
    g_noscratch_addr[dev] = p;
  }
  *out = g_noscratch_addr[dev];
  return MURM_OK;
}

}  // namespace
}  // namespace murm

extern "C" murm_status murm_slot_murmurate_fwd_noscratch(const murm_fwd_args* a, void* stream) {
  if (!a) return fail(MURM_ERR_INVALID_ARGUMENT, "args is NULL");
  if (murm_status s = check_shape(&a->shape)) return s;
  if (a->saved || a->saved_bytes || a->workspace || a->workspace_bytes)
    return fail(MURM_ERR_INVALID_ARGUMENT,
                "murm_slot_murmurate_fwd_noscratch uses its built-in scratch: saved/workspace must be NULL and 0");
  const Geom g = make_geom(&a->shape);
  const Sizes z = make_sizes(g);
  const size_t need = z.saved + z.fwd_ws;  // both already multiples of 256
  if (need > kNoScratchBytes)
    return fail(MURM_ERR_WORKSPACE,
                "problem needs %zu bytes of scratch; the built-in scratch of murm_slot_murmurate_fwd_noscratch "
                "holds %zu bytes (use murm_slot_murmurate_fwd with caller-provided buffers)",
                need, kNoScratchBytes);
  if (murm_status s = check_tensor(a->q, a->q_stride, "q", false)) return s;
  if (murm_status s = check_tensor(a->slots_k, a->sk_stride, "slots_k", true)) return s;
  if (murm_status s = check_tensor(a->slots_v, a->sv_stride, "slots_v", true)) return s;
  if (murm_status s = check_tensor(a->out, a->out_stride, "out", false)) return s;
  void* base = nullptr;
  if (murm_status s = noscratch_address(&base)) return s;
  FwdPtrs p;
  p.q = a->q; p.sk = a->slots_k; p.sv = a->slots_v; p.out = a->out;
  for (int i = 0; i < 3; ++i) {
    p.qs.s[i] = a->q_stride[i]; p.sks.s[i] = a->sk_stride[i]; p.svs.s[i] = a->sv_stride[i];
    p.os.s[i] = a->out_stride[i];
  }
  p.indices = a->indices;
  p.weights = a->weights;
  // Every byte of the scratch that a kernel reads is written earlier in the
  // same call, so nothing needs clearing between calls.
  const Saved sv = saved_views(z, base);
  FwdScratch fs;
  fs.Spart = reinterpret_cast<float*>(static_cast<char*>(base) + z.saved + z.fS);
  fs.Wpart = reinterpret_cast<float*>(static_cast<char*>(base) + z.saved + z.fW);
  fs.images = reinterpret_cast<uint8_t*>(static_cast<char*>(base) + z.saved + z.fImg);
  fs.counters = reinterpret_cast<int*>(static_cast<char*>(base) + z.saved + z.fCnt);
  fs.amax = reinterpret_cast<float*>(static_cast<char*>(base) + z.saved + z.fAmax);
  fs.fexp = reinterpret_cast<int*>(static_cast<char*>(base) + z.saved + z.fExp);
  return run_forward(g, p, sv, fs, static_cast<cudaStream_t>(stream));
}
