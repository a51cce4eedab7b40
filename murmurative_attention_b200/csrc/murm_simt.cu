// murm_simt.cu — CUDA-core kernels of the slot_murmurate round loop.
//
// Reference semantics: src/murmurative/reference.py:138-191 (round loop) with
// select  reference.py:6-39, attend reference.py:42-68, update
// reference.py:71-115, diffusion reference.py:118-135; token keys = token
// values = q and a zero residual stream.
//
// These kernels are exact fp32 arithmetic on CUDA cores. They serve every
// element type; the fp16/bf16 forward selection also has a tensor-core
// (tcgen05) kernel in murm_tc.cu. All reductions over tokens are
// deterministic: per tile, the (token, pick) entries are grouped by slot with a
// counting sort whose order is fixed by the token index, each slot is summed
// by exactly one thread in that order, and tile / chunk partials are combined
// in index order. No floating-point atomics are used anywhere.
#include "murm_kernels.cuh"

namespace murm {

// ---------------------------------------------------------------------------
// helpers
// ---------------------------------------------------------------------------
template <typename T, int D>
__device__ __forceinline__ void load_row(const T* p, float (&v)[D]) {
#pragma unroll
  for (int c = 0; c < D; ++c) v[c] = Elem<T>::load(p + c);
}

// Dot product of a register row with a shared-memory row. Four interleaved
// partial sums for instruction-level parallelism; the same function computes
// selection scores and attend logits, so both see bit-identical values.
template <int D>
__device__ __forceinline__ float dot_row(const float (&q)[D], const float* __restrict__ k) {
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  const float4* k4 = reinterpret_cast<const float4*>(k);
#pragma unroll
  for (int c = 0; c < D / 4; ++c) {
    const float4 x = k4[c];
    a0 = fmaf(q[4 * c + 0], x.x, a0);
    a1 = fmaf(q[4 * c + 1], x.y, a1);
    a2 = fmaf(q[4 * c + 2], x.z, a2);
    a3 = fmaf(q[4 * c + 3], x.w, a3);
  }
  return (a0 + a1) + (a2 + a3);
}

__device__ __forceinline__ void copy_to_smem(float* dst, const float* src, int n) {
  const float4* s4 = reinterpret_cast<const float4*>(src);
  float4* d4 = reinterpret_cast<float4*>(dst);
  for (int i = threadIdx.x; i < n / 4; i += blockDim.x) d4[i] = s4[i];
}

// Block-wide exclusive scan of cnt (one value per thread, blockDim.x == 256).
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_sums) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int s = lane < (int)(blockDim.x >> 5) ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < (int)(blockDim.x >> 5)) warp_sums[lane] = s;
  }
  __syncthreads();
  const int before = warp ? warp_sums[warp - 1] : 0;
  return before + x - v;
}

// Per-tile grouping of the tile's (token, pick) entries by slot, in token
// order. Entries are (token t in [0,nt), pick j in [0,7)). On return
// off[m]..off[m+1] index the entries of slot m in csr_t / csr_j.
struct TileCsr {
  uint32_t* mask;  // [M][4] token bitmask per slot
  int* off;        // [M+1]
  uint8_t* csr_t;  // [kTile * 7]
  uint8_t* csr_j;  // [kTile * 7]
  int* warp_sums;  // [8]
};

__device__ void build_tile_csr(const TileCsr& cs, const uint8_t* tidx /*[kTile][8]*/, int nt, int M) {
  for (int i = threadIdx.x; i < M * 4; i += blockDim.x) cs.mask[i] = 0u;
  __syncthreads();
  for (int e = threadIdx.x; e < nt * kTopK; e += blockDim.x) {
    const int t = e / kTopK, j = e - t * kTopK;
    const int m = tidx[t * 8 + j];
    atomicOr(&cs.mask[m * 4 + (t >> 5)], 1u << (t & 31));  // integer OR: order-free
  }
  __syncthreads();
  int cnt = 0;
  if ((int)threadIdx.x < M) {
    const uint32_t* mk = cs.mask + threadIdx.x * 4;
    cnt = __popc(mk[0]) + __popc(mk[1]) + __popc(mk[2]) + __popc(mk[3]);
  }
  const int ex = block_exclusive_scan(cnt, cs.warp_sums);
  if ((int)threadIdx.x < M) cs.off[threadIdx.x] = ex;
  if ((int)threadIdx.x == M - 1) cs.off[M] = ex + cnt;
  __syncthreads();
  for (int e = threadIdx.x; e < nt * kTopK; e += blockDim.x) {
    const int t = e / kTopK, j = e - t * kTopK;
    const int m = tidx[t * 8 + j];
    const uint32_t* mk = cs.mask + m * 4;
    const int word = t >> 5;
    int pos = cs.off[m];
    for (int w = 0; w < word; ++w) pos += __popc(mk[w]);
    pos += __popc(mk[word] & ((1u << (t & 31)) - 1u));
    cs.csr_t[pos] = (uint8_t)t;
    cs.csr_j[pos] = (uint8_t)j;
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// K0: slot tables -> fp32 round-0 state
// ---------------------------------------------------------------------------
template <typename T>
__global__ void k_load_slots(Geom g, const T* sk, Strides3 sks, const T* sv, Strides3 svs, float* K0,
                             float* V0) {
  const int bh = blockIdx.x, b = bh / g.H, h = bh - b * g.H;
  const int MD = g.M * g.D;
  float* Kd = K0 + (size_t)bh * MD;
  float* Vd = V0 + (size_t)bh * MD;
  for (int e = blockIdx.y * blockDim.x + threadIdx.x; e < MD; e += gridDim.y * blockDim.x) {
    const int m = e / g.D, c = e - m * g.D;
    Kd[e] = Elem<T>::load(row_ptr(sk, sks, b, h, m) + c);
    Vd[e] = Elem<T>::load(row_ptr(sv, svs, b, h, m) + c);
  }
}

// ---------------------------------------------------------------------------
// K1: select (top-7) + attend for one round, thread per token.
//   reference.py:19-38 scores / causal mask / topk;  reference.py:56-68 attend.
// ---------------------------------------------------------------------------
// Thread-per-token kernels whose blocks hold a (b,h)'s slot tables in shared memory (one block
// per SM) run kSimtTPB threads, so that an SM has 16 warps to hide latency with.
constexpr int kSimtTPB = 4 * kTile;

template <typename T, int D>
__global__ void __launch_bounds__(kSimtTPB) k_select_attend(Geom g, int r, const T* q, Strides3 qs, T* out,
                                                         Strides3 os, int64_t* indices, float* weights,
                                                         Saved sv) {
  extern __shared__ __align__(16) float smem[];
  float* Ks = smem;
  float* Vs = smem + g.M * D;
  const int bh = blockIdx.y, b = bh / g.H, h = bh - b * g.H;
  const size_t slot_off = ((size_t)r * g.BH + bh) * g.M * D;
  copy_to_smem(Ks, sv.K + slot_off, g.M * D);
  copy_to_smem(Vs, sv.V + slot_off, g.M * D);
  __syncthreads();

  const int n = blockIdx.x * kSimtTPB + threadIdx.x;
  if (n >= g.N) return;
  float qv[D];
  load_row<T, D>(row_ptr(q, qs, b, h, n), qv);

  Top7 top;
  top.init();
  const int visible = g.causal ? min(g.M, n + 1) : g.M;  // causal: slot m > n is -inf
  for (int m = 0; m < visible; ++m) top.offer(rank_key(dot_row<D>(qv, Ks + m * D)), m);
  for (int m = visible; m < g.M && top.k[kTopK - 1] == 0u; ++m) top.offer(kNegInfKey, m);

  // Attend recomputes the logits of the picks without any mask (reference.py:61).
  float a[kTopK], mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < kTopK; ++j) {
    a[j] = dot_row<D>(qv, Ks + top.i[j] * D) * g.scale;
    mx = fmaxf(mx, a[j]);
  }
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < kTopK; ++j) {
    a[j] = expf(a[j] - mx);
    sum += a[j];
  }
#pragma unroll
  for (int j = 0; j < kTopK; ++j) a[j] = a[j] / sum;

  T* orow = row_ptr(out, os, b, h, n);
#pragma unroll
  for (int c4 = 0; c4 < D / 4; ++c4) {
    float o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < kTopK; ++j) {
      const float4 v = reinterpret_cast<const float4*>(Vs + top.i[j] * D)[c4];
      o[0] = fmaf(a[j], v.x, o[0]);
      o[1] = fmaf(a[j], v.y, o[1]);
      o[2] = fmaf(a[j], v.z, o[2]);
      o[3] = fmaf(a[j], v.w, o[3]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float prev = r ? Elem<T>::load(orow + 4 * c4 + i) : 0.f;
      Elem<T>::store(orow + 4 * c4 + i, prev + o[i]);
    }
  }

  const size_t trow = ((size_t)r * g.BH + bh) * g.N + n;
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) lo |= (uint32_t)top.i[j] << (8 * j);
#pragma unroll
  for (int j = 4; j < kTopK; ++j) hi |= (uint32_t)top.i[j] << (8 * (j - 4));
  reinterpret_cast<uint2*>(sv.idx)[trow] = make_uint2(lo, hi);
  float4* wrow = reinterpret_cast<float4*>(sv.w + trow * 8);
  wrow[0] = make_float4(a[0], a[1], a[2], a[3]);
  wrow[1] = make_float4(a[4], a[5], a[6], 0.f);
  if (r == g.R - 1) {
    const size_t orow7 = ((size_t)bh * g.N + n) * kTopK;
    if (indices) {
#pragma unroll
      for (int j = 0; j < kTopK; ++j) indices[orow7 + j] = top.i[j];
    }
    if (weights) {
#pragma unroll
      for (int j = 0; j < kTopK; ++j) weights[orow7 + j] = a[j];
    }
  }
}

// ---------------------------------------------------------------------------
// K2: update partial sums for one round (reference.py:93-103), per token chunk.
//   Spart[bh][chunk][m][:] = sum over the chunk's picks of slot m of w * q,
//   Wpart[bh][chunk][m]    = sum of those w.
// ---------------------------------------------------------------------------
template <typename T, int D>
__global__ void __launch_bounds__(256) k_update_partial(Geom g, int r, const T* q, Strides3 qs, Saved sv,
                                                        FwdScratch f) {
  extern __shared__ __align__(16) float smem[];
  float* Sacc = smem;                      // [M][D]
  float* Wacc = Sacc + g.M * D;            // [M]
  float* qt = Wacc + g.M;                  // [kTile][D]
  float* tw = qt + kTile * D;              // [kTile][8]
  uint32_t* mask = reinterpret_cast<uint32_t*>(tw + kTile * 8);  // [M][4]
  int* off = reinterpret_cast<int*>(mask + g.M * 4);              // [M+1] (+pad)
  int* wsum = off + kMaxSlots + 4;                                // [8]
  uint8_t* tidx = reinterpret_cast<uint8_t*>(wsum + 8);           // [kTile][8]
  uint8_t* csr_t = tidx + kTile * 8;
  uint8_t* csr_j = csr_t + kTile * kTopK;
  TileCsr cs{mask, off, csr_t, csr_j, wsum};

  const int bh = blockIdx.y, b = bh / g.H, h = bh - b * g.H, chunk = blockIdx.x;
  for (int i = threadIdx.x; i < g.M * D + g.M; i += blockDim.x) Sacc[i] = 0.f;

  const int t_beg = chunk * g.red_chunk_tokens;
  const int t_end = min(g.N, t_beg + g.red_chunk_tokens);
  const int c = threadIdx.x % D, grp = threadIdx.x / D, ngrp = blockDim.x / D;
  for (int t0 = t_beg; t0 < t_end; t0 += kTile) {
    const int nt = min(kTile, t_end - t0);
    __syncthreads();
    for (int e = threadIdx.x; e < nt * D; e += blockDim.x) {
      const int t = e / D, cc = e - t * D;
      qt[e] = Elem<T>::load(row_ptr(q, qs, b, h, t0 + t) + cc);
    }
    const size_t trow = ((size_t)r * g.BH + bh) * g.N + t0;
    for (int e = threadIdx.x; e < nt * 8; e += blockDim.x) {
      tidx[e] = sv.idx[trow * 8 + e];
      tw[e] = sv.w[trow * 8 + e];
    }
    __syncthreads();
    build_tile_csr(cs, tidx, nt, g.M);
    for (int m = grp; m < g.M; m += ngrp) {
      float acc = 0.f, wacc = 0.f;
      for (int e = off[m]; e < off[m + 1]; ++e) {
        const int t = csr_t[e];
        const float w = tw[t * 8 + csr_j[e]];
        acc = __fadd_rn(acc, __fmul_rn(qt[t * D + c], w));
        wacc = __fadd_rn(wacc, w);
      }
      Sacc[m * D + c] = __fadd_rn(Sacc[m * D + c], acc);
      if (c == 0) Wacc[m] = __fadd_rn(Wacc[m], wacc);
    }
  }
  __syncthreads();
  const size_t po = (size_t)bh * g.red_chunks + chunk;
  float* Sp = f.Spart + po * g.M * D;
  for (int i = threadIdx.x; i < g.M * D; i += blockDim.x) Sp[i] = Sacc[i];
  for (int i = threadIdx.x; i < g.M; i += blockDim.x) f.Wpart[po * g.M + i] = Wacc[i];
}

// ---------------------------------------------------------------------------
// K3: combine partials, EMA (reference.py:105-113), diffusion (reference.py:128-133).
//   Writes the state entering round r+1 and the U/W records of round r.
//   grid (BH, D/8), block 256: thread m owns slot m for 8 columns.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_update_finalize(Geom g, int r, Saved sv, FwdScratch f) {
  __shared__ float kn[kMaxSlots][8];
  __shared__ float vn[kMaxSlots][8];
  const int bh = blockIdx.x, c0 = blockIdx.y * 8, m = threadIdx.x;
  const size_t MD = (size_t)g.M * g.D;
  const size_t cur = ((size_t)r * g.BH + bh) * MD;
  if (m < g.M) {
    float W = 0.f;
    for (int ch = 0; ch < g.red_chunks; ++ch) W = __fadd_rn(W, f.Wpart[((size_t)bh * g.red_chunks + ch) * g.M + m]);
    const bool hit = W > 0.f;
    const float den = __fadd_rn(W, kEmaEps);
    if (blockIdx.y == 0) sv.W[((size_t)r * g.BH + bh) * g.M + m] = W;
#pragma unroll
    for (int cc = 0; cc < 8; ++cc) {
      const int c = c0 + cc;
      float S = 0.f;
      for (int ch = 0; ch < g.red_chunks; ++ch)
        S = __fadd_rn(S, f.Spart[((size_t)bh * g.red_chunks + ch) * MD + (size_t)m * g.D + c]);
      const float U = __fdiv_rn(S, den);
      sv.U[cur + (size_t)m * g.D + c] = U;
      const float K = sv.K[cur + (size_t)m * g.D + c];
      const float V = sv.V[cur + (size_t)m * g.D + c];
      const float du = __fmul_rn(g.one_minus_alpha, U);
      kn[m][cc] = hit ? __fadd_rn(__fmul_rn(g.alpha, K), du) : K;
      vn[m][cc] = hit ? __fadd_rn(__fmul_rn(g.alpha, V), du) : V;
    }
  }
  __syncthreads();
  if (m < g.M) {
    const size_t nxt = ((size_t)(r + 1) * g.BH + bh) * MD;
    const bool inner = m > 0 && m < g.M - 1;
#pragma unroll
    for (int cc = 0; cc < 8; ++cc) {
      float k = kn[m][cc], v = vn[m][cc];
      if (inner) {
        const float tk = __fsub_rn(__fadd_rn(kn[m - 1][cc], kn[m + 1][cc]), __fmul_rn(2.f, k));
        const float tv = __fsub_rn(__fadd_rn(vn[m - 1][cc], vn[m + 1][cc]), __fmul_rn(2.f, v));
        k = __fadd_rn(k, __fmul_rn(g.gamma, tk));
        v = __fadd_rn(v, __fmul_rn(g.gamma, tv));
      }
      sv.K[nxt + (size_t)m * g.D + c0 + cc] = k;
      sv.V[nxt + (size_t)m * g.D + c0 + cc] = v;
    }
  }
}

// ---------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------

// Adjoint of the diffusion map applied to slot-gradient row m, column c.
__device__ __forceinline__ float diffuse_adj(const float* gr, int M, int D, int m, int c, float gamma) {
  const bool in_m = m > 0 && m < M - 1;
  float x = gr[(size_t)m * D + c];
  float res = in_m ? __fadd_rn(x, __fmul_rn(-2.f * gamma, x)) : x;
  if (m - 1 > 0) res = __fadd_rn(res, __fmul_rn(gamma, gr[(size_t)(m - 1) * D + c]));
  if (m + 1 < M - 1) res = __fadd_rn(res, __fmul_rn(gamma, gr[(size_t)(m + 1) * D + c]));
  return res;
}

// B1: per-slot backward of diffusion + EMA for round r (needs dL/d state_{r+1}).
//   dS = dU/(W+eps), dW = -(dU . U)/(W+eps), direct parts alpha*g (or g).
__global__ void __launch_bounds__(256) k_bwd_prep(Geom g, int r, Saved sv, const float* dKn, const float* dVn,
                                                  BwdScratch bs) {
  const int bh = blockIdx.x, m = threadIdx.x;
  if (m >= g.M) return;
  const size_t MD = (size_t)g.M * g.D;
  const float* gk = dKn + bh * MD;
  const float* gv = dVn + bh * MD;
  const float W = sv.W[((size_t)r * g.BH + bh) * g.M + m];
  const bool hit = W > 0.f;
  const float den = __fadd_rn(W, kEmaEps);
  const float* U = sv.U + ((size_t)r * g.BH + bh) * MD + (size_t)m * g.D;
  float dot = 0.f;
  for (int c = 0; c < g.D; ++c) {
    const float a = diffuse_adj(gk, g.M, g.D, m, c, g.gamma);
    const float v = diffuse_adj(gv, g.M, g.D, m, c, g.gamma);
    const float dU = hit ? __fmul_rn(g.one_minus_alpha, __fadd_rn(a, v)) : 0.f;
    const size_t e = bh * MD + (size_t)m * g.D + c;
    bs.dS[e] = __fdiv_rn(dU, den);
    dot = fmaf(dU, U[c], dot);
    bs.dKdir[e] = hit ? __fmul_rn(g.alpha, a) : a;
    bs.dVdir[e] = hit ? __fmul_rn(g.alpha, v) : v;
  }
  bs.dW[(size_t)bh * g.M + m] = -__fdiv_rn(dot, den);
}

// B2: token-side backward of attend + update for round r, thread per token.
//   dw_j  = G . V[i_j] + q . dS[i_j] + dW[i_j] (+ grad_weights in the last round)
//   da_j  = w_j (dw_j - sum_k w_k dw_k)
//   dq   += sum_j w_j dS[i_j] + scale da_j K[i_j]
//   coef_j = scale da_j   (used by the scatter kernel for dK)
template <typename T, int D>
__global__ void __launch_bounds__(kSimtTPB) k_bwd_tokens(Geom g, int r, int has_slot_grad, const T* q,
                                                      Strides3 qs, const T* go, Strides3 gos, const float* gw,
                                                      T* gq, Strides3 gqs, Saved sv, BwdScratch bs) {
  extern __shared__ __align__(16) float smem[];
  float* Ks = smem;
  float* Vs = Ks + g.M * D;
  float* dSs = Vs + g.M * D;
  float* dWs = dSs + g.M * D;
  const int bh = blockIdx.y, b = bh / g.H, h = bh - b * g.H;
  const size_t MD = (size_t)g.M * D;
  const size_t slot_off = ((size_t)r * g.BH + bh) * MD;
  copy_to_smem(Ks, sv.K + slot_off, g.M * D);
  copy_to_smem(Vs, sv.V + slot_off, g.M * D);
  if (has_slot_grad) {
    copy_to_smem(dSs, bs.dS + bh * MD, g.M * D);
    for (int i = threadIdx.x; i < g.M; i += blockDim.x) dWs[i] = bs.dW[(size_t)bh * g.M + i];
  }
  __syncthreads();
  const int n = blockIdx.x * kSimtTPB + threadIdx.x;
  if (n >= g.N) return;

  const size_t trow = ((size_t)r * g.BH + bh) * g.N + n;
  const uint2 pk = reinterpret_cast<const uint2*>(sv.idx)[trow];
  int ix[kTopK];
#pragma unroll
  for (int j = 0; j < 4; ++j) ix[j] = (pk.x >> (8 * j)) & 0xff;
#pragma unroll
  for (int j = 4; j < kTopK; ++j) ix[j] = (pk.y >> (8 * (j - 4))) & 0xff;
  float w[kTopK];
  {
    const float4* wr = reinterpret_cast<const float4*>(sv.w + trow * 8);
    const float4 w0 = wr[0], w1 = wr[1];
    w[0] = w0.x; w[1] = w0.y; w[2] = w0.z; w[3] = w0.w; w[4] = w1.x; w[5] = w1.y; w[6] = w1.z;
  }
  float dw[kTopK];
  {
    float gv_[D];
    load_row<T, D>(row_ptr(go, gos, b, h, n), gv_);
#pragma unroll
    for (int j = 0; j < kTopK; ++j) dw[j] = dot_row<D>(gv_, Vs + ix[j] * D);
  }
  if (has_slot_grad) {
    float qv[D];
    load_row<T, D>(row_ptr(q, qs, b, h, n), qv);
#pragma unroll
    for (int j = 0; j < kTopK; ++j) dw[j] += dot_row<D>(qv, dSs + ix[j] * D) + dWs[ix[j]];
  }
  if (gw && r == g.R - 1) {
    const float* gr = gw + ((size_t)bh * g.N + n) * kTopK;
#pragma unroll
    for (int j = 0; j < kTopK; ++j) dw[j] += gr[j];
  }
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < kTopK; ++j) s = fmaf(w[j], dw[j], s);
  float cf[kTopK];
#pragma unroll
  for (int j = 0; j < kTopK; ++j) cf[j] = g.scale * (w[j] * (dw[j] - s));
  float4* crow = reinterpret_cast<float4*>(bs.coef + ((size_t)bh * g.N + n) * 8);
  crow[0] = make_float4(cf[0], cf[1], cf[2], cf[3]);
  crow[1] = make_float4(cf[4], cf[5], cf[6], 0.f);

  const bool first = (r == g.R - 1);
  float* acc_row = bs.dq + ((size_t)bh * g.N + n) * D;
  T* gq_row = row_ptr(gq, gqs, b, h, n);
#pragma unroll
  for (int c4 = 0; c4 < D / 4; ++c4) {
    float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < kTopK; ++j) {
      const float4 k = reinterpret_cast<const float4*>(Ks + ix[j] * D)[c4];
      d[0] = fmaf(cf[j], k.x, d[0]);
      d[1] = fmaf(cf[j], k.y, d[1]);
      d[2] = fmaf(cf[j], k.z, d[2]);
      d[3] = fmaf(cf[j], k.w, d[3]);
      if (has_slot_grad) {
        const float4 ds = reinterpret_cast<const float4*>(dSs + ix[j] * D)[c4];
        d[0] = fmaf(w[j], ds.x, d[0]);
        d[1] = fmaf(w[j], ds.y, d[1]);
        d[2] = fmaf(w[j], ds.z, d[2]);
        d[3] = fmaf(w[j], ds.w, d[3]);
      }
    }
    if (!first) {
      const float4 p = reinterpret_cast<const float4*>(acc_row)[c4];
      d[0] += p.x; d[1] += p.y; d[2] += p.z; d[3] += p.w;
    }
    if (r == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i) Elem<T>::store(gq_row + 4 * c4 + i, d[i]);
    } else {
      reinterpret_cast<float4*>(acc_row)[c4] = make_float4(d[0], d[1], d[2], d[3]);
    }
  }
}

// B3: slot-side scatter of round r, per token chunk:
//   dKpart[m] = sum over picks of m of coef * q,  dVpart[m] = sum of w * G.
template <typename T, int D>
__global__ void __launch_bounds__(256) k_bwd_scatter(Geom g, int r, const T* q, Strides3 qs, const T* go,
                                                     Strides3 gos, Saved sv, BwdScratch bs) {
  extern __shared__ __align__(16) float smem[];
  float* Kacc = smem;                       // [M][D]
  float* Vacc = Kacc + g.M * D;             // [M][D]
  float* qt = Vacc + g.M * D;               // [kTile][D]
  float* gt = qt + kTile * D;               // [kTile][D]
  float* tw = gt + kTile * D;               // [kTile][8]
  float* tc = tw + kTile * 8;               // [kTile][8]
  uint32_t* mask = reinterpret_cast<uint32_t*>(tc + kTile * 8);
  int* off = reinterpret_cast<int*>(mask + g.M * 4);
  int* wsum = off + kMaxSlots + 4;
  uint8_t* tidx = reinterpret_cast<uint8_t*>(wsum + 8);
  uint8_t* csr_t = tidx + kTile * 8;
  uint8_t* csr_j = csr_t + kTile * kTopK;
  TileCsr cs{mask, off, csr_t, csr_j, wsum};

  const int bh = blockIdx.y, b = bh / g.H, h = bh - b * g.H, chunk = blockIdx.x;
  for (int i = threadIdx.x; i < 2 * g.M * D; i += blockDim.x) Kacc[i] = 0.f;
  const int t_beg = chunk * g.red_chunk_tokens;
  const int t_end = min(g.N, t_beg + g.red_chunk_tokens);
  const int c = threadIdx.x % D, grp = threadIdx.x / D, ngrp = blockDim.x / D;
  for (int t0 = t_beg; t0 < t_end; t0 += kTile) {
    const int nt = min(kTile, t_end - t0);
    __syncthreads();
    for (int e = threadIdx.x; e < nt * D; e += blockDim.x) {
      const int t = e / D, cc = e - t * D;
      qt[e] = Elem<T>::load(row_ptr(q, qs, b, h, t0 + t) + cc);
      gt[e] = Elem<T>::load(row_ptr(go, gos, b, h, t0 + t) + cc);
    }
    const size_t trow = ((size_t)r * g.BH + bh) * g.N + t0;
    const size_t crow = (size_t)bh * g.N + t0;
    for (int e = threadIdx.x; e < nt * 8; e += blockDim.x) {
      tidx[e] = sv.idx[trow * 8 + e];
      tw[e] = sv.w[trow * 8 + e];
      tc[e] = bs.coef[crow * 8 + e];
    }
    __syncthreads();
    build_tile_csr(cs, tidx, nt, g.M);
    for (int m = grp; m < g.M; m += ngrp) {
      float ak = 0.f, av = 0.f;
      for (int e = off[m]; e < off[m + 1]; ++e) {
        const int t = csr_t[e], j = csr_j[e];
        ak = fmaf(tc[t * 8 + j], qt[t * D + c], ak);
        av = fmaf(tw[t * 8 + j], gt[t * D + c], av);
      }
      Kacc[m * D + c] += ak;
      Vacc[m * D + c] += av;
    }
  }
  __syncthreads();
  const size_t po = ((size_t)bh * g.red_chunks + chunk) * g.M * D;
  for (int i = threadIdx.x; i < g.M * D; i += blockDim.x) {
    bs.dKpart[po + i] = Kacc[i];
    bs.dVpart[po + i] = Vacc[i];
  }
}

// B4: dK_r = direct part + sum of chunk partials; written as fp32 state
// gradient (r > 0) or as the slot gradients in the caller's dtype (r == 0).
template <typename T>
__global__ void __launch_bounds__(256) k_bwd_finalize(Geom g, int r, BwdScratch bs, int has_dir, float* dKout,
                                                      float* dVout, T* gsk, Strides3 gsks, T* gsv,
                                                      Strides3 gsvs) {
  const int bh = blockIdx.x, b = bh / g.H, h = bh - b * g.H;
  const size_t MD = (size_t)g.M * g.D;
  for (int e = blockIdx.y * blockDim.x + threadIdx.x; e < (int)MD; e += gridDim.y * blockDim.x) {
    float k = has_dir ? bs.dKdir[bh * MD + e] : 0.f;
    float v = has_dir ? bs.dVdir[bh * MD + e] : 0.f;
    for (int ch = 0; ch < g.red_chunks; ++ch) {
      const size_t po = ((size_t)bh * g.red_chunks + ch) * MD + e;
      k += bs.dKpart[po];
      v += bs.dVpart[po];
    }
    if (r == 0) {
      const int m = e / g.D, c = e - m * g.D;
      Elem<T>::store(row_ptr(gsk, gsks, b, h, m) + c, k);
      Elem<T>::store(row_ptr(gsv, gsvs, b, h, m) + c, v);
    } else {
      dKout[bh * MD + e] = k;
      dVout[bh * MD + e] = v;
    }
  }
}

template <typename T>
__global__ void k_fill_zero_rows(Geom g, T* p, Strides3 st, int rows) {
  const int bh = blockIdx.x, b = bh / g.H, h = bh - b * g.H;
  for (int e = threadIdx.x; e < rows * g.D; e += blockDim.x) {
    const int n = e / g.D, c = e - n * g.D;
    Elem<T>::store(row_ptr(p, st, b, h, n) + c, 0.f);
  }
}

// ---------------------------------------------------------------------------
// Host-side launchers (called from murm_capi.cu)
// ---------------------------------------------------------------------------
template <typename T>
void launch_load_slots(const Geom& g, const FwdPtrs& p, const Saved& sv, cudaStream_t st) {
  MURM_LAUNCH("load_slots", k_load_slots<T>, dim3(g.BH, 4), 256, 0, st, g, static_cast<const T*>(p.sk), p.sks,
              static_cast<const T*>(p.sv), p.svs, sv.K, sv.V);
}
template void launch_load_slots<float>(const Geom&, const FwdPtrs&, const Saved&, cudaStream_t);
template void launch_load_slots<__half>(const Geom&, const FwdPtrs&, const Saved&, cudaStream_t);
template void launch_load_slots<__nv_bfloat16>(const Geom&, const FwdPtrs&, const Saved&, cudaStream_t);

void launch_update_finalize(const Geom& g, int r, const Saved& sv, const FwdScratch& fs, cudaStream_t st) {
  MURM_LAUNCH("update_finalize", k_update_finalize, dim3(g.BH, g.D / 8), 256, 0, st, g, r, sv, fs);
}

template <typename T, int D>
static cudaError_t run_fwd_simt(const Geom& g, const FwdPtrs& p, const Saved& sv, const FwdScratch& fs,
                                cudaStream_t st) {
  const int smem_sa = 2 * g.M * D * (int)sizeof(float);
  const int smem_up = (g.M * D + g.M + kTile * D + kTile * 8) * 4 + g.M * 16 + (kMaxSlots + 4 + 8) * 4 +
                      kTile * 8 + 2 * kTile * kTopK;
  if (cudaError_t e = smem_opt_in(k_select_attend<T, D>, smem_sa)) return e;
  if (cudaError_t e = smem_opt_in(k_update_partial<T, D>, smem_up)) return e;
  const T* q = static_cast<const T*>(p.q);
  if (g.R > 0 && p.slots_f32)  // with zero rounds the saved block is empty and nothing reads the slots
    MURM_LAUNCH("load_slots", k_load_slots<float>, dim3(g.BH, 4), 256, 0, st, g, static_cast<const float*>(p.sk),
                p.sks, static_cast<const float*>(p.sv), p.svs, sv.K, sv.V);
  else if (g.R > 0)
    MURM_LAUNCH("load_slots", k_load_slots<T>, dim3(g.BH, 4), 256, 0, st, g, static_cast<const T*>(p.sk), p.sks,
                static_cast<const T*>(p.sv), p.svs, sv.K, sv.V);
  for (int r = 0; r < g.R; ++r) {
    MURM_LAUNCH("select_attend_simt", (k_select_attend<T, D>), dim3((g.N + kSimtTPB - 1) / kSimtTPB, g.BH), kSimtTPB,
                smem_sa, st, 
        g, r, q, p.qs, static_cast<T*>(p.out), p.os, p.indices, p.weights, sv);
    if (r + 1 < g.R) {
      MURM_LAUNCH("update_partial", (k_update_partial<T, D>), dim3(g.red_chunks, g.BH), 256, smem_up, st, g, r, q, p.qs, sv, fs);
      MURM_LAUNCH("update_finalize", k_update_finalize, dim3(g.BH, g.D / 8), 256, 0, st, g, r, sv, fs);
    }
  }
  if (g.R == 0) {
    MURM_LAUNCH("fill_zero", k_fill_zero_rows<T>, g.BH, 256, 0, st, g, static_cast<T*>(p.out), p.os, g.N);
    const size_t n7 = (size_t)g.BH * g.N * kTopK;
    if (p.indices) cudaMemsetAsync(p.indices, 0, n7 * sizeof(int64_t), st);
    if (p.weights) cudaMemsetAsync(p.weights, 0, n7 * sizeof(float), st);
  }
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t run_bwd_simt(const Geom& g, const BwdPtrs& p, const Saved& sv, const BwdScratch& bs,
                                cudaStream_t st) {
  const int smem_tok = (3 * g.M * D + g.M) * (int)sizeof(float);
  const int smem_sc = (2 * g.M * D + 2 * kTile * D + 2 * kTile * 8) * 4 + g.M * 16 + (kMaxSlots + 4 + 8) * 4 +
                      kTile * 8 + 2 * kTile * kTopK;
  if (cudaError_t e = smem_opt_in(k_bwd_tokens<T, D>, smem_tok)) return e;
  if (cudaError_t e = smem_opt_in(k_bwd_scatter<T, D>, smem_sc)) return e;
  const T* q = static_cast<const T*>(p.q);
  const T* go = static_cast<const T*>(p.go);
  if (g.R == 0) {
    MURM_LAUNCH("fill_zero", k_fill_zero_rows<T>, g.BH, 256, 0, st, g, static_cast<T*>(p.gq), p.gqs, g.N);
    MURM_LAUNCH("fill_zero", k_fill_zero_rows<T>, g.BH, 256, 0, st, g, static_cast<T*>(p.gsk), p.gsks, g.M);
    MURM_LAUNCH("fill_zero", k_fill_zero_rows<T>, g.BH, 256, 0, st, g, static_cast<T*>(p.gsv), p.gsvs, g.M);
    return cudaGetLastError();
  }
  int cur = 0;
  const int fin_y = (g.M * D + 255) / 256;
  for (int r = g.R - 1; r >= 0; --r) {
    const int has_slot_grad = r < g.R - 1;
    if (has_slot_grad) MURM_LAUNCH("bwd_prep", k_bwd_prep, g.BH, 256, 0, st, g, r, sv, bs.dK[cur], bs.dV[cur], bs);
    MURM_LAUNCH("bwd_tokens", (k_bwd_tokens<T, D>), dim3((g.N + kSimtTPB - 1) / kSimtTPB, g.BH), kSimtTPB,
                smem_tok, st, 
        g, r, has_slot_grad, q, p.qs, go, p.gos, p.gw, static_cast<T*>(p.gq), p.gqs, sv, bs);
    MURM_LAUNCH("bwd_scatter", (k_bwd_scatter<T, D>), dim3(g.red_chunks, g.BH), 256, smem_sc, st, g, r, q, p.qs, go, p.gos, sv, bs);
    MURM_LAUNCH("bwd_finalize", k_bwd_finalize<T>, dim3(g.BH, fin_y), 256, 0, st, g, r, bs, has_slot_grad, bs.dK[cur ^ 1],
                                                           bs.dV[cur ^ 1], static_cast<T*>(p.gsk), p.gsks,
                                                           static_cast<T*>(p.gsv), p.gsvs);
    cur ^= 1;
  }
  return cudaGetLastError();
}

template <typename T>
cudaError_t fwd_simt(const Geom& g, const FwdPtrs& p, const Saved& sv, const FwdScratch& fs, cudaStream_t st) {
  switch (g.D) {
    case 16: return run_fwd_simt<T, 16>(g, p, sv, fs, st);
    case 32: return run_fwd_simt<T, 32>(g, p, sv, fs, st);
    case 64: return run_fwd_simt<T, 64>(g, p, sv, fs, st);
  }
  return cudaErrorInvalidValue;
}
template <typename T>
cudaError_t bwd_simt(const Geom& g, const BwdPtrs& p, const Saved& sv, const BwdScratch& bs, cudaStream_t st) {
  switch (g.D) {
    case 16: return run_bwd_simt<T, 16>(g, p, sv, bs, st);
    case 32: return run_bwd_simt<T, 32>(g, p, sv, bs, st);
    case 64: return run_bwd_simt<T, 64>(g, p, sv, bs, st);
  }
  return cudaErrorInvalidValue;
}

template cudaError_t fwd_simt<float>(const Geom&, const FwdPtrs&, const Saved&, const FwdScratch&, cudaStream_t);
template cudaError_t fwd_simt<__half>(const Geom&, const FwdPtrs&, const Saved&, const FwdScratch&, cudaStream_t);
template cudaError_t fwd_simt<__nv_bfloat16>(const Geom&, const FwdPtrs&, const Saved&, const FwdScratch&,
                                             cudaStream_t);
template cudaError_t bwd_simt<float>(const Geom&, const BwdPtrs&, const Saved&, const BwdScratch&, cudaStream_t);
template cudaError_t bwd_simt<__half>(const Geom&, const BwdPtrs&, const Saved&, const BwdScratch&, cudaStream_t);
template cudaError_t bwd_simt<__nv_bfloat16>(const Geom&, const BwdPtrs&, const Saved&, const BwdScratch&,
                                             cudaStream_t);

}  // namespace murm
