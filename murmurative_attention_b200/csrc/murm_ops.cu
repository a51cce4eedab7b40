// murm_ops.cu — per-phase operations of the reference's op surface (include/murm.h,
// "Per-phase operations"): select+attend with mask / position bias / effective M,
// slot update with separate token keys and values, slot diffusion, each with its
// backward. General CUDA-core kernels (any head_dim that is a multiple of 8 up to
// 128, M up to 1024); the fused round loop (murm_tc.cu, murm_simt.cu) remains the
// fast path for the north-star operation.
//
// Semantics: reference.py:6-39 (select), 42-68 (attend), 71-115 (update),
// 118-135 (diffusion). Slot sums are deterministic: the (token, pick) pairs are
// sorted by slot with a stable counting sort (k_csr), then each slot sums its pairs
// in token order; no floating-point atomics.
#include <cmath>
#include <cstdarg>
#include <cstdio>

#include "murm_kernels.cuh"

namespace murm {
namespace ph {

constexpr int kMaxD = 128;
constexpr int kMaxM = 1024;
constexpr size_t kMaxStage = 200 * 1024;   // transposed fp32 key table per block
constexpr int kTokPerWarp = 8;             // select+attend: tokens per warp
constexpr int kWarps = 8;

struct Dims {
  int B, H, N, M, D;
};

__device__ __forceinline__ int clampi(int64_t v, int M) { return (int)(v < 0 ? 0 : (v >= M ? M - 1 : v)); }

// Insert into a 7-entry list kept in rank order; offers must come in ascending slot
// order (then equal keys never displace an earlier slot).
__device__ __forceinline__ void offer7(uint32_t (&k)[kTopK], int (&s)[kTopK], uint32_t xk, int xs) {
  bool gt[kTopK];
#pragma unroll
  for (int j = 0; j < kTopK; ++j) gt[j] = xk > k[j];
#pragma unroll
  for (int j = kTopK - 1; j >= 1; --j) {
    k[j] = gt[j - 1] ? k[j - 1] : (gt[j] ? xk : k[j]);
    s[j] = gt[j - 1] ? s[j - 1] : (gt[j] ? xs : s[j]);
  }
  k[0] = gt[0] ? xk : k[0];
  s[0] = gt[0] ? xs : s[0];
}

// The warp's best 7 of all lanes' lists (each in rank order), in 7 rounds: the largest head
// key over the lanes (one reduction), the lowest slot among the heads with that key (another),
// and the lane holding that entry moves its list up. Every lane returns the same list.
__device__ __forceinline__ void warp_top7(uint32_t (&k)[kTopK], int (&s)[kTopK]) {
  uint32_t ok[kTopK];
  int os[kTopK];
#pragma unroll
  for (int r = 0; r < kTopK; ++r) {
    const uint32_t best = __reduce_max_sync(0xffffffffu, k[0]);
    const uint32_t slot = __reduce_min_sync(0xffffffffu, k[0] == best ? (uint32_t)s[0] : 0xffffffffu);
    ok[r] = best;
    os[r] = (int)slot;
    if (k[0] == best && (uint32_t)s[0] == slot) {
#pragma unroll
      for (int j = 0; j < kTopK - 1; ++j) {
        k[j] = k[j + 1];
        s[j] = s[j + 1];
      }
      k[kTopK - 1] = 0u;
      s[kTopK - 1] = 0;
    }
  }
#pragma unroll
  for (int j = 0; j < kTopK; ++j) {
    k[j] = ok[j];
    s[j] = os[j];
  }
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

template <typename T>
__device__ __forceinline__ float ld(const void* base, int64_t i) {
  return Elem<T>::load(static_cast<const T*>(base) + i);
}
template <typename T>
__device__ __forceinline__ void st(void* base, int64_t i, float v) {
  Elem<T>::store(static_cast<T*>(base) + i, v);
}
__device__ __forceinline__ int64_t off3(const int64_t* s, int b, int h, int r) {
  return (int64_t)b * s[0] + (int64_t)h * s[1] + (int64_t)r * s[2];
}
__device__ __forceinline__ int64_t off4(const int64_t* s, int b, int h, int n, int m) {
  return (int64_t)b * s[0] + (int64_t)h * s[1] + (int64_t)n * s[2] + (int64_t)m * s[3];
}

// ---------------------------------------------------------------------------
// select + attend, forward. grid (ceil(N / 64), B*H), 8 warps, a warp per token.
// Shared memory: the (b,h) key table transposed to [d][Mp] fp32 (lanes read
// consecutive slots), and each warp's q row.
// ---------------------------------------------------------------------------
// The (b,h) key table into shared memory, transposed to [D][Mp] fp32.
template <typename T>
__device__ __forceinline__ void stage_keys(const murm_select_attend_args& a, float* Kt, int Mp, int vec, int b, int h) {
  const int M = a.shape.slots, D = a.shape.head_dim;
  if (vec) {  // 16-byte loads (rows 16-byte aligned), several in flight per thread
    constexpr int E = 16 / (int)sizeof(T);
    const int C = D / E;
#pragma unroll 4
    for (int e = threadIdx.x; e < M * C; e += blockDim.x) {
      const int m = e / C, c = e - m * C;
      const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const T*>(a.slot_keys) +
                                                      off3(a.sk_stride, b, h, m) + c * E);
      const T* t = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int i = 0; i < E; ++i) Kt[(size_t)(c * E + i) * Mp + m] = Elem<T>::load(t + i);
    }
  } else {
    for (int e = threadIdx.x; e < M * D; e += blockDim.x) {
      const int m = e / D, d = e - m * D;
      Kt[(size_t)d * Mp + m] = ld<T>(a.slot_keys, off3(a.sk_stride, b, h, m) + d);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(32 * kWarps) k_sa_fwd(murm_select_attend_args a, int Mp, int vec) {
  extern __shared__ float sh[];
  const int M = a.shape.slots, D = a.shape.head_dim, N = a.shape.tokens;
  float* Kt = sh;                       // [D][Mp]
  float* qs = sh + (size_t)D * Mp;      // [kWarps][D]
  const int bh = blockIdx.y, b = bh / a.shape.heads, h = bh - b * a.shape.heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  stage_keys<T>(a, Kt, Mp, vec, b, h);
  __syncthreads();
  const int em = (a.effective_m > 0 && a.effective_m < M) ? a.effective_m : M;
  const float scale = a.scale > 0 ? (float)a.scale : rsqrtf((float)D);
  float* q = qs + warp * D;
  for (int tt = 0; tt < kTokPerWarp; ++tt) {
    const int n = (blockIdx.x * kWarps + warp) * kTokPerWarp + tt;
    if (n >= N) break;
    for (int d = lane; d < D; d += 32) q[d] = ld<T>(a.q, off3(a.q_stride, b, h, n) + d);
    __syncwarp();
    const int64_t rec = ((int64_t)bh * N + n) * kTopK;
    int pick[kTopK];
    if (a.indices_in) {
#pragma unroll
      for (int j = 0; j < kTopK; ++j) pick[j] = clampi(a.indices_in[rec + j], M);
    } else {
      uint32_t tk[kTopK];
      int ts[kTopK];
#pragma unroll
      for (int j = 0; j < kTopK; ++j) { tk[j] = 0u; ts[j] = 0; }
      // 8 slots per lane at a time (m = m0 + lane + 32 j): independent dot products over the
      // same q[d] (each in d order), offered in slot order
      for (int m0 = 0; m0 < M; m0 += 256) {
        float sj[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) sj[j] = 0.f;
        const int mc = min(M - 1, m0 + lane);  // clamped columns: reads stay inside Kt
        for (int d = 0; d < D; ++d) {
          const float qd = q[d];
          const float* row = Kt + (size_t)d * Mp;
#pragma unroll
          for (int j = 0; j < 8; ++j) sj[j] = fmaf(qd, row[min(M - 1, mc + 32 * j)], sj[j]);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int m = m0 + lane + 32 * j;
          if (m < M) {
            float s = sj[j];
            if (a.position_bias) s += ld<T>(a.position_bias, off4(a.bias_stride, b, h, n, m));     // reference.py:21-22
            bool masked = m >= em || (a.causal && m > n);                                            // :27-36
            if (a.mask) masked = masked || a.mask[off4(a.mask_stride, b, h, n, m)] == 0;               // :24-25
            offer7(tk, ts, rank_key(masked ? -INFINITY : s), m);
          }
        }
      }
      warp_top7(tk, ts);
#pragma unroll
      for (int j = 0; j < kTopK; ++j) pick[j] = ts[j];
    }
    // attend over the picks with the plain scaled scores (reference.py:58-66)
    float sc[kTopK], mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < kTopK; ++j) {
      float p = 0.f;
      for (int d = lane; d < D; d += 32) p = fmaf(q[d], Kt[(size_t)d * Mp + pick[j]], p);
      sc[j] = warp_sum(p) * scale;
      mx = fmaxf(mx, sc[j]);
    }
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < kTopK; ++j) {
      sc[j] = expf(sc[j] - mx);
      sum += sc[j];
    }
#pragma unroll
    for (int j = 0; j < kTopK; ++j) sc[j] = sc[j] / sum;
    for (int d = lane; d < D; d += 32) {
      float o = 0.f;
#pragma unroll
      for (int j = 0; j < kTopK; ++j) o = fmaf(sc[j], ld<T>(a.slot_values, off3(a.sv_stride, b, h, pick[j]) + d), o);
      st<T>(a.out, off3(a.out_stride, b, h, n) + d, o);
    }
    if (lane < kTopK) {
      int pj = pick[0];
      float wj = sc[0];
#pragma unroll
      for (int j = 1; j < kTopK; ++j)
        if (lane == j) { pj = pick[j]; wj = sc[j]; }
      a.indices[rec + lane] = pj;
      a.weights[rec + lane] = wj;
    }
    __syncwarp();
  }
}

// x[j] for a run-time j in [0, 8) over 8 values held in registers (select tree).
__device__ __forceinline__ uint32_t pick8(const uint32_t (&x)[8], int j) {
  const uint32_t a0 = (j & 1) ? x[1] : x[0], a1 = (j & 1) ? x[3] : x[2];
  const uint32_t a2 = (j & 1) ? x[5] : x[4], a3 = (j & 1) ? x[7] : x[6];
  const uint32_t b0 = (j & 2) ? a1 : a0, b1 = (j & 2) ? a3 : a2;
  return (j & 4) ? b1 : b0;
}

// ---------------------------------------------------------------------------
// select + attend, forward, M <= 256 and selection on the GPU: the picks of k_sa_fwd (the same
// scores, in the same operation order; ties to the lowest slot) with the key table read once
// per four tokens. Shared memory: the transposed key table [D][kMp4] (columns M..255 zero), each
// warp's four q rows [D][4], and per warp a candidate list and the picks.
//   - scores: a warp takes four tokens at a time, a lane slots lane + 32 j (8 x 4 independent
//     dot products in d order over the key rows it loads once);
//   - candidates: thr = the 7th largest of the 32 lanes' maximum keys, ties counted; at least 7
//     of the row's keys are >= thr, so its top 7 are among the keys >= thr (typically 7-10);
//   - ranking: the candidates are packed into a per-warp list and each one's rank in the order
//     (key descending, slot ascending) is counted over the list; more than 32 candidates (ties,
//     rows with most slots masked) take the lane-list merge of k_sa_fwd instead;
//   - attend: the picks' plain scores (without bias or mask), scaled, softmax, weighted values.
// ---------------------------------------------------------------------------
constexpr int kTokGroup = 4;
constexpr int kMp4 = 257;  // key-table row stride of k_sa_fwd4 (odd: lanes read distinct banks)
template <typename T>
__global__ void __launch_bounds__(32 * kWarps, 3) k_sa_fwd4(murm_select_attend_args a, int vec) {
  extern __shared__ float sh[];
  const int M = a.shape.slots, D = a.shape.head_dim, N = a.shape.tokens;
  float* Kt = sh;                                                                  // [D][kMp4]
  float4* qs = reinterpret_cast<float4*>(sh + (((size_t)D * kMp4 + 3) & ~(size_t)3));  // [kWarps][D]
  uint2* cand = reinterpret_cast<uint2*>(qs + kWarps * D);                         // [kWarps][32]
  uint2* picks = cand + kWarps * 32;                                               // [kWarps][8]
  const int bh = blockIdx.y, b = bh / a.shape.heads, h = bh - b * a.shape.heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (M < 256)
    for (int e = threadIdx.x; e < D * 256; e += blockDim.x)
      if (e % 256 >= M) Kt[(size_t)(e / 256) * kMp4 + e % 256] = 0.f;
  stage_keys<T>(a, Kt, kMp4, vec, b, h);
  __syncthreads();
  const int em = (a.effective_m > 0 && a.effective_m < M) ? a.effective_m : M;
  const float scale = a.scale > 0 ? (float)a.scale : rsqrtf((float)D);
  float4* q4 = qs + warp * D;
  uint2* cw = cand + warp * 32;
  uint2* pw = picks + warp * 8;
  const T* sv = static_cast<const T*>(a.slot_values) + (int64_t)b * a.sv_stride[0] + (int64_t)h * a.sv_stride[1];
  for (int g0 = 0; g0 < kTokPerWarp; g0 += kTokGroup) {
    const int nb = (blockIdx.x * kWarps + warp) * kTokPerWarp + g0;
    if (nb >= N) break;
    for (int d = lane; d < D; d += 32) {
      float v[kTokGroup];
#pragma unroll
      for (int t = 0; t < kTokGroup; ++t) v[t] = nb + t < N ? ld<T>(a.q, off3(a.q_stride, b, h, nb + t) + d) : 0.f;
      q4[d] = make_float4(v[0], v[1], v[2], v[3]);
    }
    __syncwarp();
    float sj[kTokGroup][8];
#pragma unroll
    for (int t = 0; t < kTokGroup; ++t)
#pragma unroll
      for (int j = 0; j < 8; ++j) sj[t][j] = 0.f;
    const float* kp = Kt + lane;
#pragma unroll 2
    for (int d = 0; d < D; ++d) {  // each score in d order, as k_sa_fwd
      const float4 qd = q4[d];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float kv = kp[32 * j];
        sj[0][j] = fmaf(qd.x, kv, sj[0][j]);
        sj[1][j] = fmaf(qd.y, kv, sj[1][j]);
        sj[2][j] = fmaf(qd.z, kv, sj[2][j]);
        sj[3][j] = fmaf(qd.w, kv, sj[3][j]);
      }
      kp += kMp4;
    }
#pragma unroll 1
    for (int t = 0; t < kTokGroup; ++t) {
      const int n = nb + t;
      if (n >= N) break;
      // this lane's rank keys (0: no slot); bias and mask rows walked 32 slots at a time
      const T* bp = a.position_bias ? static_cast<const T*>(a.position_bias) + off4(a.bias_stride, b, h, n, lane)
                                    : nullptr;
      const uint8_t* mp = a.mask ? a.mask + off4(a.mask_stride, b, h, n, lane) : nullptr;
      const int64_t bstep = 32 * a.bias_stride[3], mstep = 32 * a.mask_stride[3];
      uint32_t kk[8];
      uint32_t lm = 0u;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int m = lane + 32 * j;
        kk[j] = 0u;
        if (m < M) {
          float sc = sj[0][j];
          if (bp) sc += Elem<T>::load(bp + j * bstep);                      // reference.py:21-22
          bool masked = m >= em || (a.causal && m > n);                      // :27-36
          if (mp) masked = masked || mp[j * mstep] == 0;                     // :24-25
          kk[j] = rank_key(masked ? -INFINITY : sc);
        }
        lm = max(lm, kk[j]);
      }
      uint32_t thr = 0u, v = lm;
      int cnt = 0;
#pragma unroll 1
      for (int r = 0; r < kTopK && cnt < kTopK; ++r) {
        const uint32_t best = __reduce_max_sync(0xffffffffu, v);
        thr = best;
        cnt += __popc(__ballot_sync(0xffffffffu, v == best));
        v = v == best ? 0u : v;
      }
      uint32_t cm = 0u;  // this lane's candidates
#pragma unroll
      for (int j = 0; j < 8; ++j) cm |= (kk[j] != 0u && kk[j] >= thr ? 1u : 0u) << j;
      const int c = __popc(cm);
      int pre = c;  // inclusive prefix over the lanes
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, pre, o);
        if (lane >= o) pre += y;
      }
      const int total = __shfl_sync(0xffffffffu, pre, 31);
      int ps[kTopK];
      if (total <= 32) {  // warp-uniform
        int p = pre - c;
        for (uint32_t mm = cm; mm; mm &= mm - 1) {
          const int j = __ffs(mm) - 1;
          cw[p++] = make_uint2(pick8(kk, j), (uint32_t)(lane + 32 * j));
        }
        __syncwarp();
        if (lane < total) {
          const uint2 me = cw[lane];
          int rank = 0;
          for (int i = 0; i < total; ++i) {
            const uint2 o = cw[i];
            rank += (o.x > me.x || (o.x == me.x && o.y < me.y)) ? 1 : 0;
          }
          if (rank < kTopK) pw[rank] = me;
        }
        __syncwarp();
#pragma unroll
        for (int j = 0; j < kTopK; ++j) ps[j] = (int)pw[j].y;
        __syncwarp();  // the lists are reused by the next token
      } else {
        uint32_t tk[kTopK];
#pragma unroll
        for (int j = 0; j < kTopK; ++j) { tk[j] = 0u; ps[j] = 0; }
        for (uint32_t mm = cm; mm; mm &= mm - 1) {  // ascending slot order within the lane
          const int j = __ffs(mm) - 1;
          offer7(tk, ps, pick8(kk, j), lane + 32 * j);
        }
        warp_top7(tk, ps);
      }
      // attend over the picks with their plain scaled scores (reference.py:58-66): the score of
      // slot s is lane s % 32's sj[s / 32]
      float sc[kTopK], mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < kTopK; ++j) {
        const int q = ps[j] >> 5;
        const float a0 = (q & 1) ? sj[0][1] : sj[0][0], a1 = (q & 1) ? sj[0][3] : sj[0][2];
        const float a2 = (q & 1) ? sj[0][5] : sj[0][4], a3 = (q & 1) ? sj[0][7] : sj[0][6];
        const float b0 = (q & 2) ? a1 : a0, b1 = (q & 2) ? a3 : a2;
        sc[j] = __shfl_sync(0xffffffffu, (q & 4) ? b1 : b0, ps[j] & 31) * scale;
        mx = fmaxf(mx, sc[j]);
      }
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < kTopK; ++j) {
        sc[j] = expf(sc[j] - mx);
        sum += sc[j];
      }
#pragma unroll
      for (int j = 0; j < kTopK; ++j) sc[j] = sc[j] / sum;
      for (int d = lane; d < D; d += 32) {
        float o = 0.f;
#pragma unroll
        for (int j = 0; j < kTopK; ++j) o = fmaf(sc[j], Elem<T>::load(sv + (int64_t)ps[j] * a.sv_stride[2] + d), o);
        st<T>(a.out, off3(a.out_stride, b, h, n) + d, o);
      }
      const int64_t rec = ((int64_t)bh * N + n) * kTopK;
      if (lane < kTopK) {
        int pj = ps[0];
        float wj = sc[0];
#pragma unroll
        for (int j = 1; j < kTopK; ++j)
          if (lane == j) { pj = ps[j]; wj = sc[j]; }
        a.indices[rec + lane] = pj;
        a.weights[rec + lane] = wj;
      }
      // the next token's scores to the front
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        sj[0][j] = sj[1][j];
        sj[1][j] = sj[2][j];
        sj[2][j] = sj[3][j];
      }
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// Stable counting sort of the (token, pick) pairs of every (b,h) by slot:
// offsets [BH][M+1], entries [BH][N*7] = token*8 + pick, ordered by slot, then
// token, then pick. Parallel over token tiles: (1) each tile marks its pairs in a
// per-slot bitmap and counts them per slot, (2) per slot, an exclusive scan over
// the tiles gives each tile's base (and the slot offsets), (3) each tile places its
// pairs at offset + base + the number of earlier pairs of the tile in that slot.
// Integer work only: the order, and so every sum taken over it, is deterministic.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tile_bitmap(const int64_t* ix, int N, int M, int tile, int words, int base,
                                            uint32_t* bm, int (&mm)[kTopK], bool& live) {
  const int tid = threadIdx.x;
  for (int e = tid; e < M * words; e += blockDim.x) bm[e] = 0u;
  __syncthreads();
  const int t = base + tid;
  live = tid < tile && t < N;
  if (live) {
#pragma unroll
    for (int j = 0; j < kTopK; ++j) {
      mm[j] = clampi(ix[(int64_t)t * kTopK + j], M);
      const int p = tid * kTopK + j;
      atomicOr(&bm[mm[j] * words + (p >> 5)], 1u << (p & 31));
    }
  }
  __syncthreads();
}

// (1) grid (ntiles, BH): per-tile, per-slot pair counts -> cnt [BH][ntiles][M] (shared-memory
// counters: the counts alone need no order)
__global__ void __launch_bounds__(256) k_csr_count(const int64_t* idx, int N, int M, int tile, int* cnt) {
  extern __shared__ uint32_t smu[];  // [M] counters
  const int bh = blockIdx.y, ti = blockIdx.x;
  for (int m = threadIdx.x; m < M; m += blockDim.x) smu[m] = 0u;
  __syncthreads();
  const int t = ti * tile + threadIdx.x;
  if (threadIdx.x < tile && t < N) {
    const int64_t* ix = idx + ((int64_t)bh * N + t) * kTopK;
#pragma unroll
    for (int j = 0; j < kTopK; ++j) atomicAdd(&smu[clampi(ix[j], M)], 1u);
  }
  __syncthreads();
  int* c = cnt + ((int64_t)bh * gridDim.x + ti) * M;
  for (int m = threadIdx.x; m < M; m += blockDim.x) c[m] = (int)smu[m];
}

// (2) grid BH: per slot, tile bases (in place) and the slot offsets
__global__ void __launch_bounds__(256) k_csr_scan(int ntiles, int M, int* cnt, int* offsets) {
  __shared__ int tot[1024];
  const int bh = blockIdx.x;
  int* c = cnt + (int64_t)bh * ntiles * M;
  for (int m = threadIdx.x; m < M; m += blockDim.x) {
    int run = 0;
    for (int t0 = 0; t0 < ntiles; t0 += 8) {  // eight tiles' counts loaded at once
      int x[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = t0 + i < ntiles ? c[(int64_t)(t0 + i) * M + m] : 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (t0 + i < ntiles) c[(int64_t)(t0 + i) * M + m] = run;
        run += x[i];
      }
    }
    tot[m] = run;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int* off = offsets + (int64_t)bh * (M + 1);
    int acc = 0;
    for (int m = 0; m < M; ++m) {
      off[m] = acc;
      acc += tot[m];
    }
    off[M] = acc;
  }
}

// (3) grid (ntiles, BH): place the tile's pairs
__global__ void __launch_bounds__(256) k_csr_fill(const int64_t* idx, int N, int M, int tile, int words,
                                                  const int* cnt, const int* offsets, int* entries) {
  extern __shared__ uint32_t smu[];  // [M][words] bitmap, then [M][words] uint16 prefix counts
  uint16_t* pre = reinterpret_cast<uint16_t*>(smu + M * words);
  const int bh = blockIdx.y, ti = blockIdx.x;
  int mm[kTopK];
  bool live;
  tile_bitmap(idx + (int64_t)bh * N * kTopK, N, M, tile, words, ti * tile, smu, mm, live);
  for (int m = threadIdx.x; m < M; m += blockDim.x) {  // pairs of the slot in the row's earlier words
    int acc = 0;
    for (int w = 0; w < words; ++w) {
      pre[m * words + w] = (uint16_t)acc;
      acc += __popc(smu[m * words + w]);
    }
  }
  __syncthreads();
  if (!live) return;
  const int* c = cnt + ((int64_t)bh * gridDim.x + ti) * M;
  const int* off = offsets + (int64_t)bh * (M + 1);
  int* ent = entries + (int64_t)bh * N * kTopK;
  const int t = ti * tile + threadIdx.x;
#pragma unroll
  for (int j = 0; j < kTopK; ++j) {
    const int p = threadIdx.x * kTopK + j, w = p >> 5;
    const uint32_t* row = smu + mm[j] * words;
    const int before = pre[mm[j] * words + w] + __popc(row[w] & ((1u << (p & 31)) - 1u));
    ent[off[mm[j]] + c[mm[j]] + before] = t * 8 + j;
  }
}

// ---------------------------------------------------------------------------
// select + attend, backward, token side: a warp per token. kStaged: the (b,h) key and value
// tables are first copied into shared memory and a block's warps take kTokS tokens each (the
// picked rows then come from shared memory instead of L2); the arithmetic is the same.
//   dw_j = g . V[i_j] (+ grad_weights), da_j = w_j (dw_j - sum_k w_k dw_k),
//   dq = scale sum_j da_j K[i_j]; coef[t][j] = scale da_j for the slot side.
// ---------------------------------------------------------------------------
constexpr int kTokS = 16;  // tokens per warp of the staged token-side kernels
constexpr size_t kMaxStagedTables = 160 * 1024;  // shared memory for a staged (b,h) table pair
template <typename T, int U, bool kStaged>  // U head dims per lane: d = lane + 32 u, D <= 32 U
__global__ void __launch_bounds__(kStaged ? 512 : 256, kStaged ? 2 : 3) k_sa_bwd_tok(murm_select_attend_bwd_args a, float* coef) {
  extern __shared__ float sh_tab[];
  const int N = a.shape.tokens, D = a.shape.head_dim, M = a.shape.slots;
  const int bh = blockIdx.y, b = bh / a.shape.heads, h = bh - b * a.shape.heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  T* tK = reinterpret_cast<T*>(sh_tab);  // [M][D] (kStaged)
  T* tV = tK + (size_t)M * D;
  if constexpr (kStaged) {
    for (int e = threadIdx.x; e < M * D; e += blockDim.x) {
      const int m = e / D, d = e - m * D;
      tK[e] = static_cast<const T*>(a.slot_keys)[off3(a.sk_stride, b, h, m) + d];
      tV[e] = static_cast<const T*>(a.slot_values)[off3(a.sv_stride, b, h, m) + d];
    }
    __syncthreads();
  }
  auto skey = [&](int m, int d) -> float {
    if constexpr (kStaged) return Elem<T>::load(tK + (size_t)m * D + d);
    else return ld<T>(a.slot_keys, off3(a.sk_stride, b, h, m) + d);
  };
  auto sval = [&](int m, int d) -> float {
    if constexpr (kStaged) return Elem<T>::load(tV + (size_t)m * D + d);
    else return ld<T>(a.slot_values, off3(a.sv_stride, b, h, m) + d);
  };
  const int nw = blockDim.x >> 5;
  const int ntok = kStaged ? kTokS : 1;
  for (int i = 0; i < ntok; ++i) {
  const int n = kStaged ? (blockIdx.x * kTokS + i) * nw + warp : blockIdx.x * 8 + warp;
  if (n >= N) return;
  const float scale = a.scale > 0 ? (float)a.scale : rsqrtf((float)D);
  const int64_t rec = ((int64_t)bh * N + n) * kTopK;
  int pick[kTopK];
  float w[kTopK], dw[kTopK];
#pragma unroll
  for (int j = 0; j < kTopK; ++j) {
    pick[j] = clampi(a.indices[rec + j], M);
    w[j] = a.weights[rec + j];
  }
  float g[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int d = lane + 32 * u;
    g[u] = d < D ? ld<T>(a.grad_out, off3(a.go_stride, b, h, n) + d) : 0.f;
  }
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < kTopK; ++j) {
    float p = 0.f;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int d = lane + 32 * u;
      if (d < D) p = fmaf(g[u], sval(pick[j], d), p);
    }
    dw[j] = warp_sum(p) + (a.grad_weights ? a.grad_weights[rec + j] : 0.f);
    s = fmaf(w[j], dw[j], s);
  }
  float c[kTopK];
#pragma unroll
  for (int j = 0; j < kTopK; ++j) c[j] = scale * (w[j] * (dw[j] - s));
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int d = lane + 32 * u;
    if (d < D) {
      float dq = 0.f;
#pragma unroll
      for (int j = 0; j < kTopK; ++j) dq = fmaf(c[j], skey(pick[j], d), dq);
      st<T>(a.grad_q, off3(a.gq_stride, b, h, n) + d, dq);
    }
  }
  if (lane < kTopK) {
    float cj = c[0];
#pragma unroll
    for (int j = 1; j < kTopK; ++j)
      if (lane == j) cj = c[j];
    coef[((int64_t)bh * N + n) * 8 + lane] = cj;
  }
  }  // tokens
}

// Over a slot's (token, pick) entries [e0, e1) in token order: acc1 += f1 * A[t] and
// acc2 += f2 * B[t] (lane's dims d = lane + 32 u, u < U, D <= 32 U), with f1, f2 per-pair
// factors (f[(rec0 + t) * stride + pick]) and, when fsum is given, *fsum += f2. The loads of
// several entries (8 for D <= 64, else 4) are issued before their sums, so that as many rows are
// in flight; the sums are taken in entry order all the same.
template <typename T, int U>
__device__ __forceinline__ void pair_sums(const int* ent, int e0, int e1, int64_t rec0, const float* f1, int s1,
                                          const float* f2, int s2, const T* A, const int64_t* as, const T* Bp,
                                          const int64_t* bs, int b, int h, int D, int lane,
                                          float (&acc1)[U], float (&acc2)[U], float* fsum) {
  constexpr int F = U <= 2 ? 8 : 4;  // entries in flight
  int e = e0;
  for (; e + F <= e1; e += F) {
    int tt[F], jj[F];
    float x1[F], x2[F], ra[F][U], rb[F][U];
#pragma unroll
    for (int r = 0; r < F; ++r) {
      const int en = ent[e + r];
      tt[r] = en >> 3;
      jj[r] = en & 7;
    }
#pragma unroll
    for (int r = 0; r < F; ++r) {
      x1[r] = f1[(rec0 + tt[r]) * s1 + jj[r]];
      x2[r] = f2[(rec0 + tt[r]) * s2 + jj[r]];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int d = lane + 32 * u;
        ra[r][u] = d < D ? Elem<T>::load(A + off3(as, b, h, tt[r]) + d) : 0.f;
        rb[r][u] = d < D ? Elem<T>::load(Bp + off3(bs, b, h, tt[r]) + d) : 0.f;
      }
    }
#pragma unroll
    for (int r = 0; r < F; ++r) {
      if (fsum) *fsum += x2[r];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (lane + 32 * u < D) {
          acc1[u] = fmaf(x1[r], ra[r][u], acc1[u]);
          acc2[u] = fmaf(x2[r], rb[r][u], acc2[u]);
        }
      }
    }
  }
  for (; e < e1; ++e) {
    const int t = ent[e] >> 3, j = ent[e] & 7;
    const float y1 = f1[(rec0 + t) * s1 + j], y2 = f2[(rec0 + t) * s2 + j];
    if (fsum) *fsum += y2;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int d = lane + 32 * u;
      if (d < D) {
        acc1[u] = fmaf(y1, Elem<T>::load(A + off3(as, b, h, t) + d), acc1[u]);
        acc2[u] = fmaf(y2, Elem<T>::load(Bp + off3(bs, b, h, t) + d), acc2[u]);
      }
    }
  }
}

// A slot's entry sums by kSumParts warps: a block of 8 warps takes 8 / kSumParts slots, each
// slot's entry list cut into kSumParts contiguous parts, each summed in token order by pair_sums;
// the first part's warp then adds the others' sums in part order (a fixed order: deterministic).
// Returns true in the first part's warp of a slot < M, which holds the slot's sums (m set to the
// slot either way).
constexpr int kSumParts = 4;
template <typename T, int U>
__device__ __forceinline__ bool slot_sums_2(const int* off, const int* ent, int64_t rec0, const float* f1, int s1,
                                            const float* f2, int s2, const T* A, const int64_t* as, const T* Bp,
                                            const int64_t* bs, int b, int h, int D, int M, int& m, float (&acc1)[U],
                                            float (&acc2)[U], float* fsum) {
  constexpr int P = kSumParts, S = 8 / P;
  __shared__ float part[S][P][2 * U * 32 + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, sl = warp / P, pi = warp % P;
  m = blockIdx.x * S + sl;
#pragma unroll
  for (int u = 0; u < U; ++u) acc1[u] = acc2[u] = 0.f;
  if (fsum) *fsum = 0.f;
  if (m < M) {
    const int e0 = off[m], n = off[m + 1] - e0;
    pair_sums<T, U>(ent, e0 + (int)((int64_t)n * pi / P), e0 + (int)((int64_t)n * (pi + 1) / P), rec0, f1, s1, f2, s2,
                    A, as, Bp, bs, b, h, D, lane, acc1, acc2, fsum);
    if (pi) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        part[sl][pi][u * 32 + lane] = acc1[u];
        part[sl][pi][(U + u) * 32 + lane] = acc2[u];
      }
      if (fsum && lane == 0) part[sl][pi][2 * U * 32] = *fsum;
    }
  }
  __syncthreads();
  if (m >= M || pi) return false;
#pragma unroll
  for (int p = 1; p < P; ++p) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      acc1[u] += part[sl][p][u * 32 + lane];
      acc2[u] += part[sl][p][(U + u) * 32 + lane];
    }
    if (fsum) *fsum += part[sl][p][2 * U * 32];
  }
  return true;
}

// slot side: kSumParts warps per (b,h, slot), its pairs in token order:
//   dK[m] = sum coef * q[t],  dV[m] = sum w * g[t]
template <typename T, int U>  // U head dims per lane: d = lane + 32 u, D <= 32 U
__global__ void __launch_bounds__(256, 3) k_sa_bwd_slot(murm_select_attend_bwd_args a, const float* coef,
                                                     const int* offsets, const int* entries) {
  const int N = a.shape.tokens, D = a.shape.head_dim, M = a.shape.slots;
  const int bh = blockIdx.y, b = bh / a.shape.heads, h = bh - b * a.shape.heads;
  const int lane = threadIdx.x & 31;
  const int* off = offsets + (int64_t)bh * (M + 1);
  const int* ent = entries + (int64_t)bh * N * kTopK;
  int m;
  float dk[U], dv[U];
  if (!slot_sums_2<T, U>(off, ent, (int64_t)bh * N, coef, 8, a.weights, kTopK, static_cast<const T*>(a.q), a.q_stride,
                         static_cast<const T*>(a.grad_out), a.go_stride, b, h, D, M, m, dk, dv, nullptr))
    return;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int d = lane + 32 * u;
    if (d < D) {
      st<T>(a.grad_slot_keys, off3(a.gsk_stride, b, h, m) + d, dk[u]);
      st<T>(a.grad_slot_values, off3(a.gsv_stride, b, h, m) + d, dv[u]);
    }
  }
}

// ---------------------------------------------------------------------------
// slot update, forward: kSumParts warps per (b,h, slot). saved = U_k, U_v [BH][M][D] and
// W [BH][M] (fp32).
// ---------------------------------------------------------------------------
template <typename T, int U>  // U head dims per lane: d = lane + 32 u, D <= 32 U
__global__ void __launch_bounds__(256, 3) k_upd_fwd(murm_slot_update_args a, const int* offsets, const int* entries,
                                                 float* Uk, float* Uv, float* Wsum) {
  const int N = a.shape.tokens, D = a.shape.head_dim, M = a.shape.slots;
  const int bh = blockIdx.y, b = bh / a.shape.heads, h = bh - b * a.shape.heads;
  const int lane = threadIdx.x & 31;
  const int* off = offsets + (int64_t)bh * (M + 1);
  const int* ent = entries + (int64_t)bh * N * kTopK;
  int m;
  float sk[U], sv[U];
  float W = 0.f;
  if (!slot_sums_2<T, U>(off, ent, (int64_t)bh * N, a.weights, kTopK, a.weights, kTopK,
                         static_cast<const T*>(a.token_keys), a.tk_stride, static_cast<const T*>(a.token_values),
                         a.tv_stride, b, h, D, M, m, sk, sv, &W))
    return;
  const bool valid = W > 0.f;                       // reference.py:105
  const float den = __fadd_rn(W, kEmaEps);          // :106-107
  const float al = (float)a.alpha, om = (float)(1.0 - a.alpha);
  const size_t so = ((size_t)bh * M + m) * D;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int d = lane + 32 * u;
    if (d < D) {
      const float uk = __fdiv_rn(sk[u], den), uv = __fdiv_rn(sv[u], den);
      Uk[so + d] = uk;
      Uv[so + d] = uv;
      const float ok = ld<T>(a.slot_keys, off3(a.sk_stride, b, h, m) + d);
      const float ov = ld<T>(a.slot_values, off3(a.sv_stride, b, h, m) + d);
      // :112-113 alpha * old + (1 - alpha) * update where valid
      st<T>(a.new_slot_keys, off3(a.nsk_stride, b, h, m) + d,
            valid ? __fadd_rn(__fmul_rn(al, ok), __fmul_rn(om, uk)) : ok);
      st<T>(a.new_slot_values, off3(a.nsv_stride, b, h, m) + d,
            valid ? __fadd_rn(__fmul_rn(al, ov), __fmul_rn(om, uv)) : ov);
    }
  }
  if (lane == 0) Wsum[(size_t)bh * M + m] = W;
}

// slot sums alone (kSumParts warps per (b,h, slot)): fp32 [BH][M][D] key/value sums, [BH][M] weights.
template <typename T, int U>  // U head dims per lane: d = lane + 32 u, D <= 32 U
__global__ void __launch_bounds__(256, 3) k_sums_fwd(murm_slot_sums_args a, const int* offsets, const int* entries) {
  const int N = a.shape.tokens, D = a.shape.head_dim, M = a.shape.slots;
  const int bh = blockIdx.y, b = bh / a.shape.heads, h = bh - b * a.shape.heads;
  const int lane = threadIdx.x & 31;
  const int* off = offsets + (int64_t)bh * (M + 1);
  const int* ent = entries + (int64_t)bh * N * kTopK;
  int m;
  float sk[U], sv[U];
  float W = 0.f;
  if (!slot_sums_2<T, U>(off, ent, (int64_t)bh * N, a.weights, kTopK, a.weights, kTopK,
                         static_cast<const T*>(a.token_keys), a.tk_stride, static_cast<const T*>(a.token_values),
                         a.tv_stride, b, h, D, M, m, sk, sv, &W))
    return;
  const size_t so = ((size_t)bh * M + m) * D;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int d = lane + 32 * u;
    if (d < D) {
      a.key_sums[so + d] = sk[u];
      a.value_sums[so + d] = sv[u];
    }
  }
  if (lane == 0) a.weight_sums[(size_t)bh * M + m] = W;
}

// slot update, backward, slot side: grad of the old slots and the adjoints of the
// sums: dks = (1-a) g_k / (W + eps), dW = -(dks . U_k + dvs . U_v), where W > 0.
template <typename T>
__global__ void __launch_bounds__(256) k_upd_bwd_slot(murm_slot_update_bwd_args a, const float* Uk, const float* Uv,
                                                      const float* Wsum, float* dks, float* dvs, float* dW) {
  const int D = a.shape.head_dim, M = a.shape.slots;
  const int bh = blockIdx.y, b = bh / a.shape.heads, h = bh - b * a.shape.heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m = blockIdx.x * 8 + warp;
  if (m >= M) return;
  const float W = Wsum[(size_t)bh * M + m];
  const bool valid = W > 0.f;
  const float den = __fadd_rn(W, kEmaEps);
  const float al = (float)a.alpha, om = (float)(1.0 - a.alpha);
  const size_t so = ((size_t)bh * M + m) * D;
  float dot = 0.f;
  for (int d = lane; d < D; d += 32) {
    const float gk = ld<T>(a.grad_new_keys, off3(a.gnk_stride, b, h, m) + d);
    const float gv = ld<T>(a.grad_new_values, off3(a.gnv_stride, b, h, m) + d);
    st<T>(a.grad_slot_keys, off3(a.gsk_stride, b, h, m) + d, valid ? al * gk : gk);
    st<T>(a.grad_slot_values, off3(a.gsv_stride, b, h, m) + d, valid ? al * gv : gv);
    const float k2 = valid ? om * gk / den : 0.f, v2 = valid ? om * gv / den : 0.f;
    dks[so + d] = k2;
    dvs[so + d] = v2;
    dot = fmaf(k2, Uk[so + d], fmaf(v2, Uv[so + d], dot));
  }
  dot = warp_sum(dot);
  if (lane == 0) dW[(size_t)bh * M + m] = -dot;
}

// slot update, backward, token side: a warp per token. kStaged: the (b,h) slot adjoints (dks,
// dvs, dW; fp32) are first copied into shared memory and a block's warps take kTokS tokens each.
template <typename T, int U, bool kStaged>  // U head dims per lane: d = lane + 32 u, D <= 32 U
__global__ void __launch_bounds__(kStaged ? 512 : 256) k_upd_bwd_tok(murm_slot_update_bwd_args a, const float* dks,
                                                                     const float* dvs, const float* dW) {
  extern __shared__ float sh_adj[];
  const int N = a.shape.tokens, D = a.shape.head_dim, M = a.shape.slots;
  const int bh = blockIdx.y, b = bh / a.shape.heads, h = bh - b * a.shape.heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* aK = dks + (size_t)bh * M * D;  // this (b,h)'s adjoints: global, or their shared copy
  const float* aV = dvs + (size_t)bh * M * D;
  const float* aW = dW + (size_t)bh * M;
  if constexpr (kStaged) {
    float* s = sh_adj;
    const int q = M * D / 4;  // D is a multiple of 8: whole float4s
    for (int e = threadIdx.x; e < q; e += blockDim.x) {
      reinterpret_cast<float4*>(s)[e] = reinterpret_cast<const float4*>(aK)[e];
      reinterpret_cast<float4*>(s + (size_t)M * D)[e] = reinterpret_cast<const float4*>(aV)[e];
    }
    for (int m = threadIdx.x; m < M; m += blockDim.x) s[2 * (size_t)M * D + m] = aW[m];
    __syncthreads();
    aK = s;
    aV = s + (size_t)M * D;
    aW = s + 2 * (size_t)M * D;
  }
  const int nw = blockDim.x >> 5;
  const int ntok = kStaged ? kTokS : 1;
  for (int i = 0; i < ntok; ++i) {
  const int n = kStaged ? (blockIdx.x * kTokS + i) * nw + warp : blockIdx.x * 8 + warp;
  if (n >= N) return;
  const int64_t rec = ((int64_t)bh * N + n) * kTopK;
  float tk[U], tv[U], gk[U], gv[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int d = lane + 32 * u;
    tk[u] = d < D ? ld<T>(a.token_keys, off3(a.tk_stride, b, h, n) + d) : 0.f;
    tv[u] = d < D ? ld<T>(a.token_values, off3(a.tv_stride, b, h, n) + d) : 0.f;
    gk[u] = gv[u] = 0.f;
  }
  float gw[kTopK];
#pragma unroll
  for (int j = 0; j < kTopK; ++j) {
    const int m = clampi(a.indices[rec + j], M);
    const float wt = a.weights[rec + j];
    const size_t so = (size_t)m * D;
    float p = 0.f;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int d = lane + 32 * u;
      if (d < D) {
        const float k2 = aK[so + d], v2 = aV[so + d];
        gk[u] = fmaf(wt, k2, gk[u]);
        gv[u] = fmaf(wt, v2, gv[u]);
        p = fmaf(tk[u], k2, fmaf(tv[u], v2, p));
      }
    }
    gw[j] = warp_sum(p) + aW[m];
  }
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int d = lane + 32 * u;
    if (d < D) {
      st<T>(a.grad_token_keys, off3(a.gtk_stride, b, h, n) + d, gk[u]);
      st<T>(a.grad_token_values, off3(a.gtv_stride, b, h, n) + d, gv[u]);
    }
  }
  if (lane < kTopK) {
    float x = gw[0];
#pragma unroll
    for (int j = 1; j < kTopK; ++j)
      if (lane == j) x = gw[j];
    a.grad_weights[rec + lane] = x;
  }
  }  // tokens
}

// ---------------------------------------------------------------------------
// slot diffusion: grid (M, BH), a thread per head dim. Forward in the reference's
// operation order (reference.py:128-133) with explicit roundings; backward is the
// transposed stencil.
// ---------------------------------------------------------------------------
template <typename T, bool kBackward>
__global__ void k_diffusion(murm_slot_diffusion_args a) {
  const int M = a.shape.slots, D = a.shape.head_dim;
  const int m = blockIdx.x, bh = blockIdx.y, b = bh / a.shape.heads, h = bh - b * a.shape.heads;
  const float gm = (float)a.gamma;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
#pragma unroll
    for (int kv = 0; kv < 2; ++kv) {
      const void* in = kv ? a.in_values : a.in_keys;
      const int64_t* is = kv ? a.iv_stride : a.ik_stride;
      void* out = kv ? a.out_values : a.out_keys;
      const int64_t* os = kv ? a.ov_stride : a.ok_stride;
      const float x = ld<T>(in, off3(is, b, h, m) + d);
      float y;
      if (!kBackward) {
        y = x;
        if (m > 0 && m < M - 1) {
          const float l = ld<T>(in, off3(is, b, h, m - 1) + d), r = ld<T>(in, off3(is, b, h, m + 1) + d);
          y = __fadd_rn(x, __fmul_rn(gm, __fsub_rn(__fadd_rn(l, r), __fmul_rn(2.f, x))));
        }
      } else {
        const bool in_m = m > 0 && m < M - 1, in_l = m - 1 > 0, in_r = m + 1 < M - 1;
        y = in_m ? __fadd_rn(x, __fmul_rn(-2.f * gm, x)) : x;
        if (in_l) y = __fadd_rn(y, __fmul_rn(gm, ld<T>(in, off3(is, b, h, m - 1) + d)));
        if (in_r) y = __fadd_rn(y, __fmul_rn(gm, ld<T>(in, off3(is, b, h, m + 1) + d)));
      }
      st<T>(out, off3(os, b, h, m) + d, y);
    }
  }
}

// ---------------------------------------------------------------------------
// Streaming decode: one CTA per (b,h), 256 threads. The pool is staged in shared
// memory as fp32 rows of d+1 words (odd stride: a thread per slot row reads
// without bank conflicts); the 7 picked rows are updated there, rounded to the
// pool's dtype (the reference's type_as), and the diffused pool is written back.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) k_decode(murm_decode_args a) {
  extern __shared__ float sm[];
  const int M = a.slots, D = a.head_dim, Dp = D + 1;
  float* sK = sm;                          // [M][Dp]
  float* sV = sK + (size_t)M * Dp;         // [M][Dp]
  float* qv = sV + (size_t)M * Dp;         // [D]
  float* kv = qv + D;                      // [D] token key
  float* vv = kv + D;                      // [D] token value
  uint32_t* keys = reinterpret_cast<uint32_t*>(vv + D);  // [M]
  int* pick_s = reinterpret_cast<int*>(keys + M);        // [8]
  float* w_s = reinterpret_cast<float*>(pick_s + 8);     // [8]
  const int bh = blockIdx.x, b = bh / a.heads, h = bh - b * a.heads;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int e = tid; e < M * D; e += blockDim.x) {
    const int m = e / D, d = e - m * D;
    sK[m * Dp + d] = ld<T>(a.slot_keys, off3(a.sk_stride, b, h, m) + d);
    sV[m * Dp + d] = ld<T>(a.slot_values, off3(a.sv_stride, b, h, m) + d);
  }
  const int64_t qo = (int64_t)b * a.q_stride[0] + (int64_t)h * a.q_stride[1];
  const int64_t ko = (int64_t)b * a.k_stride[0] + (int64_t)h * a.k_stride[1];
  const int64_t vo = (int64_t)b * a.v_stride[0] + (int64_t)h * a.v_stride[1];
  for (int d = tid; d < D; d += blockDim.x) {
    qv[d] = ld<T>(a.q, qo + d);
    kv[d] = ld<T>(a.k, ko + d);
    vv[d] = ld<T>(a.v, vo + d);
  }
  __syncthreads();
  const int64_t pos = a.causal ? a.positions[b] : 0;
  for (int m = tid; m < M; m += blockDim.x) {  // selection scores (reference.py:19, 27-31)
    float s = 0.f;
    for (int d = 0; d < D; ++d) s = fmaf(qv[d], sK[m * Dp + d], s);
    keys[m] = rank_key((a.causal && m > pos) ? -INFINITY : s);
  }
  __syncthreads();
  const float scale = a.scale > 0 ? (float)a.scale : rsqrtf((float)D);
  if (warp == 0) {
    uint32_t tk[kTopK];
    int ts[kTopK];
#pragma unroll
    for (int j = 0; j < kTopK; ++j) { tk[j] = 0u; ts[j] = 0; }
    for (int m = lane; m < M; m += 32) offer7(tk, ts, keys[m], m);
    warp_top7(tk, ts);
    float sc[kTopK], mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < kTopK; ++j) {  // attend scores without the mask (reference.py:61)
      float p = 0.f;
      for (int d = lane; d < D; d += 32) p = fmaf(qv[d], sK[ts[j] * Dp + d], p);
      sc[j] = warp_sum(p) * scale;
      mx = fmaxf(mx, sc[j]);
    }
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < kTopK; ++j) {
      sc[j] = expf(sc[j] - mx);
      sum += sc[j];
    }
    if (lane < kTopK) {
      int pj = ts[0];
      float wj = sc[0];
#pragma unroll
      for (int j = 1; j < kTopK; ++j)
        if (lane == j) { pj = ts[j]; wj = sc[j]; }
      wj = wj / sum;
      pick_s[lane] = pj;
      w_s[lane] = wj;
      if (a.indices) a.indices[(int64_t)bh * kTopK + lane] = pj;
      if (a.weights) a.weights[(int64_t)bh * kTopK + lane] = wj;
    }
  }
  __syncthreads();
  // out = x + sum_j w_j V[i_j] (with the values before this token's update)
  const int64_t oo = (int64_t)b * a.out_stride[0] + (int64_t)h * a.out_stride[1];
  const int64_t xo = a.x ? (int64_t)b * a.x_stride[0] + (int64_t)h * a.x_stride[1] : 0;
  for (int d = tid; d < D; d += blockDim.x) {
    float o = 0.f;
#pragma unroll
    for (int j = 0; j < kTopK; ++j) o = fmaf(w_s[j], sV[pick_s[j] * Dp + d], o);
    st<T>(a.out, oo + d, (a.x ? ld<T>(a.x, xo + d) : 0.f) + o);
  }
  __syncthreads();
  // update of the picked (distinct) slots with this one token (reference.py:93-115)
  const float al = (float)a.alpha, om = (float)(1.0 - a.alpha);
  for (int e = tid; e < kTopK * D; e += blockDim.x) {
    const int j = e / D, d = e - j * D, m = pick_s[j];
    const float wj = w_s[j];
    if (wj > 0.f) {
      const float den = __fadd_rn(wj, kEmaEps);
      const float uk = __fdiv_rn(__fmul_rn(kv[d], wj), den), uv = __fdiv_rn(__fmul_rn(vv[d], wj), den);
      T rk, rv;
      Elem<T>::store(&rk, __fadd_rn(__fmul_rn(al, sK[m * Dp + d]), __fmul_rn(om, uk)));
      Elem<T>::store(&rv, __fadd_rn(__fmul_rn(al, sV[m * Dp + d]), __fmul_rn(om, uv)));
      sK[m * Dp + d] = Elem<T>::load(&rk);
      sV[m * Dp + d] = Elem<T>::load(&rv);
    }
  }
  __syncthreads();
  // diffusion of the whole pool, written back (reference.py:128-133)
  const float gm = (float)a.gamma;
  for (int e = tid; e < M * D; e += blockDim.x) {
    const int m = e / D, d = e - m * D;
    float k = sK[m * Dp + d], v = sV[m * Dp + d];
    if (m > 0 && m < M - 1) {
      k = __fadd_rn(k, __fmul_rn(gm, __fsub_rn(__fadd_rn(sK[(m - 1) * Dp + d], sK[(m + 1) * Dp + d]),
                                                __fmul_rn(2.f, k))));
      v = __fadd_rn(v, __fmul_rn(gm, __fsub_rn(__fadd_rn(sV[(m - 1) * Dp + d], sV[(m + 1) * Dp + d]),
                                                __fmul_rn(2.f, v))));
    }
    st<T>(a.slot_keys, off3(a.sk_stride, b, h, m) + d, k);
    st<T>(a.slot_values, off3(a.sv_stride, b, h, m) + d, v);
  }
}

// Decode step with 16-byte pool accesses (pool rows whose byte size and strides are multiples
// of 16): the pool stays in its own dtype in shared memory (half the footprint of an fp32
// copy, so several heads share an SM), rows of C 16-byte chunks with chunk c of row m at
// c ^ (m & swz), so that a warp's threads, one slot each, read different banks. Same
// arithmetic, in the same order, as k_decode.
template <typename T>
__global__ void __launch_bounds__(256) k_decode_v(murm_decode_args a) {
  extern __shared__ uint4 smv[];
  constexpr int E = 16 / (int)sizeof(T);  // elements per chunk
  const int M = a.slots, D = a.head_dim, C = D / E;
  const int swz = ((C & (C - 1)) == 0) ? (C < 8 ? C - 1 : 7) : 0;
  uint4* sK = smv;                                  // [M][C]
  uint4* sV = sK + (size_t)M * C;                   // [M][C]
  float* qv = reinterpret_cast<float*>(sV + (size_t)M * C);  // [D]
  float* kv = qv + D;                               // [D] token key
  float* vv = kv + D;                               // [D] token value
  uint32_t* keys = reinterpret_cast<uint32_t*>(vv + D);  // [M]
  int* pick_s = reinterpret_cast<int*>(keys + M);        // [8]
  float* w_s = reinterpret_cast<float*>(pick_s + 8);     // [8]
  const int bh = blockIdx.x, b = bh / a.heads, h = bh - b * a.heads;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  auto at = [&](int m, int c) { return m * C + (c ^ (m & swz)); };
  auto elem = [&](const uint4* arr, int m, int d) -> T* {
    return reinterpret_cast<T*>(const_cast<uint4*>(arr) + at(m, d / E)) + (d % E);
  };
  const T* gk = static_cast<const T*>(a.slot_keys);
  const T* gv = static_cast<const T*>(a.slot_values);
  for (int e = tid; e < M * C; e += blockDim.x) {
    const int m = e / C, c = e - m * C;
    sK[at(m, c)] = *reinterpret_cast<const uint4*>(gk + off3(a.sk_stride, b, h, m) + c * E);
    sV[at(m, c)] = *reinterpret_cast<const uint4*>(gv + off3(a.sv_stride, b, h, m) + c * E);
  }
  const int64_t qo = (int64_t)b * a.q_stride[0] + (int64_t)h * a.q_stride[1];
  const int64_t ko = (int64_t)b * a.k_stride[0] + (int64_t)h * a.k_stride[1];
  const int64_t vo = (int64_t)b * a.v_stride[0] + (int64_t)h * a.v_stride[1];
  for (int d = tid; d < D; d += blockDim.x) {
    qv[d] = ld<T>(a.q, qo + d);
    kv[d] = ld<T>(a.k, ko + d);
    vv[d] = ld<T>(a.v, vo + d);
  }
  __syncthreads();
  const int64_t pos = a.causal ? a.positions[b] : 0;
  for (int m = tid; m < M; m += blockDim.x) {  // selection scores (reference.py:19, 27-31)
    float s = 0.f;
    for (int c = 0; c < C; ++c) {
      const uint4 u = sK[at(m, c)];
      const T* t = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int i = 0; i < E; ++i) s = fmaf(qv[c * E + i], Elem<T>::load(t + i), s);
    }
    keys[m] = rank_key((a.causal && m > pos) ? -INFINITY : s);
  }
  __syncthreads();
  const float scale = a.scale > 0 ? (float)a.scale : rsqrtf((float)D);
  if (warp == 0) {
    uint32_t tk[kTopK];
    int ts[kTopK];
#pragma unroll
    for (int j = 0; j < kTopK; ++j) { tk[j] = 0u; ts[j] = 0; }
    for (int m = lane; m < M; m += 32) offer7(tk, ts, keys[m], m);
    warp_top7(tk, ts);
    float sc[kTopK], mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < kTopK; ++j) {  // attend scores without the mask (reference.py:61)
      float p = 0.f;
      for (int d = lane; d < D; d += 32) p = fmaf(qv[d], Elem<T>::load(elem(sK, ts[j], d)), p);
      sc[j] = warp_sum(p) * scale;
      mx = fmaxf(mx, sc[j]);
    }
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < kTopK; ++j) {
      sc[j] = expf(sc[j] - mx);
      sum += sc[j];
    }
    if (lane < kTopK) {
      int pj = ts[0];
      float wj = sc[0];
#pragma unroll
      for (int j = 1; j < kTopK; ++j)
        if (lane == j) { pj = ts[j]; wj = sc[j]; }
      wj = wj / sum;
      pick_s[lane] = pj;
      w_s[lane] = wj;
      if (a.indices) a.indices[(int64_t)bh * kTopK + lane] = pj;
      if (a.weights) a.weights[(int64_t)bh * kTopK + lane] = wj;
    }
  }
  __syncthreads();
  // out = x + sum_j w_j V[i_j] (with the values before this token's update)
  const int64_t oo = (int64_t)b * a.out_stride[0] + (int64_t)h * a.out_stride[1];
  const int64_t xo = a.x ? (int64_t)b * a.x_stride[0] + (int64_t)h * a.x_stride[1] : 0;
  for (int d = tid; d < D; d += blockDim.x) {
    float o = 0.f;
#pragma unroll
    for (int j = 0; j < kTopK; ++j) o = fmaf(w_s[j], Elem<T>::load(elem(sV, pick_s[j], d)), o);
    st<T>(a.out, oo + d, (a.x ? ld<T>(a.x, xo + d) : 0.f) + o);
  }
  __syncthreads();
  // update of the picked (distinct) slots with this one token (reference.py:93-115)
  const float al = (float)a.alpha, om = (float)(1.0 - a.alpha);
  for (int e = tid; e < kTopK * D; e += blockDim.x) {
    const int j = e / D, d = e - j * D, m = pick_s[j];
    const float wj = w_s[j];
    if (wj > 0.f) {
      const float den = __fadd_rn(wj, kEmaEps);
      const float uk = __fdiv_rn(__fmul_rn(kv[d], wj), den), uv = __fdiv_rn(__fmul_rn(vv[d], wj), den);
      T* pk = elem(sK, m, d);
      T* pv = elem(sV, m, d);
      Elem<T>::store(pk, __fadd_rn(__fmul_rn(al, Elem<T>::load(pk)), __fmul_rn(om, uk)));
      Elem<T>::store(pv, __fadd_rn(__fmul_rn(al, Elem<T>::load(pv)), __fmul_rn(om, uv)));
    }
  }
  __syncthreads();
  // diffusion of the whole pool, written back 16 bytes at a time (reference.py:128-133)
  const float gm = (float)a.gamma;
  T* ok = static_cast<T*>(a.slot_keys);
  T* ov = static_cast<T*>(a.slot_values);
  for (int e = tid; e < M * C; e += blockDim.x) {
    const int m = e / C, c = e - m * C;
    const bool inner = m > 0 && m < M - 1;
    const uint4 k0 = sK[at(m, c)], v0 = sV[at(m, c)];
    uint4 kl = k0, kr = k0, vl = v0, vr = v0;
    if (inner) {
      kl = sK[at(m - 1, c)]; kr = sK[at(m + 1, c)];
      vl = sV[at(m - 1, c)]; vr = sV[at(m + 1, c)];
    }
    uint4 ko4, vo4;
    const T *tk0 = reinterpret_cast<const T*>(&k0), *tkl = reinterpret_cast<const T*>(&kl),
            *tkr = reinterpret_cast<const T*>(&kr), *tv0 = reinterpret_cast<const T*>(&v0),
            *tvl = reinterpret_cast<const T*>(&vl), *tvr = reinterpret_cast<const T*>(&vr);
    T* tko = reinterpret_cast<T*>(&ko4);
    T* tvo = reinterpret_cast<T*>(&vo4);
#pragma unroll
    for (int i = 0; i < E; ++i) {
      float k = Elem<T>::load(tk0 + i), v = Elem<T>::load(tv0 + i);
      if (inner) {
        k = __fadd_rn(k, __fmul_rn(gm, __fsub_rn(__fadd_rn(Elem<T>::load(tkl + i), Elem<T>::load(tkr + i)),
                                                  __fmul_rn(2.f, k))));
        v = __fadd_rn(v, __fmul_rn(gm, __fsub_rn(__fadd_rn(Elem<T>::load(tvl + i), Elem<T>::load(tvr + i)),
                                                  __fmul_rn(2.f, v))));
      }
      Elem<T>::store(tko + i, k);
      Elem<T>::store(tvo + i, v);
    }
    *reinterpret_cast<uint4*>(ok + off3(a.sk_stride, b, h, m) + c * E) = ko4;
    *reinterpret_cast<uint4*>(ov + off3(a.sv_stride, b, h, m) + c * E) = vo4;
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct Sizes {
  size_t saved, ws, off_csr_entries, off_coef, off_dks, off_dvs, off_dw, off_cnt;
};
inline size_t a256(size_t x) { return (x + 255) & ~size_t(255); }

Sizes sizes(const murm_phase_shape& s) {
  const size_t BH = (size_t)s.batch * s.heads, N = s.tokens, M = s.slots, D = s.head_dim;
  Sizes z;
  z.saved = a256(BH * M * D * 4) * 2 + a256(BH * M * 4);
  size_t o = a256(BH * (M + 1) * 4);  // offsets
  z.off_csr_entries = o;
  o += a256(BH * N * kTopK * 4);
  z.off_coef = o;
  o += a256(BH * N * 8 * 4);
  z.off_dks = o;
  o += a256(BH * M * D * 4);
  z.off_dvs = o;
  o += a256(BH * M * D * 4);
  z.off_dw = o;
  o += a256(BH * M * 4);
  z.off_cnt = o;
  o += a256(BH * (size_t)((N + 63) / 64) * M * 4);  // per-tile slot counts (tiles of >= 64 tokens)
  z.ws = o;
  return z;
}

murm_status bad(murm_status s, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
murm_status bad(murm_status s, const char* fmt, ...) {
  char msg[256];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(msg, sizeof(msg), fmt, ap);
  va_end(ap);
  return report_error(s, msg);
}

murm_status check(const murm_phase_shape& s) {
  if (s.batch < 1 || s.heads < 1 || s.tokens < 1)
    return bad(MURM_ERR_INVALID_ARGUMENT, "batch, heads and tokens must be >= 1");
  if (s.slots < kTopK) return bad(MURM_ERR_INVALID_ARGUMENT, "slots=%d < top_k=%d", s.slots, kTopK);
  if (s.slots > kMaxM) return bad(MURM_ERR_UNSUPPORTED, "slots=%d > %d not supported", s.slots, kMaxM);
  if (s.head_dim < 8 || s.head_dim > kMaxD || s.head_dim % 8)
    return bad(MURM_ERR_UNSUPPORTED, "head_dim must be a multiple of 8 in [8, %d], got %d", kMaxD, s.head_dim);
  if ((size_t)s.head_dim * (s.slots + 1) * 4 > kMaxStage)
    return bad(MURM_ERR_UNSUPPORTED, "slots x head_dim too large (%d x %d)", s.slots, s.head_dim);
  if (s.dtype < MURM_F32 || s.dtype > MURM_BF16) return bad(MURM_ERR_DTYPE, "unsupported dtype code %d", s.dtype);
  if ((double)s.batch * s.heads * s.tokens * kTopK * 8 > 2147483647.0)
    return bad(MURM_ERR_UNSUPPORTED, "batch*heads*tokens too large");
  return MURM_OK;
}

// The instance of a warp-per-row kernel for the head dims per lane (1, 2 or 4: D <= 32, 64,
// 128), so that a lane holds registers for the dims it owns only.
template <typename F>
F per_lane_dims(int D, F u1, F u2, F u4) {
  return D <= 32 ? u1 : (D <= 64 ? u2 : u4);
}

murm_status launched(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return bad(MURM_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return MURM_OK;
}

murm_status ws_ok(const murm_phase_shape& s, const void* ws, size_t bytes) {
  if (!ws || bytes < sizes(s).ws || (reinterpret_cast<uintptr_t>(ws) & 255))
    return bad(MURM_ERR_WORKSPACE, "workspace NULL, unaligned or smaller than %zu bytes", sizes(s).ws);
  return MURM_OK;
}

void launch_csr(const murm_phase_shape& s, const int64_t* idx, uint8_t* ws, cudaStream_t st) {
  const int M = s.slots, N = s.tokens, BH = s.batch * s.heads;
  const int tile = M <= 256 ? 256 : (M <= 512 ? 128 : 64);
  const int words = (tile * kTopK + 31) / 32;
  const int ntiles = (N + tile - 1) / tile;
  const size_t smem = (size_t)M * words * 4;  // bitmap
  const size_t smem_fill = smem + (size_t)M * words * 2;  // + prefix counts
  const Sizes z = sizes(s);
  int* offsets = reinterpret_cast<int*>(ws);
  int* entries = reinterpret_cast<int*>(ws + z.off_csr_entries);
  int* cnt = reinterpret_cast<int*>(ws + z.off_cnt);
  smem_opt_in(k_csr_fill, smem_fill);
  MURM_LAUNCH("phase_csr_count", k_csr_count, dim3(ntiles, BH), 256, (size_t)M * 4, st, idx, N, M, tile, cnt);
  MURM_LAUNCH("phase_csr_scan", k_csr_scan, dim3(BH), 256, 0, st, ntiles, M, cnt, offsets);
  MURM_LAUNCH("phase_csr_fill", k_csr_fill, dim3(ntiles, BH), 256, smem_fill, st, idx, N, M, tile, words, cnt, offsets,
              entries);
}

template <typename T>
murm_status sa_fwd(const murm_select_attend_args& a, cudaStream_t st) {
  const int Mp = ((a.shape.slots + 31) / 32) * 32 + 1;
  const dim3 grid((a.shape.tokens + kWarps * kTokPerWarp - 1) / (kWarps * kTokPerWarp), a.shape.batch * a.shape.heads);
  const int64_t es = (int64_t)sizeof(T);
  int vec = (a.shape.head_dim * es) % 16 == 0 && (reinterpret_cast<uintptr_t>(a.slot_keys) & 15) == 0;
  for (int i = 0; i < 3; ++i) vec = vec && (a.sk_stride[i] * es) % 16 == 0;
  if (!a.indices_in && a.shape.slots <= 256) {  // four tokens per pass over the key table
    const size_t smem = ((((size_t)a.shape.head_dim * kMp4 + 3) & ~(size_t)3) + (size_t)kWarps * a.shape.head_dim * 4) * 4 +
                        (size_t)kWarps * 40 * sizeof(uint2);
    smem_opt_in(k_sa_fwd4<T>, smem);
    MURM_LAUNCH("phase_select_attend", k_sa_fwd4<T>, grid, 32 * kWarps, smem, st, a, vec);
  } else {
    const size_t smem = ((size_t)a.shape.head_dim * Mp + (size_t)kWarps * a.shape.head_dim) * 4;
    smem_opt_in(k_sa_fwd<T>, smem);
    MURM_LAUNCH("phase_select_attend", k_sa_fwd<T>, grid, 32 * kWarps, smem, st, a, Mp, vec);
  }
  return launched("select_attend forward");
}

template <typename T>
murm_status sa_bwd(const murm_select_attend_bwd_args& a, cudaStream_t st) {
  uint8_t* ws = static_cast<uint8_t*>(a.workspace);
  const Sizes z = sizes(a.shape);
  const int BH = a.shape.batch * a.shape.heads;
  launch_csr(a.shape, a.indices, ws, st);
  float* coef = reinterpret_cast<float*>(ws + z.off_coef);
  const int D = a.shape.head_dim;
  const auto kslot = per_lane_dims(D, k_sa_bwd_slot<T, 1>, k_sa_bwd_slot<T, 2>, k_sa_bwd_slot<T, 4>);
  const size_t tab = 2 * (size_t)a.shape.slots * D * sizeof(T);
  if (tab <= kMaxStagedTables) {  // the (b,h) key and value tables in shared memory
    const auto ktok = per_lane_dims(D, k_sa_bwd_tok<T, 1, true>, k_sa_bwd_tok<T, 2, true>, k_sa_bwd_tok<T, 4, true>);
    smem_opt_in(ktok, tab);
    MURM_LAUNCH("phase_select_attend_bwd_tokens", ktok, dim3((a.shape.tokens + 16 * kTokS - 1) / (16 * kTokS), BH), 512,
                tab, st, a, coef);
  } else {
    const auto ktok = per_lane_dims(D, k_sa_bwd_tok<T, 1, false>, k_sa_bwd_tok<T, 2, false>, k_sa_bwd_tok<T, 4, false>);
    MURM_LAUNCH("phase_select_attend_bwd_tokens", ktok, dim3((a.shape.tokens + 7) / 8, BH), 256, 0, st, a, coef);
  }
  MURM_LAUNCH("phase_select_attend_bwd_slots", kslot, dim3((a.shape.slots + 8 / kSumParts - 1) / (8 / kSumParts), BH), 256, 0, st, a,
              coef, reinterpret_cast<const int*>(ws), reinterpret_cast<const int*>(ws + z.off_csr_entries));
  return launched("select_attend backward");
}

template <typename T>
murm_status upd_fwd(const murm_slot_update_args& a, cudaStream_t st) {
  uint8_t* ws = static_cast<uint8_t*>(a.workspace);
  uint8_t* sv = static_cast<uint8_t*>(a.saved);
  const Sizes z = sizes(a.shape);
  const size_t BH = (size_t)a.shape.batch * a.shape.heads, MD = (size_t)a.shape.slots * a.shape.head_dim;
  launch_csr(a.shape, a.indices, ws, st);
  float* Uk = reinterpret_cast<float*>(sv);
  float* Uv = reinterpret_cast<float*>(sv + a256(BH * MD * 4));
  float* W = reinterpret_cast<float*>(sv + 2 * a256(BH * MD * 4));
  const auto kupd = per_lane_dims(a.shape.head_dim, k_upd_fwd<T, 1>, k_upd_fwd<T, 2>, k_upd_fwd<T, 4>);
  MURM_LAUNCH("phase_update", kupd, dim3((a.shape.slots + 8 / kSumParts - 1) / (8 / kSumParts), (unsigned)BH), 256, 0, st, a,
              reinterpret_cast<const int*>(ws), reinterpret_cast<const int*>(ws + z.off_csr_entries), Uk, Uv, W);
  return launched("slot_update forward");
}

// The token side of the update's backward: with the (b,h) adjoints staged in shared memory where
// they fit, else reading them from global memory.
template <typename T>
void launch_upd_bwd_tok(const char* name, const murm_slot_update_bwd_args& a, const float* dks, const float* dvs,
                        const float* dW, cudaStream_t st) {
  const int D = a.shape.head_dim;
  const unsigned BH = (unsigned)(a.shape.batch * a.shape.heads);
  const size_t tab = (2 * (size_t)a.shape.slots * D + a.shape.slots) * sizeof(float);
  if (tab <= kMaxStagedTables) {
    const auto k = per_lane_dims(D, k_upd_bwd_tok<T, 1, true>, k_upd_bwd_tok<T, 2, true>, k_upd_bwd_tok<T, 4, true>);
    smem_opt_in(k, tab);
    MURM_LAUNCH(name, k, dim3((a.shape.tokens + 16 * kTokS - 1) / (16 * kTokS), BH), 512, tab, st, a, dks, dvs, dW);
  } else {
    const auto k = per_lane_dims(D, k_upd_bwd_tok<T, 1, false>, k_upd_bwd_tok<T, 2, false>, k_upd_bwd_tok<T, 4, false>);
    MURM_LAUNCH(name, k, dim3((a.shape.tokens + 7) / 8, BH), 256, 0, st, a, dks, dvs, dW);
  }
}

template <typename T>
murm_status upd_bwd(const murm_slot_update_bwd_args& a, cudaStream_t st) {
  uint8_t* ws = static_cast<uint8_t*>(a.workspace);
  const uint8_t* sv = static_cast<const uint8_t*>(a.saved);
  const Sizes z = sizes(a.shape);
  const size_t BH = (size_t)a.shape.batch * a.shape.heads, MD = (size_t)a.shape.slots * a.shape.head_dim;
  const float* Uk = reinterpret_cast<const float*>(sv);
  const float* Uv = reinterpret_cast<const float*>(sv + a256(BH * MD * 4));
  const float* W = reinterpret_cast<const float*>(sv + 2 * a256(BH * MD * 4));
  float* dks = reinterpret_cast<float*>(ws + z.off_dks);
  float* dvs = reinterpret_cast<float*>(ws + z.off_dvs);
  float* dW = reinterpret_cast<float*>(ws + z.off_dw);
  MURM_LAUNCH("phase_update_bwd_slots", k_upd_bwd_slot<T>, dim3((a.shape.slots + 7) / 8, (unsigned)BH), 256, 0, st,
              a, Uk, Uv, W, dks, dvs, dW);
  launch_upd_bwd_tok<T>("phase_update_bwd_tokens", a, dks, dvs, dW, st);
  return launched("slot_update backward");
}

template <typename T>
murm_status sums_fwd(const murm_slot_sums_args& a, cudaStream_t st) {
  uint8_t* ws = static_cast<uint8_t*>(a.workspace);
  const Sizes z = sizes(a.shape);
  launch_csr(a.shape, a.indices, ws, st);
  const auto ksum = per_lane_dims(a.shape.head_dim, k_sums_fwd<T, 1>, k_sums_fwd<T, 2>, k_sums_fwd<T, 4>);
  MURM_LAUNCH("phase_sums", ksum, dim3((a.shape.slots + 8 / kSumParts - 1) / (8 / kSumParts), a.shape.batch * a.shape.heads), 256, 0, st,
              a, reinterpret_cast<const int*>(ws), reinterpret_cast<const int*>(ws + z.off_csr_entries));
  return launched("slot sums forward");
}

template <typename T>
murm_status sums_bwd(const murm_slot_sums_bwd_args& a, cudaStream_t st) {
  // the token side of the update's backward, with the sums' gradients as its slot adjoints
  murm_slot_update_bwd_args u{};
  u.shape = a.shape;
  u.token_keys = a.token_keys;
  u.token_values = a.token_values;
  for (int i = 0; i < 3; ++i) {
    u.tk_stride[i] = a.tk_stride[i];
    u.tv_stride[i] = a.tv_stride[i];
    u.gtk_stride[i] = a.gtk_stride[i];
    u.gtv_stride[i] = a.gtv_stride[i];
  }
  u.indices = a.indices;
  u.weights = a.weights;
  u.grad_token_keys = a.grad_token_keys;
  u.grad_token_values = a.grad_token_values;
  u.grad_weights = a.grad_weights;
  launch_upd_bwd_tok<T>("phase_sums_bwd", u, a.grad_key_sums, a.grad_value_sums, a.grad_weight_sums, st);
  return launched("slot sums backward");
}
template <typename T> struct SumFwd { static murm_status run(const murm_slot_sums_args& a, cudaStream_t s) { return sums_fwd<T>(a, s); } };
template <typename T> struct SumBwd { static murm_status run(const murm_slot_sums_bwd_args& a, cudaStream_t s) { return sums_bwd<T>(a, s); } };

template <typename T>
murm_status diff(const murm_slot_diffusion_args& a, bool backward, cudaStream_t st) {
  const dim3 grid(a.shape.slots, a.shape.batch * a.shape.heads);
  const int threads = a.shape.head_dim < 32 ? 32 : (a.shape.head_dim > 128 ? 128 : a.shape.head_dim);
  auto kern = backward ? k_diffusion<T, true> : k_diffusion<T, false>;
  MURM_LAUNCH(backward ? "phase_diffusion_bwd" : "phase_diffusion", kern, grid, threads, 0, st, a);
  return launched("slot_diffusion");
}

template <template <typename> class F, typename A>
murm_status dispatch(int dtype, const A& a, cudaStream_t st) {
  switch (dtype) {
    case MURM_F32: return F<float>::run(a, st);
    case MURM_F16: return F<__half>::run(a, st);
    case MURM_BF16: return F<__nv_bfloat16>::run(a, st);
  }
  return bad(MURM_ERR_DTYPE, "unsupported dtype code %d", dtype);
}
template <typename T> struct SaFwd { static murm_status run(const murm_select_attend_args& a, cudaStream_t s) { return sa_fwd<T>(a, s); } };
template <typename T> struct SaBwd { static murm_status run(const murm_select_attend_bwd_args& a, cudaStream_t s) { return sa_bwd<T>(a, s); } };
template <typename T> struct UpFwd { static murm_status run(const murm_slot_update_args& a, cudaStream_t s) { return upd_fwd<T>(a, s); } };
template <typename T> struct UpBwd { static murm_status run(const murm_slot_update_bwd_args& a, cudaStream_t s) { return upd_bwd<T>(a, s); } };

#define PH_REQUIRE(ptr, name) \
  if (!(ptr)) return ::murm::ph::bad(MURM_ERR_INVALID_ARGUMENT, "%s is NULL", name)

}  // namespace ph
}  // namespace murm

using namespace murm;

extern "C" {

MURM_API murm_status murm_phase_sizes(const murm_phase_shape* shape, size_t* update_saved_bytes,
                                      size_t* workspace_bytes) {
  if (!shape) return ph::bad(MURM_ERR_INVALID_ARGUMENT, "shape is NULL");
  if (murm_status s = ph::check(*shape)) return s;
  const ph::Sizes z = ph::sizes(*shape);
  if (update_saved_bytes) *update_saved_bytes = z.saved;
  if (workspace_bytes) *workspace_bytes = z.ws;
  return MURM_OK;
}

MURM_API murm_status murm_select_attend_fwd(const murm_select_attend_args* a, void* stream) {
  if (!a) return ph::bad(MURM_ERR_INVALID_ARGUMENT, "args is NULL");
  if (murm_status s = ph::check(a->shape)) return s;
  PH_REQUIRE(a->q, "q");
  PH_REQUIRE(a->slot_keys, "slot_keys");
  PH_REQUIRE(a->slot_values, "slot_values");
  PH_REQUIRE(a->out, "out");
  PH_REQUIRE(a->indices, "indices");
  PH_REQUIRE(a->weights, "weights");
  if (!std::isfinite(a->scale)) return ph::bad(MURM_ERR_INVALID_ARGUMENT, "scale must be finite");
  return ph::dispatch<ph::SaFwd>(a->shape.dtype, *a, static_cast<cudaStream_t>(stream));
}

MURM_API murm_status murm_select_attend_bwd(const murm_select_attend_bwd_args* a, void* stream) {
  if (!a) return ph::bad(MURM_ERR_INVALID_ARGUMENT, "args is NULL");
  if (murm_status s = ph::check(a->shape)) return s;
  PH_REQUIRE(a->q, "q");
  PH_REQUIRE(a->slot_keys, "slot_keys");
  PH_REQUIRE(a->slot_values, "slot_values");
  PH_REQUIRE(a->indices, "indices");
  PH_REQUIRE(a->weights, "weights");
  PH_REQUIRE(a->grad_out, "grad_out");
  PH_REQUIRE(a->grad_q, "grad_q");
  PH_REQUIRE(a->grad_slot_keys, "grad_slot_keys");
  PH_REQUIRE(a->grad_slot_values, "grad_slot_values");
  if (murm_status s = ph::ws_ok(a->shape, a->workspace, a->workspace_bytes)) return s;
  return ph::dispatch<ph::SaBwd>(a->shape.dtype, *a, static_cast<cudaStream_t>(stream));
}

MURM_API murm_status murm_slot_update_fwd(const murm_slot_update_args* a, void* stream) {
  if (!a) return ph::bad(MURM_ERR_INVALID_ARGUMENT, "args is NULL");
  if (murm_status s = ph::check(a->shape)) return s;
  PH_REQUIRE(a->token_keys, "token_keys");
  PH_REQUIRE(a->token_values, "token_values");
  PH_REQUIRE(a->slot_keys, "slot_keys");
  PH_REQUIRE(a->slot_values, "slot_values");
  PH_REQUIRE(a->indices, "indices");
  PH_REQUIRE(a->weights, "weights");
  PH_REQUIRE(a->new_slot_keys, "new_slot_keys");
  PH_REQUIRE(a->new_slot_values, "new_slot_values");
  if (!a->saved || a->saved_bytes < ph::sizes(a->shape).saved || (reinterpret_cast<uintptr_t>(a->saved) & 255))
    return ph::bad(MURM_ERR_WORKSPACE, "saved NULL, unaligned or smaller than %zu bytes", ph::sizes(a->shape).saved);
  if (murm_status s = ph::ws_ok(a->shape, a->workspace, a->workspace_bytes)) return s;
  if (!std::isfinite(a->alpha)) return ph::bad(MURM_ERR_INVALID_ARGUMENT, "alpha must be finite");
  return ph::dispatch<ph::UpFwd>(a->shape.dtype, *a, static_cast<cudaStream_t>(stream));
}

MURM_API murm_status murm_slot_update_bwd(const murm_slot_update_bwd_args* a, void* stream) {
  if (!a) return ph::bad(MURM_ERR_INVALID_ARGUMENT, "args is NULL");
  if (murm_status s = ph::check(a->shape)) return s;
  PH_REQUIRE(a->token_keys, "token_keys");
  PH_REQUIRE(a->token_values, "token_values");
  PH_REQUIRE(a->indices, "indices");
  PH_REQUIRE(a->weights, "weights");
  PH_REQUIRE(a->grad_new_keys, "grad_new_keys");
  PH_REQUIRE(a->grad_new_values, "grad_new_values");
  PH_REQUIRE(a->grad_token_keys, "grad_token_keys");
  PH_REQUIRE(a->grad_token_values, "grad_token_values");
  PH_REQUIRE(a->grad_slot_keys, "grad_slot_keys");
  PH_REQUIRE(a->grad_slot_values, "grad_slot_values");
  PH_REQUIRE(a->grad_weights, "grad_weights");
  if (!a->saved || a->saved_bytes < ph::sizes(a->shape).saved)
    return ph::bad(MURM_ERR_WORKSPACE, "saved NULL or smaller than %zu bytes", ph::sizes(a->shape).saved);
  if (murm_status s = ph::ws_ok(a->shape, a->workspace, a->workspace_bytes)) return s;
  return ph::dispatch<ph::UpBwd>(a->shape.dtype, *a, static_cast<cudaStream_t>(stream));
}

MURM_API murm_status murm_slot_sums_fwd(const murm_slot_sums_args* a, void* stream) {
  if (!a) return ph::bad(MURM_ERR_INVALID_ARGUMENT, "args is NULL");
  if (murm_status s = ph::check(a->shape)) return s;
  PH_REQUIRE(a->token_keys, "token_keys");
  PH_REQUIRE(a->token_values, "token_values");
  PH_REQUIRE(a->indices, "indices");
  PH_REQUIRE(a->weights, "weights");
  PH_REQUIRE(a->key_sums, "key_sums");
  PH_REQUIRE(a->value_sums, "value_sums");
  PH_REQUIRE(a->weight_sums, "weight_sums");
  if (murm_status s = ph::ws_ok(a->shape, a->workspace, a->workspace_bytes)) return s;
  return ph::dispatch<ph::SumFwd>(a->shape.dtype, *a, static_cast<cudaStream_t>(stream));
}

MURM_API murm_status murm_slot_sums_bwd(const murm_slot_sums_bwd_args* a, void* stream) {
  if (!a) return ph::bad(MURM_ERR_INVALID_ARGUMENT, "args is NULL");
  if (murm_status s = ph::check(a->shape)) return s;
  PH_REQUIRE(a->token_keys, "token_keys");
  PH_REQUIRE(a->token_values, "token_values");
  PH_REQUIRE(a->indices, "indices");
  PH_REQUIRE(a->weights, "weights");
  PH_REQUIRE(a->grad_key_sums, "grad_key_sums");
  PH_REQUIRE(a->grad_value_sums, "grad_value_sums");
  PH_REQUIRE(a->grad_weight_sums, "grad_weight_sums");
  PH_REQUIRE(a->grad_token_keys, "grad_token_keys");
  PH_REQUIRE(a->grad_token_values, "grad_token_values");
  PH_REQUIRE(a->grad_weights, "grad_weights");
  return ph::dispatch<ph::SumBwd>(a->shape.dtype, *a, static_cast<cudaStream_t>(stream));
}

static murm_status diffusion(const murm_slot_diffusion_args* a, bool backward, void* stream) {
  if (!a) return ph::bad(MURM_ERR_INVALID_ARGUMENT, "args is NULL");
  murm_phase_shape s = a->shape;
  s.tokens = 1;
  if (murm_status e = ph::check(s)) return e;
  PH_REQUIRE(a->in_keys, "in_keys");
  PH_REQUIRE(a->in_values, "in_values");
  PH_REQUIRE(a->out_keys, "out_keys");
  PH_REQUIRE(a->out_values, "out_values");
  if (!std::isfinite(a->gamma)) return ph::bad(MURM_ERR_INVALID_ARGUMENT, "gamma must be finite");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (a->shape.dtype) {
    case MURM_F32: return ph::diff<float>(*a, backward, st);
    case MURM_F16: return ph::diff<__half>(*a, backward, st);
    case MURM_BF16: return ph::diff<__nv_bfloat16>(*a, backward, st);
  }
  return ph::bad(MURM_ERR_DTYPE, "unsupported dtype code %d", a->shape.dtype);
}

MURM_API murm_status murm_slot_diffusion_fwd(const murm_slot_diffusion_args* a, void* stream) {
  return diffusion(a, false, stream);
}
MURM_API murm_status murm_slot_diffusion_bwd(const murm_slot_diffusion_args* a, void* stream) {
  return diffusion(a, true, stream);
}

MURM_API murm_status murm_decode_step(const murm_decode_args* a, void* stream) {
  if (!a) return ph::bad(MURM_ERR_INVALID_ARGUMENT, "args is NULL");
  murm_phase_shape s{a->batch, a->heads, 1, a->slots, a->head_dim, a->dtype};
  if (murm_status e = ph::check(s)) return e;
  const size_t smem = (size_t)a->slots * (a->head_dim + 1) * 8 + (size_t)a->head_dim * 12 + (size_t)a->slots * 4 + 64;
  if (smem > ph::kMaxStage)
    return ph::bad(MURM_ERR_UNSUPPORTED, "decode pool too large for shared memory (%d slots x %d)", a->slots,
                   a->head_dim);
  PH_REQUIRE(a->q, "q");
  PH_REQUIRE(a->k, "k");
  PH_REQUIRE(a->v, "v");
  PH_REQUIRE(a->out, "out");
  PH_REQUIRE(a->slot_keys, "slot_keys");
  PH_REQUIRE(a->slot_values, "slot_values");
  if (a->causal) PH_REQUIRE(a->positions, "positions");
  if (!std::isfinite(a->alpha) || !std::isfinite(a->gamma) || !std::isfinite(a->scale))
    return ph::bad(MURM_ERR_INVALID_ARGUMENT, "alpha, gamma and scale must be finite");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // 16-byte pool accesses when every pool row starts on a 16-byte boundary
  const size_t es = a->dtype == MURM_F32 ? 4 : 2;
  bool vec = ((size_t)a->head_dim * es) % 16 == 0 && (reinterpret_cast<uintptr_t>(a->slot_keys) & 15) == 0 &&
             (reinterpret_cast<uintptr_t>(a->slot_values) & 15) == 0;
  for (int i = 0; i < 3; ++i) vec = vec && (a->sk_stride[i] * (int64_t)es) % 16 == 0 && (a->sv_stride[i] * (int64_t)es) % 16 == 0;
  const size_t smem_v = (size_t)a->slots * a->head_dim * es * 2 + (size_t)a->head_dim * 12 + (size_t)a->slots * 4 + 64;
  auto go = [&](auto kern, size_t bytes) {
    smem_opt_in(kern, bytes);
    MURM_LAUNCH("decode_step", kern, dim3(a->batch * a->heads), 256, bytes, st, *a);
    return ph::launched("decode step");
  };
  switch (a->dtype) {
    case MURM_F32: return vec ? go(ph::k_decode_v<float>, smem_v) : go(ph::k_decode<float>, smem);
    case MURM_F16: return vec ? go(ph::k_decode_v<__half>, smem_v) : go(ph::k_decode<__half>, smem);
    case MURM_BF16: return vec ? go(ph::k_decode_v<__nv_bfloat16>, smem_v) : go(ph::k_decode<__nv_bfloat16>, smem);
  }
  return ph::bad(MURM_ERR_DTYPE, "unsupported dtype code %d", a->dtype);
}

}  // extern "C"
