// murm_common.cuh — shared definitions for the slot_murmurate kernels.
//
// Numerics follow the reference's fp32 CPU path (src/murmurative/reference.py):
// every slot-state quantity is fp32, and the EMA / diffusion arithmetic uses
// explicitly rounded operations in the order reference.py evaluates them, so
// no fused multiply-add changes a rounding there.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/murm.h"

namespace murm {

constexpr int kTopK = MURM_TOP_K;  // reference.py:38 hard-codes k = 7
constexpr int kMaxSlots = 256;     // indices are stored as one byte per pick
constexpr float kEmaEps = 1e-8f;   // reference.py:106-107
constexpr int kTile = 128;         // tokens per tile (one thread or TMEM lane each)
constexpr int kBwdTile = 64;       // tokens per tile of the tensor-core backward token kernel
constexpr int kSlotRows = 16;              // slot rows per block of the slot-side kernels
constexpr int kSlotHalo = kSlotRows + 2;   // plus one diffusion halo row on each side: a warp each
constexpr int kSlotBlocks = 256 / kSlotRows;  // covers the 256 padded slot rows of the operand images

// ---------------------------------------------------------------------------
// Element types
// ---------------------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float load(const float* p) { return *p; }
  static __device__ __forceinline__ void store(float* p, float v) { *p = v; }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float load(const __half* p) { return __half2float(*p); }
  static __device__ __forceinline__ void store(__half* p, float v) { *p = __float2half_rn(v); }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float load(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
};

// Order-preserving map of an fp32 score onto uint32. 0 means "empty" and is
// below every real key, including -inf (0x007FFFFF); NaN ranks above +inf as in
// torch.topk. Equal scores give equal keys; the selection keeps the earlier
// (lower) slot index on equal keys.
__device__ __forceinline__ uint32_t rank_key(float x) {
  uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
constexpr uint32_t kNegInfKey = 0x007FFFFFu;

// Sorted (descending) top-7 list. Insert only when key > k[6].
struct Top7 {
  uint32_t k[kTopK];
  int i[kTopK];
  __device__ __forceinline__ void init() {
#pragma unroll
    for (int j = 0; j < kTopK; ++j) { k[j] = 0u; i[j] = 0; }
  }
  __device__ __forceinline__ void insert(uint32_t key, int idx) {
    bool done = false;
#pragma unroll
    for (int j = kTopK - 1; j > 0; --j) {
      const bool shift = !done && key > k[j - 1];
      const bool place = !done && !shift;
      k[j] = shift ? k[j - 1] : (place ? key : k[j]);
      i[j] = shift ? i[j - 1] : (place ? idx : i[j]);
      done = done || place;
    }
    if (!done) { k[0] = key; i[0] = idx; }
  }
  __device__ __forceinline__ void offer(uint32_t key, int idx) {
    if (key > k[kTopK - 1]) insert(key, idx);
  }
};

// ---------------------------------------------------------------------------
// Problem description shared by host and device
// ---------------------------------------------------------------------------
struct Geom {
  int B, H, N, M, D, R, causal, dtype;
  int BH;
  float alpha, one_minus_alpha, gamma, scale;
  // token chunks: chunk c covers tokens [c*chunk_tokens, min(N, (c+1)*chunk_tokens))
  int red_chunks, red_chunk_tokens;   // CUDA-core path's reduction kernels (many tiles per CTA)
  int bwd_chunks, bwd_chunk_tokens;   // tensor-core backward token kernel (64-token tiles)
  int ft_parts;                       // tensor-core forward: slot-sum partials per (b,h) (TileSplit)
};

// The tensor-core forward's split of the flat list of (b,h) x token tiles ("units": unit u is
// tile u % tpb of pair u / tpb) over at most one CTA per SM. CTA c takes units
// [start[c], start[c+1]): a run that may finish one pair and start the next. A change of pair
// costs a CTA a pipeline drain and refill and new operand images, about one tile, so the host
// plan charges it as one: each CTA gets at most K tiles, or K - 1 when its run changes pair once,
// with the smallest K whose plan fits in the SMs. Each pair gets one slot-sum partial per CTA
// that covers some of its tiles, numbered from 0 in token order.
constexpr int kMaxSplitCtas = 148;
struct TileSplit {
  int G;    // CTAs
  int tpb;  // tiles per (b,h)
  int start[kMaxSplitCtas + 1];
  __host__ __device__ int cta_of(int u) const {  // the CTA whose run holds unit u
    int lo = 0, hi = G - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (start[mid] <= u) lo = mid;
      else hi = mid - 1;
    }
    return lo;
  }
  __host__ __device__ int first_cta(int bh) const { return cta_of(bh * tpb); }
  __host__ __device__ int parts(int bh) const { return cta_of(bh * tpb + tpb - 1) - first_cta(bh) + 1; }
};
// Host: the plan for BH pairs of N tokens in tiles of `tile` tokens over at most `sms` CTAs
// (sms <= kMaxSplitCtas).
inline void plan_split(int BH, int N, int tile, int sms, TileSplit* s) {
  const int tpb = (N + tile - 1) / tile;
  const int U = BH * tpb;  // B*H*N*D < 2^31 is checked, so this fits
  const int pen = 1;       // tiles charged for a change of pair
  for (int K = (U + sms - 1) / sms;; ++K) {
    int c = 0, u = 0;
    while (u < U && c < sms) {
      s->start[c++] = u;
      int b = K;
      const int rest = (u / tpb + 1) * tpb - u;  // tiles left in this pair
      const int t = rest < b ? rest : b;
      u += t;
      b -= t;
      if (b > pen && u < U) {  // at a pair boundary with budget left: whole pairs, then part of one
        int k = b / (pen + tpb);
        if (k > (U - u) / tpb) k = (U - u) / tpb;
        u += k * tpb;
        b -= k * (pen + tpb);
        if (u < U && b > pen) u += b - pen;  // b - pen < tpb tiles of the next pair
      }
    }
    if (u >= U) {
      s->G = c;
      s->tpb = tpb;
      s->start[c] = U;
      return;
    }
  }
}
// A bound on the partials of any pair under a plan: the CTAs whose runs start in the pair, plus
// one whose run started in an earlier pair and reaches into it (counted over the G CTAs, not the
// pairs, of which there may be many).
inline int max_parts(const TileSplit& s) {
  int m = 1, bh_prev = -1, count = 0;
  for (int c = 0; c < s.G; ++c) {
    const int bh = s.start[c] / s.tpb;
    count = (bh == bh_prev) ? count + 1 : 1;
    bh_prev = bh;
    m = count > m ? count : m;
  }
  return m + 1;
}

// Round records kept from forward to backward and scratch areas. All fp32
// slot tensors are [BH][M][D] row-major; token tensors [BH][N][...].
struct Saved {
  float* K;      // [R][BH][M][D] slot keys entering round r
  float* V;      // [R][BH][M][D] slot values entering round r
  float* U;      // [R][BH][M][D] update means ksum/(wsum+eps) of round r
  float* W;      // [R][BH][M]    weight sums of round r
  uint8_t* idx;  // [R][BH][N][8] selected slots (7 used)
  float* w;      // [R][BH][N][8] softmax weights (7 used)
};
constexpr int kAmaxBlocks = 32;  // blocks per (b,h) pair of the forward's maxima pass (bf16 tensor-core path)
struct FwdScratch {
  float* Spart;     // CUDA-core path: [BH][red_chunks][M][D]; tensor-core path: [BH][ft_parts][D/4][M][4]
                    // (4-column chunks, slot rows contiguous: coalesced stores from the TMEM lanes)
  float* Wpart;     // [BH][parts][M]
  uint8_t* images;  // [BH][3][256][64] 16-bit operand images (tensor-core path)
  int* counters;    // [2][BH] partials written / finalize shares done (multi-round tensor-core launch)
  float* amax;      // [BH][kAmaxBlocks][3] bf16 tensor-core path: block maxima of |q|, |slots_k|, |slots_v|
  int* fexp;        // [BH][4] the pair's operand-scale exponents (q, keys, values; 0 for fp16)
};
struct BwdScratch {
  float* dK[2];  // [BH][M][D] ping-pong slot-key gradients
  float* dV[2];
  float* dS;     // [BH][M][D] gradient w.r.t. the update sum
  float* dW;     // [BH][M]    gradient w.r.t. the weight sum
  float* dKdir;  // [BH][M][D] direct (EMA-kept) part of dK
  float* dVdir;
  float* dKpart; // CUDA-core path: [BH][red_chunks][M][D]; tensor-core path: [BH][bwd_chunks][D/4][M][4]
  float* dVpart;
  float* coef;   // [BH][N][8] scale * dlogit per pick
  float* dq;     // [BH][N][D] running dL/dq over rounds
  uint8_t* tables;  // [BH][3][256][64] 16-bit K, V, dS of a round + [BH][256] fp32 dW (tensor-core path)
  float* amax;      // [BH][64] bf16 tensor-core path: block maxima of |q| (0..31) and |grad_out| (32..63)
};

}  // namespace murm
