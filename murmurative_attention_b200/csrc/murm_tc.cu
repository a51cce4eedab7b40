// murm_tc.cu — tensor-core (tcgen05/TMEM/TMA) forward round for fp16/bf16, head_dim 64.
//
// One CTA owns one (batch, head) and a chunk of 128-token tiles. Per tile:
//   1. select  (reference.py:19-38): S = Q . [K_1; ...; K_s]^T on tcgen05 into a
//      128 x 256 fp32 TMEM tile. The fp32 slot keys are split into s 16-bit
//      terms (K = K_1 + K_2 (+ K_3) + O(2^-22..2^-24 |K|): two fp16 terms, three
//      bf16 terms), so the scores carry fp32-level precision; the N x M scores
//      never leave the SM.
//   2. top-7 per token, exact, ties to the lowest slot (thread = TMEM lane =
//      token): a group-max pass bounds the 7th score from below, the few
//      scores above the bound are compacted to shared memory and ranked
//      exactly; rows where the bound is not finite take an exact full scan.
//   3. softmax over the 7 picks (reference.py:61-63) in fp32.
//   4. the picks' weights w are written into a zeroed 128 x 256 tile P in shared
//      memory as two 16-bit terms, first w_hi = rn(w) and then w_lo = rn(w - w_hi):
//      tcgen05 computes the attend output O = P_hi . V (reference.py:65-66) and
//      accumulates the slot update sums S += P^T . Q and W += P^T . 1
//      (reference.py:93-103) over both terms in TMEM across all tiles of the
//      chunk — fp32-level sums, deterministic, no atomics.
// The chunk's S/W partials go to global memory; k_update_finalize (murm_simt.cu)
// combines chunks in index order, applies the EMA and the diffusion.
//
// Shared memory (from a 1024-byte aligned base; operand tiles use the 128-byte
// swizzle, rows of 64 16-bit elements):
//   K terms (32K each) | V 32K | P 64K (4 slot blocks) | Q tiles (16K each) | ONES 1K | CAND | misc
//   fp16: 2 key terms, 2 Q buffers (prefetch), 24 candidates per row
//   bf16: 3 key terms, 1 Q buffer, 16 candidates per row
#include <cstdlib>
#include <cudaTypedefs.h>

#include "murm_kernels.cuh"
#include "murm_sm100.cuh"

namespace murm {
using namespace sm100;

__device__ int g_device_error;  // set by a bounded wait that expired; read by murm_device_status

namespace tc {
constexpr int kD = 64;
constexpr int kSlotsPad = 256;
constexpr uint32_t kImg = kSlotsPad * 128;  // one [256][64] 16-bit operand image
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t COL_S = 0, COL_O = 0, COL_U = 256, COL_W = 384;
constexpr uint32_t kQBytes = 128 * 128;

enum : int { kErrImgWait = 1, kErrQWait = 2, kErrMmaWait = 4 };

template <typename T> struct Cfg;
template <> struct Cfg<__half> {
  static constexpr uint32_t fmt = 0;
  static constexpr int kSplits = 2, kQBufs = 2, kCand = 24;
  static __device__ __forceinline__ uint16_t one() { return 0x3C00u; }
};
template <> struct Cfg<__nv_bfloat16> {
  static constexpr uint32_t fmt = 1;
  static constexpr int kSplits = 3, kQBufs = 1, kCand = 16;
  static __device__ __forceinline__ uint16_t one() { return 0x3F80u; }
};
template <typename T> struct Layout {
  static constexpr uint32_t kImages = (Cfg<T>::kSplits + 1) * kImg;  // key terms + V
  static constexpr uint32_t OFF_V = Cfg<T>::kSplits * kImg;
  static constexpr uint32_t OFF_P = OFF_V + kImg;
  static constexpr uint32_t OFF_Q = OFF_P + 4 * 16384;
  static constexpr uint32_t OFF_ONES = OFF_Q + Cfg<T>::kQBufs * kQBytes;
  static constexpr uint32_t OFF_CAND = OFF_ONES + 1024;
  static constexpr uint32_t OFF_MISC = OFF_CAND + kTile * Cfg<T>::kCand * 8;
  static constexpr uint32_t kSmem = OFF_MISC + 128 + 1024;  // + alignment slack
  static_assert(kSmem <= 232448, "shared memory budget");
};

__device__ __forceinline__ bool timed_wait(uint64_t* bar, uint32_t parity) {
  // About one second of polling, measured on the global timer.
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 256; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    uint64_t t1;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t1));
    if (t1 - t0 > 1000000000ull) return false;
  }
}

template <typename T>
__device__ __forceinline__ uint16_t to_bits(float x) {
  T h;
  Elem<T>::store(&h, x);
  return *reinterpret_cast<uint16_t*>(&h);
}
template <typename T>
__device__ __forceinline__ float from_bits(uint16_t b) {
  return Elem<T>::load(reinterpret_cast<const T*>(&b));
}

}  // namespace tc

// ---------------------------------------------------------------------------
// Operand images of one round, laid out exactly as the kernel's shared-memory
// tiles (swizzled rows of 128 B): the key terms K_1..K_s and V in the dtype.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) k_tc_images(Geom g, int r, Saved sv, uint8_t* images) {
  constexpr int S = tc::Cfg<T>::kSplits;
  const int bh = blockIdx.x, m = threadIdx.x;
  const size_t st = ((size_t)r * g.BH + bh) * g.M * tc::kD;
  uint8_t* base = images + (size_t)bh * tc::Layout<T>::kImages;
  for (int c = 0; c < tc::kD; ++c) {
    float k = 0.f, v = 0.f;
    if (m < g.M) {
      k = sv.K[st + (size_t)m * tc::kD + c];
      v = sv.V[st + (size_t)m * tc::kD + c];
    }
    const uint32_t off = sm100::sw128_offset(m, c);
#pragma unroll
    for (int s = 0; s < S; ++s) {
      T term;
      Elem<T>::store(&term, k);
      *reinterpret_cast<T*>(base + s * tc::kImg + off) = term;
      k -= Elem<T>::load(&term);  // exact in fp32: the next term carries the residual
    }
    T vv;
    Elem<T>::store(&vv, v);
    *reinterpret_cast<T*>(base + tc::Layout<T>::OFF_V + off) = vv;
  }
}

// ---------------------------------------------------------------------------
// The forward round kernel
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kTile, 1)
    k_fwd_tc(Geom g, int r, const __grid_constant__ CUtensorMap qmap, T* out, Strides3 os, int64_t* indices,
             float* weights, Saved sv, FwdScratch fs, const uint8_t* images) {
  using C = tc::Cfg<T>;
  using L = tc::Layout<T>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t s_base = smem_u32(sm);
  uint64_t* bar_img = reinterpret_cast<uint64_t*>(sm + L::OFF_MISC);
  uint64_t* bar_q = bar_img + 1;  // [2]
  uint64_t* bar_mma = bar_img + 3;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + L::OFF_MISC + 64);
  volatile int* s_abort = reinterpret_cast<volatile int*>(sm + L::OFF_MISC + 68);
  float2* cand = reinterpret_cast<float2*>(sm + L::OFF_CAND) + threadIdx.x * C::kCand;

  const int tid = threadIdx.x, warp = tid >> 5;
  const int bh = blockIdx.y, b = bh / g.H, h = bh - b * g.H, chunk = blockIdx.x;
  const int t_beg = chunk * g.red_chunk_tokens;
  const int t_end = min(g.N, t_beg + g.red_chunk_tokens);
  const int ntiles = (t_end - t_beg + kTile - 1) / kTile;
  constexpr uint32_t ID_SEL = idesc_f16(C::fmt, 128, 256, 0, 0);
  constexpr uint32_t ID_ATT = idesc_f16(C::fmt, 128, 64, 0, 1);
  constexpr uint32_t ID_UPD = idesc_f16(C::fmt, 128, 64, 1, 1);
  constexpr uint32_t ID_W = idesc_f16(C::fmt, 128, 16, 1, 0);

  // ---- set-up: barriers, zeroed P, ones, TMEM ----
  if (tid == 0) {
    mbar_init(bar_img, 1);
    mbar_init(&bar_q[0], 1);
    mbar_init(&bar_q[1], 1);
    mbar_init(bar_mma, 1);
    *s_abort = 0;
    fence_barrier_init();
  }
  {
    float4* p4 = reinterpret_cast<float4*>(sm + L::OFF_P);
    for (int i = tid; i < 4 * 16384 / 16; i += kTile) p4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    uint16_t* ones = reinterpret_cast<uint16_t*>(sm + L::OFF_ONES);
    for (int i = tid; i < 512; i += kTile) ones[i] = C::one();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, tc::kTmemCols);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;

  // thread 0's bookkeeping of asynchronous copies
  bool img_pending = false, q_pending0 = false, q_pending1 = false;
  uint32_t q_phase0 = 0, q_phase1 = 0, mma_phase = 0;
  auto issue_q = [&](int tile_idx) {  // thread 0 only
    const int bsel = (C::kQBufs == 2) ? (tile_idx & 1) : 0;
    mbar_arrive_expect_tx(&bar_q[bsel], tc::kQBytes);
    tma_load_4d(sm + L::OFF_Q + bsel * tc::kQBytes, &qmap, 0, t_beg + tile_idx * kTile, h, b, &bar_q[bsel]);
    if (bsel) q_pending1 = true; else q_pending0 = true;
  };
  if (tid == 0) {
    mbar_arrive_expect_tx(bar_img, L::kImages);
    bulk_g2s(sm, images + (size_t)bh * L::kImages, L::kImages, bar_img);
    img_pending = true;
    issue_q(0);
  }
  const uint32_t a_v = s_base + L::OFF_V, a_p = s_base + L::OFF_P, a_ones = s_base + L::OFF_ONES;
  const bool last_round = (r == g.R - 1);

  // Wait for the MMA group committed last; on timeout record and abort.
  auto wait_mma = [&]() {
    if (tc::timed_wait(bar_mma, mma_phase)) {
      mma_phase ^= 1;
    } else {
      atomicOr(&g_device_error, tc::kErrMmaWait);
      *s_abort = 1;
    }
    tc_fence_after();
  };
  auto sync_all = [&]() {  // smem writes -> async proxy; TMEM reads done; CTA barrier
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
  };

  for (int tile = 0; tile < ntiles; ++tile) {
    const int buf = (C::kQBufs == 2) ? (tile & 1) : 0;
    const int n0 = t_beg + tile * kTile;
    const int n = n0 + tid;
    const bool valid = n < t_end;
    const uint32_t a_q = s_base + L::OFF_Q + buf * tc::kQBytes;

    // ---- select MMA ----
    if (tid == 0) {
      bool ok = true;
      if (C::kQBufs == 2 && tile + 1 < ntiles) issue_q(tile + 1);  // the other buffer is free
      if (img_pending) {
        ok = tc::timed_wait(bar_img, 0);
        img_pending = !ok;
        if (!ok) atomicOr(&g_device_error, tc::kErrImgWait);
      }
      if (ok) {
        uint32_t& ph = buf ? q_phase1 : q_phase0;
        ok = tc::timed_wait(&bar_q[buf], ph);
        if (ok) {
          ph ^= 1;
          if (buf) q_pending1 = false; else q_pending0 = false;
        } else {
          atomicOr(&g_device_error, tc::kErrQWait);
        }
      }
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int s = 0; s < C::kSplits; ++s)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_f16(tmem + tc::COL_S, smem_desc(a_q + k * 32, 16, 1024, kSwizzle128B),
                    smem_desc(s_base + s * tc::kImg + k * 32, 16, 1024, kSwizzle128B), ID_SEL, (s | k) != 0);
        mma_commit(bar_mma);
      } else {
        *s_abort = 1;
      }
    }
    wait_mma();

    // ---- top-7 of this thread's row ----
    // TMEM loads are warp-collective: every lane executes them; rows past the
    // chunk end (last tile) ignore the values.
    int pick[kTopK];
    float wgt[kTopK];
    const bool aborting = __any_sync(0xffffffffu, *s_abort != 0);  // warp-uniform
    const bool active = valid && !aborting;
    const int lim = g.causal ? min(g.M, n + 1) : g.M;  // columns >= lim score -inf
    if (!aborting) {
      const bool need_mask = __any_sync(0xffffffffu, lim < tc::kSlotsPad);
      float gm[32];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float v[32];
        tmem_ld32(tmem + lane_base + tc::COL_S + 32 * c, v);
        tmem_wait_ld();
        if (need_mask) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = (32 * c + i < lim) ? v[i] : -INFINITY;
        }
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          float x = v[8 * q4];
#pragma unroll
          for (int i = 1; i < 8; ++i) x = fmaxf(x, v[8 * q4 + i]);
          gm[4 * c + q4] = x;
        }
      }
      // 7th largest group maximum: a lower bound of the 7th largest score.
      float t7[kTopK];
#pragma unroll
      for (int j = 0; j < kTopK; ++j) t7[j] = -INFINITY;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        float x = gm[i];
#pragma unroll
        for (int j = 0; j < kTopK; ++j) {
          const float hi = fmaxf(t7[j], x);
          x = fminf(t7[j], x);
          t7[j] = hi;
        }
      }
      const float thr = t7[kTopK - 1];
      const bool bounded = thr > -INFINITY;
      int cnt = 0;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float v[32];
        tmem_ld32(tmem + lane_base + tc::COL_S + 32 * c, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int m = 32 * c + i;
          if (bounded && m < lim && v[i] >= thr) {
            if (cnt < C::kCand) cand[cnt] = make_float2(v[i], __int_as_float(m));
            ++cnt;
          }
        }
      }
      const bool exact_scan = !bounded || cnt > C::kCand;
      Top7 top;
      top.init();
      float masked_raw[kTopK];
#pragma unroll
      for (int j = 0; j < kTopK; ++j) masked_raw[j] = 0.f;
      if (!exact_scan) {
        for (int e = 0; e < cnt; ++e) {  // candidates are in slot order: ties keep the lower slot
          const float2 cd = cand[e];
          top.offer(rank_key(cd.x), __float_as_int(cd.y));
        }
      }
      if (__any_sync(0xffffffffu, exact_scan)) {
        // exact full scan (rows with fewer than 7 finite group maxima, or many ties)
        for (int c = 0; c < 8; ++c) {
          float v[32];
          tmem_ld32(tmem + lane_base + tc::COL_S + 32 * c, v);
          tmem_wait_ld();
          if (exact_scan) {
            for (int i = 0; i < 32; ++i) {
              const int m = 32 * c + i;
              if (m >= g.M) break;
              if (m < lim) {
                top.offer(rank_key(v[i]), m);
              } else {
                if (m - lim < kTopK) masked_raw[m - lim] = v[i];
                top.offer(kNegInfKey, m);
              }
            }
          }
        }
      }
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < kTopK; ++j) {
        pick[j] = top.i[j];
        // masked picks (causal rows n < 6) attend with their real score (reference.py:61)
        const uint32_t kk = top.k[j];
        const float s = (pick[j] < lim) ? __uint_as_float((kk & 0x80000000u) ? (kk & 0x7FFFFFFFu) : ~kk)
                                        : masked_raw[min(max(pick[j] - lim, 0), kTopK - 1)];
        wgt[j] = s * g.scale;
        mx = fmaxf(mx, wgt[j]);
      }
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < kTopK; ++j) {
        wgt[j] = expf(wgt[j] - mx);
        sum += wgt[j];
      }
#pragma unroll
      for (int j = 0; j < kTopK; ++j) wgt[j] = wgt[j] / sum;
    }
    uint16_t w_lo_bits[kTopK];
    if (active) {
      // P row (first term), round records, last-round outputs
#pragma unroll
      for (int j = 0; j < kTopK; ++j) {
        const uint16_t hb = tc::to_bits<T>(wgt[j]);
        w_lo_bits[j] = tc::to_bits<T>(wgt[j] - tc::from_bits<T>(hb));
        *reinterpret_cast<uint16_t*>(sm + L::OFF_P + (pick[j] >> 6) * 16384 + sw128_offset(tid, pick[j] & 63)) = hb;
      }
      const size_t trow = ((size_t)r * g.BH + bh) * g.N + n;
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) lo |= (uint32_t)pick[j] << (8 * j);
#pragma unroll
      for (int j = 4; j < kTopK; ++j) hi |= (uint32_t)pick[j] << (8 * (j - 4));
      reinterpret_cast<uint2*>(sv.idx)[trow] = make_uint2(lo, hi);
      float4* wrow = reinterpret_cast<float4*>(sv.w + trow * 8);
      wrow[0] = make_float4(wgt[0], wgt[1], wgt[2], wgt[3]);
      wrow[1] = make_float4(wgt[4], wgt[5], wgt[6], 0.f);
      if (last_round) {
        const size_t o7 = ((size_t)bh * g.N + n) * kTopK;
        if (indices) {
#pragma unroll
          for (int j = 0; j < kTopK; ++j) indices[o7 + j] = pick[j];
        }
        if (weights) {
#pragma unroll
          for (int j = 0; j < kTopK; ++j) weights[o7 + j] = wgt[j];
        }
      }
    }
    sync_all();
    if (*s_abort) break;

    // ---- MMAs with the first weight term: O = P.V, S += P^T.Q, W += P^T.1 ----
    auto issue_update = [&](bool first) {  // thread 0
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t a = smem_desc(a_p + 2 * hh * 16384 + kk * 2048, 16384, 1024, kSwizzle128B);
          const uint32_t acc = (first && kk == 0) ? 0u : 1u;
          mma_f16(tmem + tc::COL_U + 64 * hh, a, smem_desc(a_q + kk * 2048, 16384, 1024, kSwizzle128B), ID_UPD,
                  acc);
          mma_f16(tmem + tc::COL_W + 16 * hh, a, smem_desc(a_ones, 256, 128, kSwizzleNone), ID_W, acc);
        }
      }
    };
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < 16; ++kk)
        mma_f16(tmem + tc::COL_O, smem_desc(a_p + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024, kSwizzle128B),
                smem_desc(a_v + kk * 2048, 16384, 1024, kSwizzle128B), ID_ATT, kk != 0);
      issue_update(tile == 0);
      mma_commit(bar_mma);
    }
    wait_mma();
    // second weight term: overwrite this row's entries of P
    if (active) {
#pragma unroll
      for (int j = 0; j < kTopK; ++j)
        *reinterpret_cast<uint16_t*>(sm + L::OFF_P + (pick[j] >> 6) * 16384 + sw128_offset(tid, pick[j] & 63)) =
            w_lo_bits[j];
    }
    sync_all();
    if (*s_abort) break;
    if (tid == 0) {
      tc_fence_after();
      issue_update(false);
      mma_commit(bar_mma);
    }

    // ---- output (overlaps the second update group): out (+)= O ----
    if (!__any_sync(0xffffffffu, *s_abort != 0)) {
      T* orow = row_ptr(out, os, b, h, valid ? n : n0);
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float o[32];
        tmem_ld32(tmem + lane_base + tc::COL_O + 32 * c, o);
        tmem_wait_ld();
        if (valid) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 pk;
            uint16_t* ph = reinterpret_cast<uint16_t*>(&pk);
            if (r) {
              const uint4 prev = *reinterpret_cast<const uint4*>(orow + 32 * c + i);
              const T* pv = reinterpret_cast<const T*>(&prev);
#pragma unroll
              for (int e = 0; e < 8; ++e) ph[e] = tc::to_bits<T>(Elem<T>::load(pv + e) + o[i + e]);
            } else {
#pragma unroll
              for (int e = 0; e < 8; ++e) ph[e] = tc::to_bits<T>(o[i + e]);
            }
            *reinterpret_cast<uint4*>(orow + 32 * c + i) = pk;
          }
        }
      }
    }
    wait_mma();
    if (tid == 0 && C::kQBufs == 1 && tile + 1 < ntiles && !*s_abort) issue_q(tile + 1);  // Q is free now
    if (active) {  // clear this row of P for the next tile
#pragma unroll
      for (int j = 0; j < kTopK; ++j)
        *reinterpret_cast<uint16_t*>(sm + L::OFF_P + (pick[j] >> 6) * 16384 + sw128_offset(tid, pick[j] & 63)) = 0;
    }
    sync_all();
    if (*s_abort) break;
  }

  // ---- chunk partials: TMEM lanes are slots here ----
  if (!__any_sync(0xffffffffu, *s_abort != 0)) {
    const size_t po = (size_t)bh * g.red_chunks + chunk;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int m = 128 * hh + tid;
      float s0[32], s1[32], wv[16];
      tmem_ld32(tmem + lane_base + tc::COL_U + 64 * hh, s0);
      tmem_ld32(tmem + lane_base + tc::COL_U + 64 * hh + 32, s1);
      tmem_ld16(tmem + lane_base + tc::COL_W + 16 * hh, wv);
      tmem_wait_ld();
      if (m < g.M) {
        float4* dst = reinterpret_cast<float4*>(fs.Spart + (po * g.M + m) * tc::kD);
#pragma unroll
        for (int i = 0; i < 8; ++i) dst[i] = make_float4(s0[4 * i], s0[4 * i + 1], s0[4 * i + 2], s0[4 * i + 3]);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          dst[8 + i] = make_float4(s1[4 * i], s1[4 * i + 1], s1[4 * i + 2], s1[4 * i + 3]);
        fs.Wpart[po * g.M + m] = wv[0];
      }
    }
  }
  // ---- wind down: wait (bounded) for copies still in flight, free TMEM ----
  if (tid == 0) {
    if (img_pending) tc::timed_wait(bar_img, 0);
    if (q_pending0) tc::timed_wait(&bar_q[0], q_phase0);
    if (q_pending1) tc::timed_wait(&bar_q[1], q_phase1);
    if (*s_abort) tc::timed_wait(bar_mma, mma_phase);  // an MMA group whose completion was not seen
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, tc::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {
PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}
}  // namespace

size_t tc_images_bytes(const Geom& g) {
  if (g.D != tc::kD) return 0;
  if (g.dtype == MURM_F16) return (size_t)g.BH * tc::Layout<__half>::kImages;
  if (g.dtype == MURM_BF16) return (size_t)g.BH * tc::Layout<__nv_bfloat16>::kImages;
  return 0;
}

bool tc_forward_supported(const Geom& g, int dtype, const FwdPtrs& p) {
  if (dtype != MURM_F16 && dtype != MURM_BF16) return false;
  if (g.D != tc::kD || g.R < 1) return false;
  for (int i = 0; i < 3; ++i)  // TMA strides and 16-byte output rows
    if ((p.qs.s[i] % 8) || (p.os.s[i] % 8)) return false;
  if ((reinterpret_cast<uintptr_t>(p.q) | reinterpret_cast<uintptr_t>(p.out)) & 15) return false;
  const char* force = getenv("MURM_FORCE_SIMT");
  return !(force && force[0] == '1');
}

cudaError_t read_and_clear_device_error(int* code, cudaStream_t st) {
  cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return e;
  e = cudaMemcpyFromSymbol(code, g_device_error, sizeof(int));
  if (e != cudaSuccess) return e;
  if (*code) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
  }
  return e;
}

template <typename T>
cudaError_t fwd_tc(const Geom& g, const FwdPtrs& p, const Saved& sv, const FwdScratch& fs, cudaStream_t st) {
  uint8_t* images = fs.images;
  auto encode = get_encode();
  if (!encode) return cudaErrorNotSupported;
  CUtensorMap qmap;
  const cuuint64_t esz = sizeof(T);
  cuuint64_t dims[4] = {(cuuint64_t)g.D, (cuuint64_t)g.N, (cuuint64_t)g.H, (cuuint64_t)g.B};
  cuuint64_t strides[3] = {(cuuint64_t)p.qs.s[2] * esz, (cuuint64_t)p.qs.s[1] * esz,
                           (cuuint64_t)(p.qs.s[0] ? p.qs.s[0] : 1) * esz};
  cuuint32_t box[4] = {64, 128, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt =
      tc::Cfg<T>::fmt == 1 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult cr = encode(&qmap, dt, 4, const_cast<void*>(p.q), dims, strides, box, estr,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return cudaErrorInvalidValue;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k_fwd_tc<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc::Layout<T>::kSmem);
    attr = true;
  }
  launch_load_slots<T>(g, p, sv, st);
  for (int r = 0; r < g.R; ++r) {
    MURM_LAUNCH("tc_images", k_tc_images<T>, g.BH, 256, 0, st, g, r, sv, images);
    MURM_LAUNCH("select_attend_update_tc", k_fwd_tc<T>, dim3(g.red_chunks, g.BH), kTile, tc::Layout<T>::kSmem, st, g, r,
                qmap, static_cast<T*>(p.out), p.os, p.indices, p.weights, sv, fs, images);
    if (r + 1 < g.R) launch_update_finalize(g, r, sv, fs, st);
  }
  return cudaGetLastError();
}

template cudaError_t fwd_tc<__half>(const Geom&, const FwdPtrs&, const Saved&, const FwdScratch&, cudaStream_t);
template cudaError_t fwd_tc<__nv_bfloat16>(const Geom&, const FwdPtrs&, const Saved&, const FwdScratch&,
                                           cudaStream_t);

}  // namespace murm
