// murm_tc.cu — tensor-core (tcgen05/TMEM/TMA) forward rounds for fp16/bf16, head_dim 64.
//
// One CTA per SM; the (batch, head) x 128-token tile list is split over them by
// TileSplit (murm_common.cuh), so a CTA takes a run of tiles that may finish one
// (batch, head) and start the next: one segment per (batch, head), each with its
// own operand images and slot-sum partial. Per tile:
//   1. select  (reference.py:19-38): S = Q . [K_1; ...; K_s]^T on tcgen05 into a
//      128 x 256 fp32 TMEM tile. The fp32 slot keys are split into s 16-bit
//      terms (K = K_1 + K_2 (+ K_3) + O(2^-22..2^-24 |K|): two fp16 terms, three
//      bf16 terms), so the scores carry fp32-level precision; the N x M scores
//      never leave the SM.
//   2. top-7 per token, exact, ties to the lowest slot (two threads per token
//      row, 128 slot columns each): the 7th largest of 32 group maxima (groups
//      of 8 slots at stride 16) bounds the 7th score from below; each thread
//      ranks its few scores above the bound into a 7-entry list (bit masks and
//      select-tree reads of registers), and the two lists are merged through
//      shared memory; rows where the bound is not finite take an exact scan.
//   3. softmax over the 7 picks (reference.py:61-63) in fp32.
//   4. the picks' weights w are written into a zeroed 128 x 256 tile P in shared
//      memory as two 16-bit terms, first w_hi = rn(w) and then w_lo = rn(w - w_hi):
//      tcgen05 computes the attend output O = P_hi . V (reference.py:65-66) and
//      accumulates the slot update sums S += P^T . Q and W += P^T . 1
//      (reference.py:93-103) over both terms in TMEM across all tiles of the
//      segment — fp32-level sums, deterministic, no atomics.
// A segment's S/W partials go to global memory. All R rounds run in one cooperative launch:
// between rounds the CTAs whose runs end in a (batch, head) combine its partials in token
// order, apply the EMA and the diffusion and write the next round's state and operand images,
// and the pair's next round starts once its own finalize is done (two counters per pair, no
// grid-wide barrier); no slot update follows the last round. Without a cooperative launch,
// one launch per round with k_tc_finalize between them does the same arithmetic.
//
// Shared memory (from a 1024-byte aligned base; operand tiles use the 128-byte
// swizzle, rows of 64 16-bit elements):
//   K terms (32K each) | V 32K | P 64K (4 slot blocks) | Q tiles (16K each) | ONES 2K |
//   XCH 14K (the threads' top-7 lists) | misc
//   fp16: 2 key terms, 3 Q buffers; bf16: 3 key terms, 1 Q buffer
#include <cstdlib>
#include <type_traits>
#include <cudaTypedefs.h>

#include "murm_kernels.cuh"
#include "murm_sm100.cuh"

namespace murm {
using namespace sm100;

__device__ int g_device_error;  // set by a bounded wait that expired; read by murm_device_status

namespace tc {
constexpr int kD = 64;
constexpr int kSlotsPad = 256;
constexpr int kRowThreads = 256;                // 8 row warps: 2 per TMEM lane quadrant
constexpr int kEpiWarp = kRowThreads / 32;       // 4 epilogue warps (8..11), one per lane quadrant
constexpr int kEpiThreads = 128;
constexpr int kIssuerWarp = kEpiWarp + 4;        // a fourth warpgroup: warp 12's lane 0 issues MMAs and
constexpr int kThreads = kRowThreads + kEpiThreads + 128;  // copies, warps 13-15 convert bf16 q tiles
// Registers: one allocation for all warps (126 a thread, no spills). No `setmaxnreg` split: ptxas
// ignores it in relocatable device code, and compiled whole, any split that lowers the fourth
// warpgroup (the issuer's code) below ~128 spills.
constexpr int kParts = 2;        // each token row's 256 scores are split over 2 threads
constexpr uint32_t kImg = kSlotsPad * 128;  // one [256][64] 16-bit operand image
constexpr uint32_t kTmemCols = 512;
// TMEM columns: scores | slot sums S and weight sums W (2 halves of 80: 64 S columns, then 16
// columns that each hold W) | group-maxima exchange of a row's two threads | the row's picks and
// scores handed from the row warps to the epilogue warps | attend output O
constexpr uint32_t COL_S = 0, COL_U = 256, COL_X = 416, COL_H = 432, COL_O = 448;
constexpr uint32_t kUW = 80;  // columns per half of the slot-sum accumulator
constexpr uint32_t kQBytes = 128 * 128;

enum : int { kErrImgWait = 1, kErrQWait = 2, kErrMmaWait = 4, kErrPeerWait = 32 };

// Barrier over the warps that share one TMEM lane quadrant.
__device__ __forceinline__ void quadrant_sync(int quadrant) {
  asm volatile("bar.sync %0, %1;" ::"r"(1 + quadrant), "r"(32 * kParts) : "memory");
}
// Named barriers that the issuer warp waits on and the others only arrive at: the tile's first (5)
// and second (6) weight terms are in P (the epilogue warps arrive); the row warps are done reading
// the tile's scores (7).
constexpr int kBarPhi = 5, kBarPlo = 6, kBarSfree = 7;
constexpr int kBarRows = 8, kBarEpi = 9;  // all row warps; all epilogue warps
constexpr int kCountP = kEpiThreads + 32, kCountS = kRowThreads + 32;
template <int kId, int kCount>
__device__ __forceinline__ void issuer_wait() {
  asm volatile("bar.sync %0, %1;" ::"n"(kId), "n"(kCount) : "memory");
}
template <int kId, int kCount>
__device__ __forceinline__ void group_arrive() {
  asm volatile("bar.arrive %0, %1;" ::"n"(kId), "n"(kCount) : "memory");
}

// Shared-memory matrix descriptor kept as two 32-bit words. The low word holds the
// start address (>> 4, bits 0-13) and the leading offset; adding a byte offset >> 4
// to it moves the start (shared addresses stay below 256 KB, so no carry leaves the
// 14-bit field). One add per MMA instead of re-encoding the whole descriptor.
struct SDesc {
  uint32_t lo, hi;
  __device__ __forceinline__ uint64_t at(uint32_t byte_off) const {
    return ((uint64_t)hi << 32) | (uint32_t)(lo + (byte_off >> 4));
  }
};
__device__ __forceinline__ SDesc sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  const uint64_t d = smem_desc(saddr, lbo, sbo, layout);
  return SDesc{(uint32_t)d, (uint32_t)(d >> 32)};
}

template <typename T> struct Cfg;
template <> struct Cfg<__half> {
  static constexpr uint32_t fmt = 0;
  static constexpr int kSplits = 2, kQBufs = 3;
  static __device__ __forceinline__ uint16_t one() { return 0x3C00u; }
};
template <> struct Cfg<__nv_bfloat16> {
  static constexpr uint32_t fmt = 1;
  static constexpr int kSplits = 3, kQBufs = 1;
  static __device__ __forceinline__ uint16_t one() { return 0x3F80u; }
};
template <typename T> struct Layout {
  static constexpr uint32_t kImages = (Cfg<T>::kSplits + 1) * kImg;  // key terms + V
  static constexpr uint32_t OFF_V = Cfg<T>::kSplits * kImg;
  static constexpr uint32_t OFF_P = OFF_V + kImg;
  static constexpr uint32_t OFF_Q = OFF_P + 4 * 16384;
  static constexpr uint32_t OFF_ONES = OFF_Q + Cfg<T>::kQBufs * kQBytes;
  static constexpr uint32_t OFF_XCH = OFF_ONES + 2048;  // [7][kRowThreads] packed ranks: per-thread top-7 lists
  static constexpr uint32_t OFF_MISC = OFF_XCH + kTopK * kRowThreads * 8;
  static constexpr uint32_t kSmem = OFF_MISC + 192 + 1024;  // + alignment slack
  static_assert(kSmem <= 232448, "shared memory budget");
};

__device__ __forceinline__ bool timed_wait(uint64_t* bar, uint32_t parity) { return mbar_timed_wait(bar, parity); }

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
// Two floats <-> two packed 16-bit values (round to nearest), one conversion instruction per pair.
template <typename T> __device__ __forceinline__ uint32_t pack2(float a, float b);
template <> __device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
template <typename T> __device__ __forceinline__ float2 unpack2(uint32_t u);
template <> __device__ __forceinline__ float2 unpack2<__half>(uint32_t u) {
  return __half22float2(*reinterpret_cast<const __half2*>(&u));
}
template <> __device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t u) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
}

// Descending sort of 8 floats (19 compare-exchanges).
__device__ __forceinline__ void sort8_desc(float (&a)[8]) {
  constexpr int P[19][2] = {{0, 1}, {2, 3}, {4, 5}, {6, 7}, {0, 2}, {1, 3}, {4, 6}, {5, 7}, {1, 2}, {5, 6},
                            {0, 4}, {3, 7}, {1, 5}, {2, 6}, {1, 4}, {3, 6}, {2, 4}, {3, 5}, {3, 4}};
#pragma unroll
  for (int e = 0; e < 19; ++e) {
    const float x = a[P[e][0]], y = a[P[e][1]];
    a[P[e][0]] = fmaxf(x, y);
    a[P[e][1]] = fminf(x, y);
  }
}
// Top 8 (descending) of two descending lists of 8: bitonic merge.
__device__ __forceinline__ void merge8_desc(const float* A, const float* B, float (&c)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) c[i] = fmaxf(A[i], B[7 - i]);
#pragma unroll
  for (int s = 4; s >= 1; s >>= 1)
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if ((i & s) == 0) {
        const float x = c[i], y = c[i + s];
        c[i] = fmaxf(x, y);
        c[i + s] = fminf(x, y);
      }
}

// A rank packs (score key, slot) into 64 bits so that larger means earlier in
// the order "score descending, lower slot first on ties": key in the high
// word, the complement of the slot in the low word. Rank 0 is below every
// real entry.
__device__ __forceinline__ uint64_t pack_rank(uint32_t key, int slot) {
  return ((uint64_t)key << 32) | (uint32_t)~slot;
}
__device__ __forceinline__ int rank_slot(uint64_t r) { return (int)~(uint32_t)r; }
__device__ __forceinline__ uint32_t rank_score_key(uint64_t r) { return (uint32_t)(r >> 32); }
__device__ __forceinline__ uint64_t max64(uint64_t a, uint64_t b) { return a > b ? a : b; }
__device__ __forceinline__ uint64_t min64(uint64_t a, uint64_t b) { return a > b ? b : a; }

// Insert (key xk, slot xs) into a list of 7 kept in rank order (branch-free).
// Offers must come in ascending slot order: then an equal key never displaces
// an earlier entry, and comparing keys alone gives the exact rank order.
__device__ __forceinline__ void offer7_asc(uint32_t (&k)[kTopK], int (&sl)[kTopK], uint32_t xk, int xs) {
  bool gt[kTopK];
#pragma unroll
  for (int j = 0; j < kTopK; ++j) gt[j] = xk > k[j];
#pragma unroll
  for (int j = kTopK - 1; j >= 1; --j) {
    k[j] = gt[j - 1] ? k[j - 1] : (gt[j] ? xk : k[j]);
    sl[j] = gt[j - 1] ? sl[j - 1] : (gt[j] ? xs : sl[j]);
  }
  k[0] = gt[0] ? xk : k[0];
  sl[0] = gt[0] ? xs : sl[0];
}
// Best 8 (descending) of two descending lists of 8 ranks: bitonic merge.
__device__ __forceinline__ void merge8_rank(const uint64_t (&A)[8], const uint64_t (&B)[8], uint64_t (&c)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) c[i] = max64(A[i], B[7 - i]);
#pragma unroll
  for (int s = 4; s >= 1; s >>= 1)
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if ((i & s) == 0) {
        const uint64_t x = c[i], y = c[i + s];
        c[i] = max64(x, y);
        c[i + s] = min64(x, y);
      }
}
// Three-input maximum (one instruction on sm_100).
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// Bit i set where x[i] >= t (t finite, x[i] finite or -inf). x - t is >= 0 exactly when
// x >= t (a difference of distinct floats never rounds to +0), so the complement of its
// sign bit is the comparison: one subtraction on the FMA pipe and one funnel shift per
// column, four independent chains of 8.
__device__ __forceinline__ uint32_t ge_mask32(const float (&x)[32], float t) {
  uint32_t c[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int i = 7; i >= 0; --i)
#pragma unroll
    for (int q = 0; q < 4; ++q) c[q] = __funnelshift_l(__float_as_uint(x[8 * q + i] - t), c[q], 1);
  return ~(c[0] | (c[1] << 8) | (c[2] << 16) | (c[3] << 24));
}
// x[b] for a run-time b in [0, 32) over 32 values held in registers (select tree).
__device__ __forceinline__ float pick32(const float* x, int b) {
  float t[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) t[j] = (b & 1) ? x[2 * j + 1] : x[2 * j];
#pragma unroll
  for (int j = 0; j < 8; ++j) t[j] = (b & 2) ? t[2 * j + 1] : t[2 * j];
#pragma unroll
  for (int j = 0; j < 4; ++j) t[j] = (b & 4) ? t[2 * j + 1] : t[2 * j];
#pragma unroll
  for (int j = 0; j < 2; ++j) t[j] = (b & 8) ? t[2 * j + 1] : t[2 * j];
  return (b & 16) ? t[1] : t[0];
}

}  // namespace tc

// ---------------------------------------------------------------------------
// Slot-side kernels of the tensor-core path: 16 threads per slot row (4 dims
// each, 16-byte coalesced accesses, two rows per warp), and they also write the
// next round's operand images.
// ---------------------------------------------------------------------------
namespace tc {
constexpr int kRowLanes = 16;  // threads per slot row
__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ void st4(float* p, float4 x) { *reinterpret_cast<float4*>(p) = x; }

// The MMA operand type of a forward over inputs of type T: fp16 for both fp16 and bf16 inputs.
// bf16 inputs enter as fp16 under per-(b,h) power-of-two scales (q tiles converted in place, key
// and value images written scaled): the largest |x| of a pair maps into [2^14, 2^15), so a bf16
// value (8 significant bits) converts exactly unless it lies below 2^-39 of that largest value.
// The slot state of every round stays within the largest |x| of the initial slots and of q (the
// EMA and the diffusion are convex combinations, the update mean a weighted mean of q rows), so
// the key and value scales are fixed once per pair, from the round-0 tables and q.
using CT = __half;
__device__ __forceinline__ float pow2f(int e) { return __uint_as_float((uint32_t)(e + 127) << 23); }  // e in [-126, 126]
__device__ __forceinline__ int scale_exp(float m) {  // m * 2^e in [2^14, 2^15); 0 for m = 0 or not finite
  if (!(m > 0.f) || !(m < INFINITY)) return 0;
  const int ex = (int)((__float_as_uint(m) >> 23) & 0xffu) - 127;
  return max(-126, min(126, 14 - ex));
}
__device__ __forceinline__ float absmax4(float4 x) { return fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))); }
__device__ __forceinline__ uint4 bf16_to_f16_scaled(const uint4& u, float s) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float lo = __uint_as_float(w[i] << 16) * s, hi = __uint_as_float(w[i] & 0xFFFF0000u) * s;
    o[i] = (uint32_t)__half_as_ushort(__float2half_rn(lo)) | ((uint32_t)__half_as_ushort(__float2half_rn(hi)) << 16);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// Write columns 4*l .. 4*l+3 of slot row m into the operand images (row m at
// m*128 bytes, 16-byte chunks XOR-swizzled by m & 7), keys and values multiplied by their
// scales (powers of two, 1 for fp16 inputs) first.
template <typename T>
__device__ __forceinline__ void put_images(uint8_t* base, int m, int l, float4 k, float4 v, float sk, float sv) {
  const uint32_t off = (uint32_t)m * 128 + ((((uint32_t)l >> 1) ^ (m & 7)) << 4) + (l & 1) * 8;
  float kk[4] = {k.x * sk, k.y * sk, k.z * sk, k.w * sk};
  v = make_float4(v.x * sv, v.y * sv, v.z * sv, v.w * sv);
#pragma unroll
  for (int s = 0; s < Cfg<T>::kSplits; ++s) {
    uint32_t a[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      a[i] = to_bits<T>(kk[i]);
      kk[i] -= from_bits<T>((uint16_t)a[i]);  // exact in fp32: the next term carries the residual
    }
    *reinterpret_cast<uint2*>(base + s * kImg + off) = make_uint2(a[0] | (a[1] << 16), a[2] | (a[3] << 16));
  }
  const uint32_t v0 = to_bits<T>(v.x), v1 = to_bits<T>(v.y), v2 = to_bits<T>(v.z), v3 = to_bits<T>(v.w);
  *reinterpret_cast<uint2*>(base + Layout<T>::OFF_V + off) = make_uint2(v0 | (v1 << 16), v2 | (v3 << 16));
}
}  // namespace tc

// bf16 inputs: the largest |q|, |slots_k|, |slots_v| over block y's 1/16 of a pair's tokens and
// slot rows -> amax[bh][y][0..2]. grid (BH, 16), 256 threads.
template <typename T, typename S>
__global__ void __launch_bounds__(256) k_tc_amax(Geom g, const T* q, Strides3 qs, const S* sk, Strides3 sks,
                                                 const S* svv, Strides3 svs, float* amax) {
  pdl_wait();  // the previous step's kernels may still read amax
  pdl_trigger();
  __shared__ float red[3][8];
  const int bh = blockIdx.x, b = bh / g.H, h = bh - b * g.H, y = blockIdx.y, ny = gridDim.y;
  const int n0 = (int)((int64_t)g.N * y / ny), n1 = (int)((int64_t)g.N * (y + 1) / ny);
  float mq = 0.f, mk = 0.f, mv = 0.f;
  // eight independent 16-byte loads in flight per thread: the pass is bound by loads outstanding
  constexpr int kU = 8;
  const int cnt = (n1 - n0) * 8;
  for (int e0 = threadIdx.x; e0 < cnt; e0 += kU * blockDim.x) {
    uint4 u[kU];
#pragma unroll
    for (int j = 0; j < kU; ++j) {
      const int e = e0 + j * blockDim.x;
      u[j] = e < cnt ? *reinterpret_cast<const uint4*>(row_ptr(q, qs, b, h, n0 + (e >> 3)) + 8 * (e & 7))
                     : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int j = 0; j < kU; ++j) {
      const uint32_t w[4] = {u[j].x, u[j].y, u[j].z, u[j].w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
        mq = fmaxf(mq, fmaxf(__uint_as_float((w[i] & 0x7FFFu) << 16), __uint_as_float(w[i] & 0x7FFF0000u)));
    }
  }
  const int m0 = g.M * y / ny, m1 = g.M * (y + 1) / ny;
  for (int e = threadIdx.x; e < (m1 - m0) * tc::kD; e += blockDim.x) {
    const int m = m0 + e / tc::kD, c = e % tc::kD;
    mk = fmaxf(mk, fabsf(Elem<S>::load(row_ptr(sk, sks, b, h, m) + c)));
    mv = fmaxf(mv, fabsf(Elem<S>::load(row_ptr(svv, svs, b, h, m) + c)));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    mq = fmaxf(mq, __shfl_xor_sync(0xffffffffu, mq, o));
    mk = fmaxf(mk, __shfl_xor_sync(0xffffffffu, mk, o));
    mv = fmaxf(mv, __shfl_xor_sync(0xffffffffu, mv, o));
  }
  if ((threadIdx.x & 31) == 0) {
    red[0][threadIdx.x >> 5] = mq;
    red[1][threadIdx.x >> 5] = mk;
    red[2][threadIdx.x >> 5] = mv;
  }
  __syncthreads();
  if (threadIdx.x < 3) {
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) m = fmaxf(m, red[threadIdx.x][i]);
    amax[((size_t)bh * ny + y) * 3 + threadIdx.x] = m;
  }
}

// The pair's operand-scale exponents (bf16 inputs: from the k_tc_amax maxima; fp16: 0): q, keys, values.
template <typename T>
__device__ __forceinline__ int3 pair_exps(const float* amax, int bh) {
  if constexpr (std::is_same<T, __half>::value) {
    return make_int3(0, 0, 0);
  } else {
    float mq = 0.f, mk = 0.f, mv = 0.f;
#pragma unroll 4
    for (int y = 0; y < kAmaxBlocks; ++y) {
      const float* a = amax + ((size_t)bh * kAmaxBlocks + y) * 3;
      mq = fmaxf(mq, a[0]);
      mk = fmaxf(mk, a[1]);
      mv = fmaxf(mv, a[2]);
    }
    return make_int3(tc::scale_exp(mq), tc::scale_exp(fmaxf(mk, mq)), tc::scale_exp(fmaxf(mv, mq)));
  }
}

// Round-0 state: slot tables (element type S: the dtype of q, or fp32 slot state; strided, batch
// stride 0 broadcasts) -> fp32 state + images. grid (BH, 256/16): block y covers 16 slot rows,
// 16 threads each (rows >= M write zero images). Also zeroes the pair's two counters of the
// multi-round forward launch that follows and records the pair's operand-scale exponents.
template <typename T, typename S>
__global__ void __launch_bounds__(tc::kRowLanes * kSlotRows) k_tc_load(Geom g, const S* sk, Strides3 sks, const S* svv,
                                                                        Strides3 svs, Saved sv, uint8_t* images,
                                                                        int* counters, const float* amax, int* fexp) {
  pdl_wait();  // the previous step's kernels may still read the state, images and counters
  pdl_trigger();
  const int bh = blockIdx.x, b = bh / g.H, h = bh - b * g.H, l = threadIdx.x & 15;
  const int3 ex = pair_exps<T>(amax, bh);
  if (blockIdx.y == 0 && threadIdx.x == 0) {
    counters[bh] = 0;
    counters[g.BH + bh] = 0;
    fexp[4 * bh] = ex.x;
    fexp[4 * bh + 1] = ex.y;
    fexp[4 * bh + 2] = ex.z;
  }
  uint8_t* base = images + (size_t)bh * tc::Layout<tc::CT>::kImages;
  const int m = blockIdx.y * kSlotRows + (threadIdx.x >> 4);
  float4 k = make_float4(0.f, 0.f, 0.f, 0.f), v = k;
  if (m < g.M) {
    const S* pk = row_ptr(sk, sks, b, h, m) + 4 * l;
    const S* pv = row_ptr(svv, svs, b, h, m) + 4 * l;
    k = make_float4(Elem<S>::load(pk), Elem<S>::load(pk + 1), Elem<S>::load(pk + 2), Elem<S>::load(pk + 3));
    v = make_float4(Elem<S>::load(pv), Elem<S>::load(pv + 1), Elem<S>::load(pv + 2), Elem<S>::load(pv + 3));
    const size_t e = (size_t)bh * g.M * tc::kD + (size_t)m * tc::kD + 4 * l;
    tc::st4(sv.K + e, k);
    tc::st4(sv.V + e, v);
  }
  tc::put_images<tc::CT>(base, m, l, k, v, tc::pow2f(ex.y), tc::pow2f(ex.z));
}

__device__ __forceinline__ float4 ema4(float a, float b, float4 x, float4 u) {
  return make_float4(__fadd_rn(__fmul_rn(a, x.x), __fmul_rn(b, u.x)), __fadd_rn(__fmul_rn(a, x.y), __fmul_rn(b, u.y)),
                     __fadd_rn(__fmul_rn(a, x.z), __fmul_rn(b, u.z)), __fadd_rn(__fmul_rn(a, x.w), __fmul_rn(b, u.w)));
}
// x + gamma * ((l + r) - 2 x), each operation rounded as the reference's fp32 tensor ops.
__device__ __forceinline__ float diffuse1(float x, float l, float r, float gamma) {
  return __fadd_rn(x, __fmul_rn(gamma, __fsub_rn(__fadd_rn(l, r), __fmul_rn(2.f, x))));
}
__device__ __forceinline__ float4 diffuse4(float4 x, float4 l, float4 r, float gamma) {
  return make_float4(diffuse1(x.x, l.x, r.x, gamma), diffuse1(x.y, l.y, r.y, gamma), diffuse1(x.z, l.z, r.z, gamma),
                     diffuse1(x.w, l.w, r.w, gamma));
}

// Finalize round r: combine the segment partials in token order, EMA (reference.py:105-113)
// and diffusion (reference.py:128-133) -> state entering round r+1, U_r, W_r and
// the images of round r+1. grid (BH, 256/16): a block owns 16 slot rows and recomputes
// one halo row on each side; 16 threads per row, up to 12 partial loads of a row in flight at once.
template <typename T>
__global__ void __launch_bounds__(tc::kRowLanes * kSlotHalo, 2) k_tc_finalize(Geom g, int r, Saved sv, FwdScratch fs,
                                                                                      const __grid_constant__ TileSplit split) {
  pdl_wait();  // the round's chunk partials
  pdl_trigger();
  __shared__ float4 kn[kSlotHalo][tc::kRowLanes];
  __shared__ float4 vn[kSlotHalo][tc::kRowLanes];
  const int bh = blockIdx.x, rr = threadIdx.x >> 4, l = threadIdx.x & 15;
  const int m0 = blockIdx.y * kSlotRows;
  const int m = m0 - 1 + rr;  // rows m0-1 .. m0+16
  const size_t MD = (size_t)g.M * tc::kD;
  const size_t cur = ((size_t)r * g.BH + bh) * MD;
  {
    float4 k = make_float4(0.f, 0.f, 0.f, 0.f), v = k;
    if (m >= 0 && m < g.M) {
      const size_t e = cur + (size_t)m * tc::kD + 4 * l;
      k = tc::ld4(sv.K + e);
      v = tc::ld4(sv.V + e);
      float4 S = make_float4(0.f, 0.f, 0.f, 0.f);
      float W = 0.f;
      const int nparts = split.parts(bh);
      constexpr int kW = 12;  // loads in flight: one round for up to 12 partials (north-star: 10)
      for (int ch = 0; ch < nparts; ch += kW) {  // added in token order
        float4 a[kW];
        float wv[kW];
#pragma unroll
        for (int u = 0; u < kW; ++u) {
          const size_t po = (size_t)bh * g.ft_parts + min(ch + u, nparts - 1);
          a[u] = reinterpret_cast<const float4*>(fs.Spart)[(po * 16 + l) * g.M + m];
          wv[u] = fs.Wpart[po * g.M + m];
        }
#pragma unroll
        for (int u = 0; u < kW; ++u) {
          if (ch + u < nparts) {
            S.x = __fadd_rn(S.x, a[u].x);
            S.y = __fadd_rn(S.y, a[u].y);
            S.z = __fadd_rn(S.z, a[u].z);
            S.w = __fadd_rn(S.w, a[u].w);
            W = __fadd_rn(W, wv[u]);
          }
        }
      }
      const bool hit = W > 0.f;
      const float den = __fadd_rn(W, kEmaEps);
      const float4 U = make_float4(__fdiv_rn(S.x, den), __fdiv_rn(S.y, den), __fdiv_rn(S.z, den), __fdiv_rn(S.w, den));
      if (rr >= 1 && rr <= kSlotRows) {  // this block's rows record U and W
        tc::st4(sv.U + e, U);
        if (l == 0) sv.W[((size_t)r * g.BH + bh) * g.M + m] = W;
      }
      if (hit) {
        k = ema4(g.alpha, g.one_minus_alpha, k, U);
        v = ema4(g.alpha, g.one_minus_alpha, v, U);
      }
    }
    kn[rr][l] = k;
    vn[rr][l] = v;
  }
  __syncthreads();
  if (rr < 1 || rr > kSlotRows) return;
  uint8_t* base = fs.images + (size_t)bh * tc::Layout<tc::CT>::kImages;
  const size_t nxt = ((size_t)(r + 1) * g.BH + bh) * MD;
  float4 k = make_float4(0.f, 0.f, 0.f, 0.f), v = k;
  if (m < g.M) {
    k = kn[rr][l];
    v = vn[rr][l];
    if (m > 0 && m < g.M - 1) {
      k = diffuse4(k, kn[rr - 1][l], kn[rr + 1][l], g.gamma);
      v = diffuse4(v, vn[rr - 1][l], vn[rr + 1][l], g.gamma);
    }
    const size_t e = nxt + (size_t)m * tc::kD + 4 * l;
    tc::st4(sv.K + e, k);
    tc::st4(sv.V + e, v);
  }
  tc::put_images<tc::CT>(base, m, l, k, v, tc::pow2f(fs.fexp[4 * bh + 1]), tc::pow2f(fs.fexp[4 * bh + 2]));  // rows >= M: zero
}

// ---------------------------------------------------------------------------
// The forward round kernel, rounds [r0, r1): 8 row warps (thread = token row x half of the
// slots) rank the tiles, 4 epilogue warps (thread = token row) write the weights, the round
// records and the output, and the issuer warp's lane 0 issues every MMA and copy, so neither
// stalls behind the tensor-core queue; 3 more warps only give their registers to the row warps.
//
// Tensor-core order per tile i (fp16): SELECT(i+1) (scores of the next tile, once the row warps
// have read tile i's), MMA_B(i-1) = {S += P_lo^T.Q, W += P_lo^T.1}, MMA_A(i) = {O = P_hi.V,
// S += P_hi^T.Q, W += P_hi^T.1}. The row warps rank tile i+1 while the epilogue warps finish
// tile i. After the last round no update is issued (no P_lo, no partials).
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(tc::kThreads, 1)
    k_fwd_tc(Geom g, int r0, int r1, const __grid_constant__ CUtensorMap qmap, T* out, Strides3 os, int64_t* indices,
             float* weights, Saved sv, FwdScratch fs, const __grid_constant__ TileSplit split) {
  using C = tc::Cfg<tc::CT>;  // MMA operands: fp16 (bf16 inputs converted under the pair's scales)
  using L = tc::Layout<tc::CT>;
  constexpr bool kConv = !std::is_same<T, __half>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t s_base = smem_u32(sm);
  uint64_t* bar_img = reinterpret_cast<uint64_t*>(sm + L::OFF_MISC);
  uint64_t* bar_q = bar_img + 1;  // [3], one per Q buffer
  uint64_t* bar_s = bar_img + 4;  // SELECT done
  uint64_t* bar_a = bar_img + 5;  // MMA_A done
  uint64_t* bar_b = bar_img + 6;  // MMA_B done
  uint64_t* hand_ready = bar_img + 7;  // [4] per lane quadrant: the row warps' picks of a tile are in TMEM
  uint64_t* hand_free = bar_img + 11;  // [4] per lane quadrant: the epilogue warp has read them
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + L::OFF_MISC + 128);
  volatile int* s_abort = reinterpret_cast<volatile int*>(sm + L::OFF_MISC + 132);
  uint64_t* q_conv = reinterpret_cast<uint64_t*>(sm + L::OFF_MISC + 136);  // [3] bf16: Q buffer converted

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool issuer_warp = warp == tc::kIssuerWarp;
  const bool row_warp = warp < tc::kEpiWarp;
  const bool epi_warp = warp >= tc::kEpiWarp && warp < tc::kIssuerWarp;
  const int row = tid & (kTile - 1);  // token row within the tile == TMEM lane
  const int part = (tid >> 7) & 1;    // which 128 of the 256 slot columns this thread scans
  const int quadrant = warp & 3;
  // entry j of thread t's top-7 list at [j][t]: a warp touches consecutive words (no bank conflicts)
  uint64_t* xch = reinterpret_cast<uint64_t*>(sm + L::OFF_XCH);
  // this CTA's run of the flat (b,h) x tile list, one segment per (b,h) it meets
  const int cta = blockIdx.x;
  const int u_end = split.start[cta + 1];
  int r = r0;               // the round being run; each role steps through [r0, r1)
  bool last_round = false;  // no slot update follows the last round: no second weight term, no partials
  // Several rounds in one launch (all CTAs resident: a cooperative launch): between rounds the
  // CTAs of each pair combine its slot-sum partials themselves, through two counters per pair.
  const bool multi = r1 - r0 > 1;
  int* cnt_part = fs.counters;         // [BH] segment partials written, over the launch
  int* cnt_fin = fs.counters + g.BH;   // [BH] finalize shares done, over the launch
  int bh = 0, b = 0, h = 0, part_idx = 0, t_beg = 0, t_end = 0, ntiles = 0;
  auto set_segment = [&](int u) {  // the segment that starts at unit u
    bh = u / split.tpb;
    b = bh / g.H;
    h = bh - b * g.H;
    const int base = bh * split.tpb;
    const int t0 = u - base, t1 = min(split.tpb, u_end - base);
    t_beg = t0 * kTile;
    t_end = min(g.N, t1 * kTile);
    ntiles = t1 - t0;
    part_idx = cta - split.first_cta(bh);
  };
  auto next_segment = [&]() -> int { return (bh + 1) * split.tpb; };
  constexpr uint32_t ID_SEL = idesc_f16(C::fmt, 128, 256, 0, 0);
  constexpr uint32_t ID_ATT = idesc_f16(C::fmt, 128, 64, 0, 1);
  // S += P^T.[Q | 1]: N = 80, the last 16 columns of B are ones, so they accumulate W
  constexpr uint32_t ID_UPD = idesc_f16(C::fmt, 128, tc::kUW, 1, 1);

  // ---- set-up: barriers, zeroed P, ones, TMEM ----
  if (tid == 0) {
    mbar_init(bar_img, 1);
    for (int i = 0; i < 3; ++i) mbar_init(&q_conv[i], 96);  // warps 13-15 (bf16 inputs)
    for (int i = 0; i < 3; ++i) mbar_init(&bar_q[i], 1);
    mbar_init(bar_s, 1);
    mbar_init(bar_a, 1);
    mbar_init(bar_b, 1);
    for (int i = 0; i < 4; ++i) {
      mbar_init(&hand_ready[i], 64);  // the quadrant's two row warps
      mbar_init(&hand_free[i], 32);   // the quadrant's epilogue warp
    }
    *s_abort = 0;
    fence_barrier_init();
  }
  {
    float4* p4 = reinterpret_cast<float4*>(sm + L::OFF_P);
    for (int i = tid; i < 4 * 16384 / 16; i += tc::kThreads) p4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    uint16_t* ones = reinterpret_cast<uint16_t*>(sm + L::OFF_ONES);
    for (int i = tid; i < 1024; i += tc::kThreads) ones[i] = C::one();  // 16 rows x 64 of 16-bit ones
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, tc::kTmemCols);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // everything above touched only this CTA's shared memory and TMEM: it overlaps the previous
  // kernel, whose outputs (the round's state and operand images) are read from here on
  pdl_wait();
  pdl_trigger();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = (uint32_t)(32 * quadrant) << 16;
  const uint32_t a_v = s_base + L::OFF_V, a_p = s_base + L::OFF_P, a_ones = s_base + L::OFF_ONES;

  // mbarrier phases of the row threads (each waits every phase once)
  uint32_t ph_s = 0, ph_a = 0, ph_b = 0;
  // the issuer's bookkeeping of asynchronous copies
  bool img_pending = false, q_pending[3] = {false, false, false};
  uint32_t img_phase = 0;
  uint32_t q_phase[3] = {0, 0, 0};

  auto fail = [&](int code) {
    atomicOr(&g_device_error, code);
    *s_abort = 1;
  };
  auto wait_bar = [&](uint64_t* bar, uint32_t& ph) {
    if (tc::timed_wait(bar, ph)) ph ^= 1;
    else fail(tc::kErrMmaWait);
    tc_fence_after();
  };
  auto q_slot = [&](int tile_idx) { return tile_idx % C::kQBufs; };
  auto issue_q = [&](int tile_idx) {  // issuer
    const int bs = q_slot(tile_idx);
    mbar_arrive_expect_tx(&bar_q[bs], tc::kQBytes);
    tma_load_4d(sm + L::OFF_Q + bs * tc::kQBytes, &qmap, 0, t_beg + tile_idx * kTile, h, b, &bar_q[bs]);
    q_pending[bs] = true;
  };
  uint32_t qc_phase[3] = {0, 0, 0};  // issuer: conversions of the Q buffers waited for (bf16 inputs)
  auto wait_q = [&](int tile_idx) -> bool {  // issuer
    const int bs = q_slot(tile_idx);
    if (!tc::timed_wait(&bar_q[bs], q_phase[bs])) {
      fail(tc::kErrQWait);
      return false;
    }
    q_phase[bs] ^= 1;
    q_pending[bs] = false;
    if (kConv) {  // warps 13-15 have converted the tile to fp16 in place
      if (!tc::timed_wait(&q_conv[bs], qc_phase[bs])) {
        fail(tc::kErrQWait);
        return false;
      }
      qc_phase[bs] ^= 1;
    }
    return true;
  };
  // operand descriptors (start addresses moved per MMA by SDesc::at)
  const tc::SDesc d_qk = tc::sdesc(s_base + L::OFF_Q, 16, 1024, kSwizzle128B);      // Q, K-major (SELECT A)
  const tc::SDesc d_key = tc::sdesc(s_base, 16, 1024, kSwizzle128B);                // key terms (SELECT B)
  const tc::SDesc d_pk = tc::sdesc(a_p, 16, 1024, kSwizzle128B);                    // P, K-major (attend A)
  const tc::SDesc d_pmn = tc::sdesc(a_p, 16384, 1024, kSwizzle128B);                // P, MN-major (update A)
  const tc::SDesc d_v = tc::sdesc(a_v, 16384, 1024, kSwizzle128B);                  // V (attend B)
  auto issue_select = [&](int tile_idx) {  // issuer
    const uint32_t q_off = q_slot(tile_idx) * tc::kQBytes;
    tc_fence_after();
#pragma unroll
    for (int s = 0; s < C::kSplits; ++s)
#pragma unroll
      for (int k = 0; k < 4; ++k)
        mma_f16(tmem + tc::COL_S, d_qk.at(q_off + k * 32), d_key.at(s * tc::kImg + k * 32), ID_SEL, (s | k) != 0);
    mma_commit(bar_s);
  };
  // issuer: [S | W] += P^T.[Q | 1]. B is MN-major with two 64-column atoms: the q tile's rows
  // kk*16.. and, LBO bytes further on, 16 rows of ones (the descriptor's LBO is set per MMA so
  // that the second atom always starts at the ones; only its first 16 columns are read).
  auto issue_update = [&](int tile_idx, bool first) {
    const uint32_t q_at = s_base + L::OFF_Q + q_slot(tile_idx) * tc::kQBytes;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint64_t a = d_pmn.at(2 * hh * 16384 + kk * 2048);
        const uint32_t b_at = q_at + kk * 2048;
        const uint64_t bq = smem_desc(b_at, a_ones - b_at, 1024, kSwizzle128B);
        mma_f16(tmem + tc::COL_U + tc::kUW * hh, a, bq, ID_UPD, (first && kk == 0) ? 0u : 1u);
      }
    }
  };
  auto p_off = [&](int m) -> uint32_t {  // byte offset of this row's entry for slot m in P
    return L::OFF_P + (m >> 6) * 16384 + sw128_offset(row, m & 63);
  };
  auto p_at = [&](uint32_t off) -> uint16_t* { return reinterpret_cast<uint16_t*>(sm + off); };

  // ---- between two rounds of one launch: the finalize of a pair, by the row warps ----
  // The CTAs whose runs end in pair p each take a share of its 256 padded slot rows (a CTA whose
  // run goes on into the next pair leaves p to the others); a pair whose only CTA runs on
  // beyond it is finalized by that CTA alone.
  auto fin_range = [&](int p, int& first, int& count) {
    first = split.first_cta(p);
    const int last = split.cta_of(p * split.tpb + split.tpb - 1);
    count = last - first + (split.start[last + 1] <= (p + 1) * split.tpb ? 1 : 0);
    if (count == 0) {
      first = last;
      count = 1;
    }
  };
  auto rows_sync = [&]() { asm volatile("bar.sync %0, %1;" ::"n"(tc::kBarRows), "n"(tc::kRowThreads) : "memory"); };
  // Share k of `count` of pair p after round r: once every CTA of p has written its partial,
  // combine the partials in token order, EMA (reference.py:105-113), diffusion
  // (reference.py:128-133); write U_r, W_r, the state entering round r+1 and its operand images.
  // Warp w takes columns 8w..8w+7 of 32 consecutive slot rows, a row per lane (the partials'
  // loads coalesce); rows base-1 and base+30 (lanes 0 and 31) are recomputed halos, so each pass
  // gives 30 rows and the diffusion's neighbours are the adjacent lanes.
  auto fin_share = [&](int p, int k, int count) {
    const int nparts = split.parts(p);
    const int done = r - r0;  // rounds of this launch finished before round r
    if (tid == 0 && !*s_abort) {
      if (!counter_wait_ge(&cnt_part[p], nparts * (done + 1)) || !counter_wait_ge(&cnt_fin[p], count * done))
        fail(tc::kErrPeerWait);
    }
    rows_sync();
    if (!*s_abort) {
      const size_t MD = (size_t)g.M * tc::kD;
      const size_t cur = ((size_t)r * g.BH + p) * MD, nxt = cur + (size_t)g.BH * MD;
      uint8_t* img = fs.images + (size_t)p * L::kImages;
      const float img_sk = kConv ? tc::pow2f(fs.fexp[4 * p + 1]) : 1.f;
      const float img_sv = kConv ? tc::pow2f(fs.fexp[4 * p + 2]) : 1.f;
      const int lo = k * tc::kSlotsPad / count, hi = (k + 1) * tc::kSlotsPad / count;
      const int c8 = warp * 8;  // this warp's first column
      for (int base = lo; base < hi; base += 30) {
        const int m = base - 1 + lane;
        const bool own = lane >= 1 && lane <= 30 && m < hi;
        float kx[8], vx[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) kx[i] = vx[i] = 0.f;
        if (m >= 0 && m < g.M) {
          const float4* ko = reinterpret_cast<const float4*>(sv.K + cur + (size_t)m * tc::kD + c8);
          const float4* vo = reinterpret_cast<const float4*>(sv.V + cur + (size_t)m * tc::kD + c8);
          const float4 k0 = ko[0], k1 = ko[1], v0 = vo[0], v1 = vo[1];
          float S[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) S[i] = 0.f;
          float W = 0.f;
          constexpr int kB = 6;  // partial loads in flight per batch
          for (int q0 = 0; q0 < nparts; q0 += kB) {  // added in token order
            float4 a0[kB], a1[kB];
            float wv[kB];
#pragma unroll
            for (int u = 0; u < kB; ++u) {
              const size_t po = (size_t)p * g.ft_parts + min(q0 + u, nparts - 1);
              const float4* sp = reinterpret_cast<const float4*>(fs.Spart) + (po * 16 + 2 * warp) * g.M + m;
              a0[u] = sp[0];
              a1[u] = sp[g.M];
              wv[u] = fs.Wpart[po * g.M + m];
            }
#pragma unroll
            for (int u = 0; u < kB; ++u) {
              if (q0 + u < nparts) {
                const float a[8] = {a0[u].x, a0[u].y, a0[u].z, a0[u].w, a1[u].x, a1[u].y, a1[u].z, a1[u].w};
#pragma unroll
                for (int i = 0; i < 8; ++i) S[i] = __fadd_rn(S[i], a[i]);
                W = __fadd_rn(W, wv[u]);
              }
            }
          }
          const float den = __fadd_rn(W, kEmaEps);
          float U[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) U[i] = __fdiv_rn(S[i], den);
          if (own) {
            float4* u = reinterpret_cast<float4*>(sv.U + cur + (size_t)m * tc::kD + c8);
            u[0] = make_float4(U[0], U[1], U[2], U[3]);
            u[1] = make_float4(U[4], U[5], U[6], U[7]);
            if (warp == 0) sv.W[((size_t)r * g.BH + p) * g.M + m] = W;
          }
          const float ko8[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
          const float vo8[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
          const bool hit = W > 0.f;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            kx[i] = hit ? __fadd_rn(__fmul_rn(g.alpha, ko8[i]), __fmul_rn(g.one_minus_alpha, U[i])) : ko8[i];
            vx[i] = hit ? __fadd_rn(__fmul_rn(g.alpha, vo8[i]), __fmul_rn(g.one_minus_alpha, U[i])) : vo8[i];
          }
        }
        float kl[8], kr[8], vl[8], vr[8];  // rows m-1 and m+1 (used by lanes 1..30 only)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          kl[i] = __shfl_up_sync(0xffffffffu, kx[i], 1);
          vl[i] = __shfl_up_sync(0xffffffffu, vx[i], 1);
          kr[i] = __shfl_down_sync(0xffffffffu, kx[i], 1);
          vr[i] = __shfl_down_sync(0xffffffffu, vx[i], 1);
        }
        if (own) {
          float kn[8], vn[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) kn[i] = vn[i] = 0.f;  // rows >= M: zero images
          if (m < g.M) {
            const bool inner = m > 0 && m < g.M - 1;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              kn[i] = inner ? diffuse1(kx[i], kl[i], kr[i], g.gamma) : kx[i];
              vn[i] = inner ? diffuse1(vx[i], vl[i], vr[i], g.gamma) : vx[i];
            }
            float4* kd = reinterpret_cast<float4*>(sv.K + nxt + (size_t)m * tc::kD + c8);
            float4* vd = reinterpret_cast<float4*>(sv.V + nxt + (size_t)m * tc::kD + c8);
            kd[0] = make_float4(kn[0], kn[1], kn[2], kn[3]);
            kd[1] = make_float4(kn[4], kn[5], kn[6], kn[7]);
            vd[0] = make_float4(vn[0], vn[1], vn[2], vn[3]);
            vd[1] = make_float4(vn[4], vn[5], vn[6], vn[7]);
          }
          // the 8 columns are one 16-byte chunk of each 16-bit image (128-byte swizzle), keys and
          // values under the pair's scales
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            kn[i] *= img_sk;
            vn[i] *= img_sv;
          }
          const uint32_t off = (uint32_t)m * 128 + (((uint32_t)warp ^ ((uint32_t)m & 7)) << 4);
#pragma unroll
          for (int sp = 0; sp < C::kSplits; ++sp) {
            uint32_t w4[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const uint32_t a = tc::to_bits<tc::CT>(kn[2 * i]), b2 = tc::to_bits<tc::CT>(kn[2 * i + 1]);
              kn[2 * i] -= tc::from_bits<tc::CT>((uint16_t)a);  // exact in fp32: the next term carries the residual
              kn[2 * i + 1] -= tc::from_bits<tc::CT>((uint16_t)b2);
              w4[i] = a | (b2 << 16);
            }
            *reinterpret_cast<uint4*>(img + sp * tc::kImg + off) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
          }
          uint32_t w4[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) w4[i] = tc::to_bits<tc::CT>(vn[2 * i]) | (tc::to_bits<tc::CT>(vn[2 * i + 1]) << 16);
          *reinterpret_cast<uint4*>(img + L::OFF_V + off) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
        }
      }
    }
    rows_sync();
    if (tid == 0) {  // even after a failure, so that the pair's other CTAs do not wait out their limit
      __threadfence();
      counter_release_add(&cnt_fin[p], 1);
    }
  };

  // fp16 (three Q buffers) runs SELECT(i+1) ahead of MMA_A(i): the row warps rank tile i+1
  // while MMA_A(i) runs, then finish tile i (second weight term, output). bf16 has one Q
  // buffer, so SELECT(i+1) waits for MMA_B(i) and the row warps finish tile i first.
  constexpr bool kEarlySelect = C::kQBufs >= 3;
  if (issuer_warp) {
    // ================= issuer warp =================
    uint32_t n_s = 0, n_a = 0, n_b = 0;  // commits per barrier
    // every committed group is complete (bounded waits): before a segment overwrites the
    // operand images and Q buffers, and before TMEM is freed
    auto drain = [&]() -> bool {
      bool ok = true;
      if (n_s) ok = tc::timed_wait(bar_s, (n_s - 1) & 1) && ok;
      if (n_a) ok = tc::timed_wait(bar_a, (n_a - 1) & 1) && ok;
      if (n_b) ok = tc::timed_wait(bar_b, (n_b - 1) & 1) && ok;
      return ok;
    };
    auto mma_b = [&](int tile_idx) {  // ---- MMA_B(tile_idx) ----
      tc::issuer_wait<tc::kBarPlo, tc::kCountP>();
      if (lane == 0 && !*s_abort) {
        tc_fence_after();
        issue_update(tile_idx, false);
        mma_commit(bar_b);
        ++n_b;
        if (!kEarlySelect && tile_idx + 1 < ntiles) {  // one Q buffer: free once MMA_B is done
          if (!tc::timed_wait(bar_b, (n_b - 1) & 1)) {
            fail(tc::kErrMmaWait);
          } else {
            tc_fence_after();
            issue_q(tile_idx + 1);
            if (wait_q(tile_idx + 1)) {
              issue_select(tile_idx + 1);
              ++n_s;
            }
          }
        }
      }
      __syncwarp();
    };
    // last round, one Q buffer: no update reads it, so SELECT(i+1) follows MMA_A(i) (the rows
    // had tile i's scores, so SELECT(i) is complete)
    auto select_next = [&](int tile_idx) {
      if (lane == 0 && !*s_abort && tile_idx + 1 < ntiles) {
        issue_q(tile_idx + 1);
        if (wait_q(tile_idx + 1)) {
          issue_select(tile_idx + 1);
          ++n_s;
        }
      }
      __syncwarp();
    };
    for (r = r0; r < r1; ++r) {
    last_round = r == g.R - 1;
    for (int u = split.start[cta]; u < u_end; u = next_segment()) {
    set_segment(u);
    if (lane == 0 && !*s_abort) {  // segment prologue: operand images, first token tiles, first SELECT
      if (!drain()) {
        fail(tc::kErrMmaWait);
      } else {
        for (int i = 0; i < C::kQBufs && i < ntiles; ++i) issue_q(i);
        if (multi && r > r0) {  // the pair's finalize after the previous round is done
          int first, count;
          fin_range(bh, first, count);
          if (!counter_wait_ge(&cnt_fin[bh], count * (r - r0))) fail(tc::kErrPeerWait);
          fence_proxy_async_global();  // images written by other CTAs, read by the bulk copy below
        }
      }
      if (!*s_abort) {
        mbar_arrive_expect_tx(bar_img, L::kImages);
        bulk_g2s(sm, fs.images + (size_t)bh * L::kImages, L::kImages, bar_img);
        img_pending = true;
        if (!tc::timed_wait(bar_img, img_phase)) {
          fail(tc::kErrImgWait);
        } else {
          img_pending = false;
          img_phase ^= 1;
        }
        if (ntiles > 0 && !*s_abort && wait_q(0)) {
          issue_select(0);
          ++n_s;
        }
      }
    }
    __syncwarp();
    for (int tile = 0; tile < ntiles; ++tile) {
      if (kEarlySelect) {
        // the row warps free tile i's scores before the epilogue warps finish tile i-1's weights,
        // so SELECT(i+1) goes first
        tc::issuer_wait<tc::kBarSfree, tc::kCountS>();  // the scores of tile i are read: SELECT(i+1)
        if (lane == 0 && !*s_abort && tile + 1 < ntiles) {
          tc_fence_after();
          if (wait_q(tile + 1)) {
            issue_select(tile + 1);
            ++n_s;
          }
        }
        __syncwarp();
        if (tile > 0 && !last_round) mma_b(tile - 1);
      }
      tc::issuer_wait<tc::kBarPhi, tc::kCountP>();
      if (lane == 0 && !*s_abort) {
        tc_fence_after();
        // ---- MMA_A(i) ----
#pragma unroll
        for (int kk = 0; kk < 16; ++kk)
          mma_f16(tmem + tc::COL_O, d_pk.at((kk >> 2) * 16384 + (kk & 3) * 32), d_v.at(kk * 2048), ID_ATT, kk != 0);
        if (!last_round) issue_update(tile, tile == 0);
        mma_commit(bar_a);
        ++n_a;
        // the epilogue warps saw MMA_B(i-1) complete before writing P (in the last round no update
        // reads the Q tiles): its Q buffer is free
        if (C::kQBufs > 1 && tile >= 1 && tile - 1 + C::kQBufs < ntiles) issue_q(tile - 1 + C::kQBufs);
      }
      __syncwarp();
      if (!kEarlySelect) {
        if (!last_round) mma_b(tile);
        else select_next(tile);
      }
    }
    if (kEarlySelect && ntiles > 0 && !last_round) mma_b(ntiles - 1);
    }  // segments
    }  // rounds
    if (lane == 0) drain();
  } else if (row_warp) {
    // ================= row warps =================
    // Per tile: the scores' group maxima, the threshold, the ranking of each half-row, the merge of a
    // row's two lists; the first row warp of each quadrant hands the row's picks and their scores
    // to the quadrant's epilogue warp through TMEM, and the row warps go on to the next tile.
    uint32_t hcount = 0;  // tiles handed over (all segments)
    auto wait_live = [&](uint64_t* bar, uint32_t& ph) {
      if (!*s_abort) wait_bar(bar, ph);
    };
    for (r = r0; r < r1; ++r) {
    last_round = r == g.R - 1;
    for (int u = split.start[cta]; u < u_end; u = next_segment()) {
    set_segment(u);
    for (int tile = 0; tile < ntiles; ++tile) {
      const int n0 = t_beg + tile * kTile;
      const int n = n0 + row;
      const bool valid = n < t_end;

      // ---- scores of this tile ----
      wait_live(bar_s, ph_s);
      const bool aborting = __any_sync(0xffffffffu, *s_abort != 0);  // warp-uniform
      const int lim = g.causal ? min(g.M, n + 1) : g.M;               // columns >= lim score -inf
      const int col0 = 128 * part;
      const bool mask_warp = __any_sync(0xffffffffu, lim < col0 + 128);

      // pass 1: 16 group maxima of this thread's 128 scores, top 8 published in TMEM.
      // Groups of 8 slots at stride 16: diffusion makes neighbouring slots alike, so
      // contiguous groups would cluster the top scores and weaken the bound below.
      auto load2 = [&](int c, float (&x0)[32], float (&x1)[32]) {  // chunks c, c+1 of this thread's half, masked
        tmem_ld32(tmem + lane_base + tc::COL_S + col0 + 32 * c, x0);
        tmem_ld32(tmem + lane_base + tc::COL_S + col0 + 32 * c + 32, x1);
        tmem_wait_ld();
        if (mask_warp) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            x0[i] = (col0 + 32 * c + i < lim) ? x0[i] : -INFINITY;
            x1[i] = (col0 + 32 * c + 32 + i < lim) ? x1[i] : -INFINITY;
          }
        }
      };
      if (!aborting) {
        float gm[16];
#pragma unroll
        for (int c = 0; c < 4; c += 2) {
          float x0[32], x1[32];
          load2(c, x0, x1);
#pragma unroll
          for (int gq = 0; gq < 16; ++gq) {
            const float y = tc::max3(x0[gq], x0[gq + 16], x1[gq]);
            gm[gq] = c ? tc::max3(y, x1[gq + 16], gm[gq]) : fmaxf(y, x1[gq + 16]);
          }
        }
        float ga[8], gb[8], top8[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          ga[j] = gm[j];
          gb[j] = gm[8 + j];
        }
        tc::sort8_desc(ga);
        tc::sort8_desc(gb);
        tc::merge8_desc(ga, gb, top8);
        tmem_st8(tmem + lane_base + tc::COL_X + 8 * part, top8);
        tmem_wait_st();
      }
      tc_fence_before();
      tc::quadrant_sync(quadrant);
      tc_fence_after();

      // pass 2: threshold = 7th largest group maximum of the row. The row's top 7 are among its
      // scores >= it; each thread ranks its own (a handful) into a top-7 list: the scores come
      // back from TMEM 64 at a time, bit masks per 32 columns, one select-tree read per set bit.
      float thr = -INFINITY;
      bool exact_scan = false;  // same for both threads of a row
      uint32_t tkey[kTopK];     // this thread's best 7, in rank order (key 0 = empty)
      int tslot[kTopK];
#pragma unroll
      for (int j = 0; j < kTopK; ++j) {
        tkey[j] = 0u;
        tslot[j] = 0;
      }
      bool scan = false;
      if (!aborting) {
        float lst[16];
        tmem_ld16(tmem + lane_base + tc::COL_X, lst);
        tmem_wait_ld();
        float all8[8];
        tc::merge8_desc(&lst[0], &lst[8], all8);
        thr = all8[kTopK - 1];
        // rows with fewer than 7 finite group maxima (causal rows near the start) scan exactly
        exact_scan = valid && !(thr > -INFINITY);
        scan = valid && !exact_scan;
      }
      // The second chunk load below is the last read of this tile's scores: a warp with no
      // exact-scan row frees them for SELECT(i+1) there, so the next tile's scores are computed
      // while the row warps finish ranking; the others free them after the scan.
      const bool scan_warp = __any_sync(0xffffffffu, exact_scan);
      bool s_freed = false;  // warp-uniform
      auto rank_chunks = [&](int c) {  // columns 32c .. 32c+63 of this thread's half
        float x[2][32];
        load2(c, x[0], x[1]);
        if (kEarlySelect && c == 2 && !scan_warp) {
          tc_fence_before();
          tc::group_arrive<tc::kBarSfree, tc::kCountS>();  // SELECT(i+1) may overwrite the scores
          s_freed = true;
        }
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          uint32_t msk = scan ? tc::ge_mask32(x[k], thr) : 0u;
          while (__any_sync(0xffffffffu, msk != 0)) {
            // uniform body, lowest column first; a lane with no bit left offers key 0 (no change)
            const int bit = __ffs(msk) - 1;
            const uint32_t key = rank_key(tc::pick32(x[k], bit & 31));
            tc::offer7_asc(tkey, tslot, msk ? key : 0u, col0 + 32 * (c + k) + bit);
            msk &= msk - 1;
          }
        }
      };
      if (!aborting) {
        rank_chunks(0);
        rank_chunks(2);
      }

      // pass 3 (the row's first thread): rows with fewer than 7 finite group maxima
      float mraw[kTopK];  // raw scores of the first masked columns lim..lim+6 (picked by causal rows n < 6)
#pragma unroll
      for (int j = 0; j < kTopK; ++j) mraw[j] = 0.f;
      if (!aborting && part == 0 && scan_warp) {  // warp-uniform
        // Rows with fewer than 7 finite group maxima have fewer than 7 finite scores: causal
        // rows n < 6, lim = n + 1 <= 6 (every column below 7 is in a group of its own). Their
        // picks are all lim finite columns and then the first masked ones in slot order (equal
        // -inf keys, lower slot first), so only columns below lim + 7 <= 13 (the first thread's
        // half) need a look.
        float w32[32];
        tmem_ld32(tmem + lane_base + tc::COL_S, w32);
        tmem_wait_ld();
        if (exact_scan) {  // rare path: kept compact (not unrolled)
          const int mend = min(g.M, lim + kTopK);
#pragma unroll 1
          for (int m = 0; m < mend; ++m) {
            if (m < lim) {
              tc::offer7_asc(tkey, tslot, rank_key(w32[m]), m);
            } else {
#pragma unroll
              for (int j = 0; j < kTopK; ++j) mraw[j] = (m == lim + j) ? w32[m] : mraw[j];
              tc::offer7_asc(tkey, tslot, kNegInfKey, m);
            }
          }
        }
      }
      if (kEarlySelect && !s_freed) {
        tc_fence_before();
        tc::group_arrive<tc::kBarSfree, tc::kCountS>();  // SELECT(i+1) may overwrite the scores
      }
      // hand-over to the quadrant's epilogue warp, which merges the row's two lists: the first
      // thread's through TMEM (keys, packed slots; an exact-scan row's final picks and scores,
      // flagged), the second thread's through shared memory; the epilogue warp has read the
      // previous tile's
      if (hcount > 0 && !*s_abort && !tc::timed_wait(&hand_free[quadrant], (hcount - 1) & 1)) fail(tc::kErrMmaWait);
      if (part == 0) {  // warp-uniform
        uint32_t hv[16];
        uint32_t s0 = 0, s1 = 0;
#pragma unroll
        for (int j = 0; j < kTopK; ++j) {
          const uint32_t pk = (valid && !aborting) ? (uint32_t)tslot[j] : 0u;
          if (j < 4) s0 |= pk << (8 * j);
          else s1 |= pk << (8 * (j - 4));
          const uint32_t kk = tkey[j];
          if (exact_scan) {  // masked picks (causal rows n < 6) attend with their real score (reference.py:61)
            float sc = __uint_as_float((kk & 0x80000000u) ? (kk & 0x7FFFFFFFu) : ~kk);
            if ((int)pk >= lim) {
#pragma unroll
              for (int k2 = 0; k2 < kTopK; ++k2) sc = ((int)pk == lim + k2) ? mraw[k2] : sc;
            }
            hv[j] = __float_as_uint(sc);
          } else {
            hv[j] = kk;
          }
          if (!valid || aborting) hv[j] = 0u;  // score 0 (the row is not written)
        }
        hv[7] = s0;
        hv[8] = s1;
        hv[9] = (exact_scan || !valid || aborting) ? 1u : 0u;  // 1: the list is final (no merge)
#pragma unroll
        for (int j = 10; j < 16; ++j) hv[j] = 0u;
        tc_fence_after();
        tmem_st16(tmem + lane_base + tc::COL_H, hv);
        tmem_wait_st();
        tc_fence_before();
      } else {
#pragma unroll
        for (int j = 0; j < kTopK; ++j) xch[j * kTile + row] = tc::pack_rank(tkey[j], tslot[j]);
      }
      mbar_arrive(&hand_ready[quadrant]);
      ++hcount;
    }
    }  // segments
    if (multi && !last_round) {  // this CTA's finalize shares of round r
      const int p_first = split.start[cta] / split.tpb, p_last = (u_end - 1) / split.tpb;
      for (int p = p_first; p <= p_last; ++p) {
        int first, count;
        fin_range(p, first, count);
        if (cta >= first && cta < first + count) fin_share(p, cta - first, count);
      }
    }
    }  // rounds
  } else if (epi_warp) {
    // ================= epilogue warps =================
    // One thread per token row (TMEM lane) of its quadrant: the softmax of the row's picks, the
    // weight tile P (both 16-bit terms), the round records and the output, while the row warps
    // rank the next tile; at a segment's end, its slot-sum partials.
    uint32_t hcount = 0;
    uint32_t old_off[kTopK];  // P offsets of the previous tile's entries (0: none)
#pragma unroll
    for (int j = 0; j < kTopK; ++j) old_off[j] = 0u;
    auto wait_live = [&](uint64_t* bar, uint32_t& ph) {
      if (!*s_abort) wait_bar(bar, ph);
    };
    for (r = r0; r < r1; ++r) {
    last_round = r == g.R - 1;
    for (int u = split.start[cta]; u < u_end; u = next_segment()) {
    set_segment(u);
    // bf16 inputs: scores, attend outputs and slot sums come out of the MMAs under the pair's
    // scales (q 2^eq, keys 2^ek, values 2^ev): undone exactly here
    const float usq = kConv ? tc::pow2f(-fs.fexp[4 * bh]) : 1.f;
    const float usk = kConv ? tc::pow2f(-fs.fexp[4 * bh + 1]) : 1.f;
    const float usv = kConv ? tc::pow2f(-fs.fexp[4 * bh + 2]) : 1.f;
    for (int tile = 0; tile < ntiles; ++tile) {
      const int n0 = t_beg + tile * kTile;
      const int n = n0 + row;
      const bool valid = n < t_end;
      T* orow = row_ptr(out, os, b, h, valid ? n : n0);
      uint4 prev[8];  // this row's output of the earlier rounds, added to this round's
      if (r && valid) {
#pragma unroll
        for (int i = 0; i < 8; ++i) prev[i] = reinterpret_cast<const uint4*>(orow)[i];
      }
      // the row warps' picks of this tile
      if (!*s_abort && !tc::timed_wait(&hand_ready[quadrant], hcount & 1)) fail(tc::kErrMmaWait);
      ++hcount;
      tc_fence_after();
      float hf[16];
      tmem_ld16(tmem + lane_base + tc::COL_H, hf);
      tmem_wait_ld();
      uint64_t other[8];
#pragma unroll
      for (int j = 0; j < kTopK; ++j) other[j] = xch[j * kTile + row];
      tc_fence_before();
      mbar_arrive(&hand_free[quadrant]);
      const bool aborting = __any_sync(0xffffffffu, *s_abort != 0);  // warp-uniform
      int pick[kTopK];
      float wgt[kTopK];
      uint32_t poff[kTopK];
      {
        const uint32_t s0 = __float_as_uint(hf[7]), s1 = __float_as_uint(hf[8]);
        uint64_t mine[8], top[8];
#pragma unroll
        for (int j = 0; j < kTopK; ++j) {
          pick[j] = (int)(((j < 4 ? s0 : s1) >> (8 * (j & 3))) & 0xffu);
          mine[j] = tc::pack_rank(__float_as_uint(hf[j]), pick[j]);
        }
        if (__float_as_uint(hf[9]) != 0u) {  // final list: an exact-scan row's picks and scores
#pragma unroll
          for (int j = 0; j < kTopK; ++j) wgt[j] = hf[j] * usq * usk * g.scale;
        } else {  // merge the two threads' lists: the row's top 7, ties to the lower slot
          other[7] = mine[7] = 0;
          tc::merge8_rank(mine, other, top);
#pragma unroll
          for (int j = 0; j < kTopK; ++j) {
            const uint32_t kk = tc::rank_score_key(top[j]);
            pick[j] = tc::rank_slot(top[j]);
            wgt[j] = __uint_as_float((kk & 0x80000000u) ? (kk & 0x7FFFFFFFu) : ~kk) * usq * usk * g.scale;
          }
        }
      }
      {
        // softmax with the hardware exponential and one reciprocal: the weights enter P as
        // 16-bit terms and the update sums, where a relative error of ~1e-6 is far below
        // the rounding of those terms and the parity tolerance
        const float mx = fmaxf(fmaxf(fmaxf(wgt[0], wgt[1]), fmaxf(wgt[2], wgt[3])),
                               fmaxf(fmaxf(wgt[4], wgt[5]), wgt[6]));
#pragma unroll
        for (int j = 0; j < kTopK; ++j) wgt[j] = __expf(wgt[j] - mx);
        const float sum = ((wgt[0] + wgt[1]) + (wgt[2] + wgt[3])) + ((wgt[4] + wgt[5]) + wgt[6]);
        const float inv = __frcp_rn(sum);
#pragma unroll
        for (int j = 0; j < kTopK; ++j) {
          wgt[j] *= inv;
          poff[j] = p_off(pick[j]);
        }
      }
      // MMA_B(i-1) still reads the previous tile's P entries and Q buffer (none after the last round)
      if (tile > 0 && !last_round) wait_live(bar_b, ph_b);
      const bool live = valid && !aborting;
      if (!aborting) {
#pragma unroll
        for (int j = 0; j < kTopK; ++j)
          if (old_off[j]) *p_at(old_off[j]) = 0;
        if (valid) {
#pragma unroll
          for (int j = 0; j < kTopK; ++j) *p_at(poff[j]) = tc::to_bits<tc::CT>(wgt[j]);
        }
        fence_proxy_async_smem();
      }
#pragma unroll
      for (int j = 0; j < kTopK; ++j) old_off[j] = live ? poff[j] : 0u;
      tc_fence_before();
      tc::group_arrive<tc::kBarPhi, tc::kCountP>();  // MMA_A(i) may start

      // round records (off the tensor-core path)
      if (live) {
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

      // MMA_A(i) has consumed P_hi and left the attend output in TMEM
      wait_live(bar_a, ph_a);
      const bool ok = !__any_sync(0xffffffffu, *s_abort != 0);
      if (ok && !last_round) {
        if (valid) {
#pragma unroll
          for (int j = 0; j < kTopK; ++j) {
            const uint16_t hb = tc::to_bits<tc::CT>(wgt[j]);
            *p_at(poff[j]) = tc::to_bits<tc::CT>(wgt[j] - tc::from_bits<tc::CT>(hb));
          }
        }
        fence_proxy_async_smem();
      }
      tc_fence_before();
      if (!last_round) tc::group_arrive<tc::kBarPlo, tc::kCountP>();  // MMA_B(i) may start
      // ---- output: out (+)= O, 64 columns ----
      if (ok) {
#pragma unroll
        for (int hc = 0; hc < 2; ++hc) {
          float o[32];
          tmem_ld32(tmem + lane_base + tc::COL_O + 32 * hc, o);
          tmem_wait_ld();
          if (kConv) {
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= usv;
          }
          if (valid) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint32_t pk[4];
              const uint32_t* pv = reinterpret_cast<const uint32_t*>(&prev[4 * hc + i]);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 a = r ? tc::unpack2<T>(pv[e]) : make_float2(0.f, 0.f);
                pk[e] = tc::pack2<T>(a.x + o[8 * i + 2 * e], a.y + o[8 * i + 2 * e + 1]);
              }
              reinterpret_cast<uint4*>(orow)[4 * hc + i] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            }
          }
        }
      }
      tc_fence_before();  // the output's TMEM reads come before the next MMA_A
    }
    if (last_round) continue;  // no slot update follows
    if (ntiles > 0) wait_live(bar_b, ph_b);

    // ---- the segment's partials: TMEM lanes are slots here ----
    if (!__any_sync(0xffffffffu, *s_abort != 0)) {
      const size_t po = (size_t)bh * g.ft_parts + part_idx;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int m = 128 * hh + row;
#pragma unroll
        for (int hc = 0; hc < 2; ++hc) {
          float s32[32];
          tmem_ld32(tmem + lane_base + tc::COL_U + tc::kUW * hh + 32 * hc, s32);
          tmem_wait_ld();
          if (kConv) {
#pragma unroll
            for (int i = 0; i < 32; ++i) s32[i] *= usq;
          }
          if (m < g.M) {  // chunk-major: a warp's store of one 4-column chunk covers 32 consecutive rows
            float4* dst = reinterpret_cast<float4*>(fs.Spart) + (po * 16 + 8 * hc) * g.M + m;
#pragma unroll
            for (int i = 0; i < 8; ++i)
              dst[(size_t)i * g.M] = make_float4(s32[4 * i], s32[4 * i + 1], s32[4 * i + 2], s32[4 * i + 3]);
          }
        }
        float wv[16];
        tmem_ld16(tmem + lane_base + tc::COL_U + tc::kUW * hh + 64, wv);
        tmem_wait_ld();
        if (m < g.M) fs.Wpart[po * g.M + m] = wv[0];
      }
    }
    tc_fence_before();  // the partials' TMEM reads come before the next segment's MMAs
    if (multi) {  // the partial is written: count it for the pair's finalize (even after a failure)
      asm volatile("bar.sync %0, %1;" ::"n"(tc::kBarEpi), "n"(tc::kEpiThreads) : "memory");
      if (tid == tc::kRowThreads) {
        __threadfence();
        counter_release_add(&cnt_part[bh], 1);
      }
    }
    }  // segments
    }  // rounds
  } else if (kConv && warp > tc::kIssuerWarp) {
    // ================= warps 13-15, bf16 inputs =================
    // Each token tile of q, once loaded, converted in place to fp16 under the pair's scale (the
    // Q buffers are loaded and read in the issuer's order: tile i of a segment into buffer i % 3).
    const int ct = tid - (tc::kIssuerWarp + 1) * 32;  // 0..95
    uint32_t cph[3] = {0, 0, 0};
    for (r = r0; r < r1; ++r) {
    for (int u = split.start[cta]; u < u_end; u = next_segment()) {
    set_segment(u);
    const float sq = tc::pow2f(fs.fexp[4 * bh]);
    for (int tile = 0; tile < ntiles; ++tile) {
      const int bs = tile % C::kQBufs;
      if (!*s_abort && !tc::timed_wait(&bar_q[bs], cph[bs])) fail(tc::kErrQWait);
      cph[bs] ^= 1;
      if (!*s_abort) {
        uint4* qb = reinterpret_cast<uint4*>(sm + L::OFF_Q + bs * tc::kQBytes);
#pragma unroll 2
        for (int c = ct; c < (int)(tc::kQBytes / 16); c += 96) qb[c] = tc::bf16_to_f16_scaled(qb[c], sq);
        fence_proxy_async_smem();  // generic writes, read by the MMAs (async proxy)
      }
      mbar_arrive(&q_conv[bs]);
    }
    }  // segments
    }  // rounds
  }
  // ---- wind down: wait (bounded) for copies still in flight, free TMEM ----
  if (issuer_warp && lane == 0) {
    if (img_pending) tc::timed_wait(bar_img, img_phase);
    for (int i = 0; i < 3; ++i)
      if (q_pending[i]) tc::timed_wait(&bar_q[i], q_phase[i]);
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

PFN_cuTensorMapEncodeTiled_v12000 tc_tensor_map_encoder() { return get_encode(); }

size_t tc_images_bytes(const Geom& g) {
  if (g.D != tc::kD) return 0;
  if (g.dtype == MURM_F16 || g.dtype == MURM_BF16) return (size_t)g.BH * tc::Layout<tc::CT>::kImages;
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

// Failure-detection probe: one warp waits, bounded by `limit_ns`, on an mbarrier of its own. With
// `arrive` set a thread arrives first and the wait ends at once; without it nothing arrives, the
// wait runs out and the kernel records kErrProbe in the device error word, as the round kernels do
// when a copy or an MMA never completes, then returns normally (no trap, no fault).
__global__ void k_wait_probe(int arrive, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (arrive) mbar_arrive(&bar);
    if (!mbar_timed_wait(&bar, 0, limit_ns)) atomicOr(&g_device_error, kErrProbe);
  }
}

cudaError_t launch_wait_probe(int arrive, uint64_t limit_ns, cudaStream_t st) {
  MURM_LAUNCH("wait_probe", k_wait_probe, 1, 32, 0, st, arrive, limit_ns);
  return cudaGetLastError();
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
  constexpr uint32_t kSmem = tc::Layout<tc::CT>::kSmem;
  if (cudaError_t e = smem_opt_in(k_fwd_tc<T>, kSmem)) return e;
  constexpr bool kConv = !std::is_same<T, __half>::value;
  if (p.slots_f32) {
    if (kConv)
      MURM_LAUNCH_PDL("tc_amax", (k_tc_amax<T, float>), dim3(g.BH, kAmaxBlocks), 256, 0, st, g, static_cast<const T*>(p.q),
                      p.qs, static_cast<const float*>(p.sk), p.sks, static_cast<const float*>(p.sv), p.svs, fs.amax);
    MURM_LAUNCH_PDL("tc_load", (k_tc_load<T, float>), dim3(g.BH, kSlotBlocks), tc::kRowLanes * kSlotRows, 0, st, g,
                    static_cast<const float*>(p.sk), p.sks, static_cast<const float*>(p.sv), p.svs, sv, images,
                    fs.counters, fs.amax, fs.fexp);
  } else {
    if (kConv)
      MURM_LAUNCH_PDL("tc_amax", (k_tc_amax<T, T>), dim3(g.BH, kAmaxBlocks), 256, 0, st, g, static_cast<const T*>(p.q), p.qs,
                      static_cast<const T*>(p.sk), p.sks, static_cast<const T*>(p.sv), p.svs, fs.amax);
    MURM_LAUNCH_PDL("tc_load", (k_tc_load<T, T>), dim3(g.BH, kSlotBlocks), tc::kRowLanes * kSlotRows, 0, st, g,
                    static_cast<const T*>(p.sk), p.sks, static_cast<const T*>(p.sv), p.svs, sv, images, fs.counters,
                    fs.amax, fs.fexp);
  }
  TileSplit split;  // the plan the workspace was sized for (make_geom)
  plan_split(g.BH, g.N, kTile, kMaxSplitCtas, &split);
  // All rounds in one launch when every CTA can be resident at once (a cooperative launch): the
  // CTAs wait on each other between rounds. Otherwise one launch per round, with k_tc_finalize
  // between them. MURM_FWD_LAUNCH_PER_ROUND=1 forces the latter.
  const char* per_round = getenv("MURM_FWD_LAUNCH_PER_ROUND");
  if (g.R > 1 && !(per_round && per_round[0] == '1') &&
      coop_fits(reinterpret_cast<const void*>(k_fwd_tc<T>), tc::kThreads, kSmem, split.G)) {
    MURM_LAUNCH_COOP_PDL("select_attend_update_tc", k_fwd_tc<T>, dim3(split.G), tc::kThreads, kSmem, st,
                         g, 0, g.R, qmap, static_cast<T*>(p.out), p.os, p.indices, p.weights, sv, fs, split);
    return cudaGetLastError();
  }
  for (int r = 0; r < g.R; ++r) {
    MURM_LAUNCH_PDL("select_attend_update_tc", k_fwd_tc<T>, dim3(split.G), tc::kThreads, kSmem, st, g, r,
                r + 1, qmap, static_cast<T*>(p.out), p.os, p.indices, p.weights, sv, fs, split);
    if (r + 1 < g.R)
      MURM_LAUNCH_PDL("tc_finalize", k_tc_finalize<T>, dim3(g.BH, kSlotBlocks), tc::kRowLanes * kSlotHalo, 0, st, g, r, sv, fs,
                      split);
  }
  return cudaGetLastError();
}

template cudaError_t fwd_tc<__half>(const Geom&, const FwdPtrs&, const Saved&, const FwdScratch&, cudaStream_t);
template cudaError_t fwd_tc<__nv_bfloat16>(const Geom&, const FwdPtrs&, const Saved&, const FwdScratch&,
                                           cudaStream_t);

}  // namespace murm
