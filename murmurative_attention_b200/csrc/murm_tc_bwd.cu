// murm_tc_bwd.cu — backward of the round loop for fp16/bf16, head_dim 64:
// CUDA-core token math + tcgen05 slot scatters.
//
// Reverse-mode of reference.py:177-189 (autograd through reference.py:42-68,
// 71-115, 118-135). For round r, with G = dL/d out (the same for every round
// because out = sum of the rounds' attend outputs):
//   dw_j = G . V[i_j] + q . dS[i_j] + dW[i_j]  (+ dL/d weights in the last round)
//   da_j = w_j (dw_j - sum_k w_k dw_k)                       (softmax adjoint)
//   dq  += sum_j w_j dS[i_j] + scale da_j K[i_j]
//   dK_r = dKdir_r + sum over picks of scale da_j q          (slot scatter)
//   dV_r = dVdir_r + sum over picks of w_j G                 (slot scatter)
// with dS = dU / (W + eps), dW = -(dU . U) / (W + eps), dU = (1-alpha)(dK' + dV')
// on slots that received picks, dK' = D^T dK_{r+1} (diffusion adjoint), and
// dKdir = alpha dK' (or dK' on slots without picks).
//
// k_bwd_tokens_tc: one CTA per (batch, head) and token chunk, 16 warps. Eight
// lanes share a token (8 head dims each), a warp takes 4 tokens of a 64-token
// tile; the slot tables K_r, V_r, dS_r (16-bit) and dW_r sit in shared memory.
// The slot scatters are dense tensor-core products over a 64 x 256 tile P that
// holds the 7 picks of every token: dV += P^T . G with P = w, then
// dK += P^T . Q with P = scale da, accumulated in TMEM over the chunk —
// deterministic, no atomics. P is double-buffered, so a tile's dK scatter runs
// under the next tile's token math.
// k_bwd_slots: finalize of round r (direct part + chunk partials, in chunk
// order) fused with the per-slot adjoints of round r-1, 16 threads per slot row.
#include <cudaTypedefs.h>

#include "murm_kernels.cuh"
#include "murm_sm100.cuh"

namespace murm {
using namespace sm100;

extern __device__ int g_device_error;

namespace tcb {
constexpr int kD = 64;
constexpr int kSlotsPad = 256;
constexpr int kMathWarps = 16;              // token math (and the tiles' records)
constexpr int kThreads = 32 * kMathWarps + 32;  // + one issuer warp
constexpr int kIssuer = 32 * kMathWarps;    // the thread that issues the MMAs and copies
constexpr uint32_t kTable = kSlotsPad * kD * 2;  // one [256][64] 16-bit table
constexpr uint32_t OFF_K = 0, OFF_V = kTable, OFF_DS = 2 * kTable;
constexpr uint32_t kTables = 3 * kTable;
constexpr int kBTile = kBwdTile;                     // tokens per tile of the token kernel
constexpr uint32_t kTileBytes = kBTile * 128;        // one [64][64] 16-bit swizzled TMA tile
constexpr uint32_t kPBlock = kBTile * 128;           // P block: [64 tokens][64 slots], swizzled
constexpr uint32_t kPBuf = 4 * kPBlock;              // P of one tile: 256 slots
constexpr uint32_t OFF_DW = kTables;                 // fp32 [256]
constexpr uint32_t OFF_P = OFF_DW + 1024;            // P[2] by tile parity (1024-aligned)
constexpr uint32_t OFF_Q = OFF_P + 2 * kPBuf;        // q tiles [3] by tile mod 3 (MMA operand)
constexpr uint32_t OFF_G = OFF_Q + 3 * kTileBytes;   // grad_out tiles [3] by tile mod 3
constexpr uint32_t OFF_TW = OFF_G + 3 * kTileBytes;  // fp32 [3][64][8] weights of the tiles' tokens
constexpr uint32_t OFF_COEF = OFF_TW + 3 * kBTile * 32;  // fp32 [64][8] scale*da per pick
constexpr uint32_t OFF_TGW = OFF_COEF + kBTile * 32;     // fp32 [2][64][8] dL/d weights (last round)
constexpr uint32_t OFF_TIX = OFF_TGW + 2 * kBTile * 32;  // u8 [2][64][8] picks
constexpr uint32_t OFF_MISC = OFF_TIX + 2 * kBTile * 8;
constexpr uint32_t kSmem = OFF_MISC + 128 + 1024;
static_assert(kSmem <= 232448, "shared memory budget");
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t COL_DV = 0, COL_DK = 128;
enum : int { kErrWait = 8 };

__device__ __forceinline__ bool timed_wait(uint64_t* bar, uint32_t parity) { return mbar_timed_wait(bar, parity); }

// acc += sum over i = 0..7 of a_i * b_i for two runs of eight 16-bit values (one uint4
// each), in order; each product is exact and added with one rounding (fp32 fma on the
// 16-bit operands: the same result as converting both to fp32 first, in fewer instructions).
#define MURM_DOT8(TY)                                                                                    \
  asm("{\n .reg .b16 a0, a1, b0, b1;\n"                                                                \
      " mov.b32 {a0, a1}, %1;\n mov.b32 {b0, b1}, %5;\n fma.rn.f32." TY " %0, a0, b0, %0;\n"          \
      " fma.rn.f32." TY " %0, a1, b1, %0;\n"                                                            \
      " mov.b32 {a0, a1}, %2;\n mov.b32 {b0, b1}, %6;\n fma.rn.f32." TY " %0, a0, b0, %0;\n"          \
      " fma.rn.f32." TY " %0, a1, b1, %0;\n"                                                            \
      " mov.b32 {a0, a1}, %3;\n mov.b32 {b0, b1}, %7;\n fma.rn.f32." TY " %0, a0, b0, %0;\n"          \
      " fma.rn.f32." TY " %0, a1, b1, %0;\n"                                                            \
      " mov.b32 {a0, a1}, %4;\n mov.b32 {b0, b1}, %8;\n fma.rn.f32." TY " %0, a0, b0, %0;\n"          \
      " fma.rn.f32." TY " %0, a1, b1, %0;\n}"                                                           \
      : "+f"(acc)                                                                                        \
      : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w))
template <typename T>
__device__ __forceinline__ float dot8(const uint4& a, const uint4& b, float acc);
template <>
__device__ __forceinline__ float dot8<__half>(const uint4& a, const uint4& b, float acc) {
  MURM_DOT8("f16");
  return acc;
}
template <>
__device__ __forceinline__ float dot8<__nv_bfloat16>(const uint4& a, const uint4& b, float acc) {
  MURM_DOT8("bf16");
  return acc;
}
#undef MURM_DOT8

// acc[i] += x * row_i over eight 16-bit values, each product an fp32 fma on 16-bit operands.
// fp16: x rounded to fp16 (the precision the fp16 scatter MMAs use for the same weights); bf16:
// x as two bf16 terms, which keeps x's rounding well below the bf16 rows' own.
template <typename T>
__device__ __forceinline__ void axpy8(float x, const uint4& row, float (&acc)[8]);
template <>
__device__ __forceinline__ void axpy8<__half>(float x, const uint4& row, float (&acc)[8]) {
  const uint16_t xh = __half_as_ushort(__float2half_rn(x));
  asm("{\n .reg .b16 r0, r1;\n"
      " mov.b32 {r0, r1}, %9;\n fma.rn.f32.f16 %0, %8, r0, %0;\n fma.rn.f32.f16 %1, %8, r1, %1;\n"
      " mov.b32 {r0, r1}, %10;\n fma.rn.f32.f16 %2, %8, r0, %2;\n fma.rn.f32.f16 %3, %8, r1, %3;\n"
      " mov.b32 {r0, r1}, %11;\n fma.rn.f32.f16 %4, %8, r0, %4;\n fma.rn.f32.f16 %5, %8, r1, %5;\n"
      " mov.b32 {r0, r1}, %12;\n fma.rn.f32.f16 %6, %8, r0, %6;\n fma.rn.f32.f16 %7, %8, r1, %7;\n}"
      : "+f"(acc[0]), "+f"(acc[1]), "+f"(acc[2]), "+f"(acc[3]), "+f"(acc[4]), "+f"(acc[5]), "+f"(acc[6]),
        "+f"(acc[7])
      : "h"(xh), "r"(row.x), "r"(row.y), "r"(row.z), "r"(row.w));
}
template <>
__device__ __forceinline__ void axpy8<__nv_bfloat16>(float x, const uint4& row, float (&acc)[8]) {
  // x as two bf16 terms (16 significant bits), each product an fp32 fma on the 16-bit operands
  const __nv_bfloat16 xh = __float2bfloat16_rn(x);
  const uint16_t h0 = __bfloat16_as_ushort(xh), h1 = __bfloat16_as_ushort(__float2bfloat16_rn(x - __bfloat162float(xh)));
  asm("{\n .reg .b16 r0, r1;\n"
      " mov.b32 {r0, r1}, %10;\n fma.rn.f32.bf16 %0, %8, r0, %0;\n fma.rn.f32.bf16 %1, %8, r1, %1;\n"
      " fma.rn.f32.bf16 %0, %9, r0, %0;\n fma.rn.f32.bf16 %1, %9, r1, %1;\n"
      " mov.b32 {r0, r1}, %11;\n fma.rn.f32.bf16 %2, %8, r0, %2;\n fma.rn.f32.bf16 %3, %8, r1, %3;\n"
      " fma.rn.f32.bf16 %2, %9, r0, %2;\n fma.rn.f32.bf16 %3, %9, r1, %3;\n"
      " mov.b32 {r0, r1}, %12;\n fma.rn.f32.bf16 %4, %8, r0, %4;\n fma.rn.f32.bf16 %5, %8, r1, %5;\n"
      " fma.rn.f32.bf16 %4, %9, r0, %4;\n fma.rn.f32.bf16 %5, %9, r1, %5;\n"
      " mov.b32 {r0, r1}, %13;\n fma.rn.f32.bf16 %6, %8, r0, %6;\n fma.rn.f32.bf16 %7, %8, r1, %7;\n"
      " fma.rn.f32.bf16 %6, %9, r0, %6;\n fma.rn.f32.bf16 %7, %9, r1, %7;\n}"
      : "+f"(acc[0]), "+f"(acc[1]), "+f"(acc[2]), "+f"(acc[3]), "+f"(acc[4]), "+f"(acc[5]), "+f"(acc[6]),
        "+f"(acc[7])
      : "h"(h0), "h"(h1), "r"(row.x), "r"(row.y), "r"(row.z), "r"(row.w));
}

// bf16 operands of the scatter MMAs as fp16 under a per-(b,h) power-of-two scale s: the largest
// |x| of the pair maps into [2^14, 2^15), so every bf16 value of the pair (8 significant bits)
// converts exactly unless it lies below 2^-39 of the largest (an fp16 subnormal, rounded).
__device__ __forceinline__ float absmax8_bf16(const uint4& u) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    m = fmaxf(m, fmaxf(__uint_as_float((w[i] & 0x7FFFu) << 16), __uint_as_float(w[i] & 0x7FFF0000u)));
  return m;
}
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
// 2^e for e in [-126, 126] (exact)
__device__ __forceinline__ float pow2i(int e) { return __uint_as_float((uint32_t)(e + 127) << 23); }
// the scale exponent for a pair whose largest |x| is m: m * 2^e in [2^14, 2^15)
__device__ __forceinline__ int scale_exp(float m) {
  if (!(m > 0.f)) return 0;
  const int ex = (int)((__float_as_uint(m) >> 23) & 0xffu) - 127;
  return max(-126, min(126, 14 - ex));
}

template <typename T> struct Fmt;
template <> struct Fmt<__half> { static constexpr uint32_t v = 0; };
template <> struct Fmt<__nv_bfloat16> { static constexpr uint32_t v = 1; };

template <typename T>
__device__ __forceinline__ uint16_t bits(float x) {
  T h;
  Elem<T>::store(&h, x);
  return *reinterpret_cast<uint16_t*>(&h);
}
// two consecutive 16-bit values -> float2
template <typename T>
__device__ __forceinline__ float2 load2(const void* p) {
  const T* t = reinterpret_cast<const T*>(p);
  return make_float2(Elem<T>::load(t), Elem<T>::load(t + 1));
}

// 8 consecutive 16-bit values (16 bytes, aligned) -> 8 floats
template <typename T>
__device__ __forceinline__ void load8(const void* p, float (&f)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const T* t = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = Elem<T>::load(t + i);
}

// Within each group of 8 lanes, sum each of v[0..7] over the group; on return
// every lane of the group holds all 8 sums.
__device__ __forceinline__ void group8_sum8(float (&v)[8]) {
  const int c = threadIdx.x & 7;
#pragma unroll
  for (int s = 4, n = 4; s >= 1; s >>= 1, n >>= 1) {
    const bool upper = (c & s) != 0;
#pragma unroll
    for (int k = 0; k < n; ++k) {
      const float send = upper ? v[k] : v[k + n];
      const float keep = upper ? v[k + n] : v[k];
      v[k] = keep + __shfl_xor_sync(0xffffffffu, send, s);
    }
  }
  // lane c of the group now holds the total of value index c
  const float x = v[0];
  const int base = threadIdx.x & 24;
#pragma unroll
  for (int j = 0; j < 8; ++j) v[j] = __shfl_sync(0xffffffffu, x, base + j);
}

// Sum each of v[0..7] over the 32 lanes; on return every lane holds all 8 sums.
__device__ __forceinline__ void warp_sum8(float (&v)[8]) {
  const int lane = threadIdx.x & 31;
  // transpose-reduce: halve the set of values per lane at each step
#pragma unroll
  for (int s = 16, n = 4; s >= 4; s >>= 1, n >>= 1) {
    const bool upper = (lane & s) != 0;
#pragma unroll
    for (int k = 0; k < n; ++k) {
      const float send = upper ? v[k] : v[k + n];
      const float keep = upper ? v[k + n] : v[k];
      v[k] = keep + __shfl_xor_sync(0xffffffffu, send, s);
    }
  }
  float x = v[0];
  x += __shfl_xor_sync(0xffffffffu, x, 2);
  x += __shfl_xor_sync(0xffffffffu, x, 1);
  // lane l now holds the total of value index ((l>>4)&1)*4 + ((l>>3)&1)*2 + ((l>>2)&1)
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int src = ((j >> 2) & 1) * 16 + ((j >> 1) & 1) * 8 + (j & 1) * 4;
    v[j] = __shfl_sync(0xffffffffu, x, src);
  }
}
}  // namespace tcb

// ---------------------------------------------------------------------------
// Slot side: finalize round r (dK_r, dV_r) and, for r > 0, the adjoints of
// round r-1 (dS, dW, direct parts) plus its 16-bit tables for the token kernel.
// grid (BH, ceil(M/16)), 288 threads: 16 threads per slot row (4 dims each,
// 16-byte accesses), rows m0-1 .. m0+16 (one diffusion halo row on each side).
// ---------------------------------------------------------------------------
// Direct parts live in bs.dK[r & 1] / bs.dV[r & 1] (round parity): a block reads
// its neighbours' rows of round r while they write round r-1.
namespace tcb {
constexpr int kRowLanes = 16;
__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ void st4(float* p, float4 x) { *reinterpret_cast<float4*>(p) = x; }
__device__ __forceinline__ void add4(float4& a, float4 b) { a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w; }
// a + c * b, each product and sum rounded (reference.py:128-133 transposed)
__device__ __forceinline__ float4 axpy4(float4 a, float c, float4 b) {
  return make_float4(__fadd_rn(a.x, __fmul_rn(c, b.x)), __fadd_rn(a.y, __fmul_rn(c, b.y)),
                     __fadd_rn(a.z, __fmul_rn(c, b.z)), __fadd_rn(a.w, __fmul_rn(c, b.w)));
}
__device__ __forceinline__ float4 scale4(float c, float4 b) {
  return make_float4(__fmul_rn(c, b.x), __fmul_rn(c, b.y), __fmul_rn(c, b.z), __fmul_rn(c, b.w));
}
template <typename T>
__device__ __forceinline__ uint2 pack4(float4 x) {
  return make_uint2(bits<T>(x.x) | ((uint32_t)bits<T>(x.y) << 16), bits<T>(x.z) | ((uint32_t)bits<T>(x.w) << 16));
}
}  // namespace tcb

template <typename T>
__global__ void __launch_bounds__(tcb::kRowLanes * kSlotHalo, 2)
    k_bwd_slots(Geom g, int r, int has_dir, int has_part, Saved sv, BwdScratch bs, uint8_t* tables, float* dWpad,
                T* gsk, Strides3 gsks, T* gsv, Strides3 gsvs) {
  pdl_wait();  // the token kernel's chunk partials
  pdl_trigger();
  const float* dir_k = bs.dK[r & 1];
  const float* dir_v = bs.dV[r & 1];
  float* nxt_k = bs.dK[(r + 1) & 1];  // direct parts of round r-1
  float* nxt_v = bs.dV[(r + 1) & 1];
  __shared__ float4 skk[kSlotHalo][tcb::kRowLanes];  // dK_r rows m0-1 .. m0+16
  __shared__ float4 svv[kSlotHalo][tcb::kRowLanes];
  const int bh = blockIdx.x, b = bh / g.H, h = bh - b * g.H;
  const int rr = threadIdx.x >> 4, l = threadIdx.x & 15;
  const int m = blockIdx.y * kSlotRows - 1 + rr;
  const size_t MD = (size_t)g.M * g.D;
  // 1. dK_r, dV_r for the block and its halo, every chunk load of a row in flight at once. Here a
  // thread takes row m0-1+t%18, columns 4*(t/18).. (consecutive threads, consecutive rows of one
  // column chunk: the chunk-major partials load coalesced); the rest of the kernel reads the rows
  // back from shared memory with 16 threads per row.
  {
    const int rr2 = threadIdx.x % kSlotHalo, l2 = threadIdx.x / kSlotHalo;
    const int m2 = blockIdx.y * kSlotRows - 1 + rr2;
    float4 k = make_float4(0.f, 0.f, 0.f, 0.f), v = k;
    if (m2 >= 0 && m2 < g.M) {
      const size_t e = bh * MD + (size_t)m2 * g.D + 4 * l2;
      if (has_dir) {
        k = tcb::ld4(dir_k + e);
        v = tcb::ld4(dir_v + e);
      }
      if (has_part) {
        for (int ch = 0; ch < g.bwd_chunks; ch += 8) {  // added in chunk order
          float4 a[8], c[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            // chunk partials are chunk-major: [BH][chunks][16 column chunks][M][4]
            const size_t po = (((size_t)bh * g.bwd_chunks + min(ch + u, g.bwd_chunks - 1)) * 16 + l2) * g.M + m2;
            a[u] = reinterpret_cast<const float4*>(bs.dKpart)[po];
            c[u] = reinterpret_cast<const float4*>(bs.dVpart)[po];
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            if (ch + u < g.bwd_chunks) {
              tcb::add4(k, a[u]);
              tcb::add4(v, c[u]);
            }
          }
        }
      }
    }
    skk[rr2][l2] = k;
    svv[rr2][l2] = v;
  }
  __syncthreads();
  if (rr < 1 || rr > kSlotRows || m >= g.M) return;  // uniform per half warp
  if (r == 0) {  // the slot gradients
    T* pk = row_ptr(gsk, gsks, b, h, m) + 4 * l;
    T* pv = row_ptr(gsv, gsvs, b, h, m) + 4 * l;
    const float4 k = skk[rr][l], v = svv[rr][l];
    Elem<T>::store(pk, k.x);
    Elem<T>::store(pk + 1, k.y);
    Elem<T>::store(pk + 2, k.z);
    Elem<T>::store(pk + 3, k.w);
    Elem<T>::store(pv, v.x);
    Elem<T>::store(pv + 1, v.y);
    Elem<T>::store(pv + 2, v.z);
    Elem<T>::store(pv + 3, v.w);
    return;
  }
  // 2. adjoints of round r-1 for slots of this block
  const int rp = r - 1;
  const size_t st = ((size_t)rp * g.BH + bh) * MD + (size_t)m * g.D + 4 * l;
  const float W = sv.W[((size_t)rp * g.BH + bh) * g.M + m];
  const float4 U = tcb::ld4(sv.U + st);
  const float4 K = tcb::ld4(sv.K + st);
  const float4 V = tcb::ld4(sv.V + st);
  const bool in_m = m > 0 && m < g.M - 1, in_l = m - 1 > 0, in_r = m + 1 < g.M - 1;
  float4 ak = skk[rr][l], av = svv[rr][l];
  if (in_m) {
    const float gm2 = -2.f * g.gamma;
    ak = tcb::axpy4(ak, gm2, ak);
    av = tcb::axpy4(av, gm2, av);
  }
  if (in_l) {
    ak = tcb::axpy4(ak, g.gamma, skk[rr - 1][l]);
    av = tcb::axpy4(av, g.gamma, svv[rr - 1][l]);
  }
  if (in_r) {
    ak = tcb::axpy4(ak, g.gamma, skk[rr + 1][l]);
    av = tcb::axpy4(av, g.gamma, svv[rr + 1][l]);
  }
  const bool hit = W > 0.f;
  const float den = __fadd_rn(W, kEmaEps);
  float4 dU = make_float4(0.f, 0.f, 0.f, 0.f);
  if (hit) {
    dU = make_float4(__fadd_rn(ak.x, av.x), __fadd_rn(ak.y, av.y), __fadd_rn(ak.z, av.z), __fadd_rn(ak.w, av.w));
    dU = tcb::scale4(g.one_minus_alpha, dU);
  }
  float dot = fmaf(dU.x, U.x, fmaf(dU.y, U.y, fmaf(dU.z, U.z, dU.w * U.w)));
  const unsigned half = 0xffffu << (threadIdx.x & 16);
#pragma unroll
  for (int o = 8; o; o >>= 1) dot += __shfl_xor_sync(half, dot, o);
  const float4 dS = make_float4(__fdiv_rn(dU.x, den), __fdiv_rn(dU.y, den), __fdiv_rn(dU.z, den), __fdiv_rn(dU.w, den));
  const size_t e = bh * MD + (size_t)m * g.D + 4 * l;
  tcb::st4(nxt_k + e, hit ? tcb::scale4(g.alpha, ak) : ak);
  tcb::st4(nxt_v + e, hit ? tcb::scale4(g.alpha, av) : av);
  if (l == 0) dWpad[(size_t)bh * tcb::kSlotsPad + m] = -__fdiv_rn(dot, den);
  // 16-bit tables of round r-1 (row-major [256][64])
  uint8_t* tab = tables + (size_t)bh * tcb::kTables;
  const uint32_t off = (uint32_t)m * 128 + 8 * l;
  *reinterpret_cast<uint2*>(tab + tcb::OFF_K + off) = tcb::pack4<T>(K);
  *reinterpret_cast<uint2*>(tab + tcb::OFF_V + off) = tcb::pack4<T>(V);
  *reinterpret_cast<uint2*>(tab + tcb::OFF_DS + off) = tcb::pack4<T>(dS);
}

// Tables of the last round (no slot gradient flows into it): K, V; dS = 0, dW = 0. For bf16 also
// the maxima of |q| and |grad_out| over block y's 1/32 of the pair's tokens (the token kernel's
// operand scales).
template <typename T>
__global__ void __launch_bounds__(256) k_bwd_tables_last(Geom g, Saved sv, uint8_t* tables, float* dWpad, const T* q,
                                                         Strides3 qs, const T* go, Strides3 gos, float* amax) {
  pdl_wait();
  pdl_trigger();
  const int bh = blockIdx.x;
  if constexpr (tcb::Fmt<T>::v == 1) {
    __shared__ float red[2][8];
    const int b = bh / g.H, h = bh - b * g.H;
    const int n0 = (int)((int64_t)g.N * blockIdx.y / gridDim.y), n1 = (int)((int64_t)g.N * (blockIdx.y + 1) / gridDim.y);
    float mq = 0.f, mg = 0.f;
    // four q and four grad_out 16-byte loads in flight per thread: the pass is bound by loads outstanding
    constexpr int kU = 4;
    const int cnt = (n1 - n0) * 8;
    for (int e0 = threadIdx.x; e0 < cnt; e0 += kU * blockDim.x) {
      uint4 uq[kU], ug[kU];
#pragma unroll
      for (int j = 0; j < kU; ++j) {
        const int e = e0 + j * blockDim.x;
        const int n = n0 + (e >> 3), c = (e & 7) * 8;
        uq[j] = e < cnt ? *reinterpret_cast<const uint4*>(row_ptr(q, qs, b, h, n) + c) : make_uint4(0u, 0u, 0u, 0u);
        ug[j] = e < cnt ? *reinterpret_cast<const uint4*>(row_ptr(go, gos, b, h, n) + c) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int j = 0; j < kU; ++j) {
        mq = fmaxf(mq, tcb::absmax8_bf16(uq[j]));
        mg = fmaxf(mg, tcb::absmax8_bf16(ug[j]));
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      mq = fmaxf(mq, __shfl_xor_sync(0xffffffffu, mq, o));
      mg = fmaxf(mg, __shfl_xor_sync(0xffffffffu, mg, o));
    }
    if ((threadIdx.x & 31) == 0) {
      red[0][threadIdx.x >> 5] = mq;
      red[1][threadIdx.x >> 5] = mg;
    }
    __syncthreads();
    if (threadIdx.x < 2) {
      float m = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) m = fmaxf(m, red[threadIdx.x][i]);
      amax[(size_t)bh * 64 + 32 * threadIdx.x + blockIdx.y] = m;
    }
  }
  const size_t st = ((size_t)(g.R - 1) * g.BH + bh) * g.M * g.D;
  uint8_t* tab = tables + (size_t)bh * tcb::kTables;
  for (int e = blockIdx.y * blockDim.x + threadIdx.x; e < tcb::kSlotsPad * 32; e += gridDim.y * blockDim.x) {
    const int m = e >> 5, l = e & 31;
    float2 K = make_float2(0.f, 0.f), V = K;
    if (m < g.M) {
      K = *reinterpret_cast<const float2*>(sv.K + st + (size_t)m * g.D + 2 * l);
      V = *reinterpret_cast<const float2*>(sv.V + st + (size_t)m * g.D + 2 * l);
    }
    const uint32_t off = (uint32_t)m * 128 + 4 * l;
    *reinterpret_cast<uint32_t*>(tab + tcb::OFF_K + off) = tcb::bits<T>(K.x) | ((uint32_t)tcb::bits<T>(K.y) << 16);
    *reinterpret_cast<uint32_t*>(tab + tcb::OFF_V + off) = tcb::bits<T>(V.x) | ((uint32_t)tcb::bits<T>(V.y) << 16);
    *reinterpret_cast<uint32_t*>(tab + tcb::OFF_DS + off) = 0u;
    if (l == 0) dWpad[(size_t)bh * tcb::kSlotsPad + m] = 0.f;
  }
}

// ---------------------------------------------------------------------------
// Token side of round r
// ---------------------------------------------------------------------------
// Tiles of 64 tokens, software-pipelined with one block barrier per tile (fp16):
//   barrier(i) -> issuer: last scatter of tile i-1 + first scatter of tile i, copies of tile i+2
//              -> warps 0-15: token math of tile i; wait for the scatters; coefficients of tile i
//                 into P[i & 1] and the weights of tile i+1 into P[(i+1) & 1]
//              -> barrier(i+1)
// P and the picks are double-buffered by tile parity, the q / grad_out tiles and weight records
// triple-buffered by tile mod 3; every copy is issued two tiles ahead of its use. Eight lanes
// share a token (8 head dims each), a warp takes 4 tokens; warp 16 issues every copy and MMA.
template <typename T>
__global__ void __launch_bounds__(tcb::kThreads, 1)
    k_bwd_tokens_tc(Geom g, int r, const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap gmap,
                    const T* q, Strides3 qs, const T* go, Strides3 gos, const float* gw, T* gq, Strides3 gqs,
                    Saved sv, BwdScratch bs, const uint8_t* tables, const float* dWpad) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t s_base = smem_u32(sm);
  uint64_t* bar_tab = reinterpret_cast<uint64_t*>(sm + tcb::OFF_MISC);
  uint64_t* bar_q = bar_tab + 1;  // [3], by tile mod 3
  uint64_t* bar_g = bar_tab + 4;  // [3], by tile mod 3
  uint64_t* bar_w = bar_tab + 7;  // [3], by tile mod 3
  uint64_t* bar_mma = bar_tab + 10;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + tcb::OFF_MISC + 96);
  volatile int* s_abort = reinterpret_cast<volatile int*>(sm + tcb::OFF_MISC + 100);
  const float* dWs = reinterpret_cast<const float*>(sm + tcb::OFF_DW);
  float* coef = reinterpret_cast<float*>(sm + tcb::OFF_COEF);

  constexpr int kBT = tcb::kBTile;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.y, b = bh / g.H, h = bh - b * g.H, chunk = blockIdx.x;
  const int t_beg = chunk * g.bwd_chunk_tokens;
  const int t_end = min(g.N, t_beg + g.bwd_chunk_tokens);
  const int ntiles = (t_end - t_beg + kBT - 1) / kBT;
  const bool has_slot_grad = r < g.R - 1;
  const bool first = (r == g.R - 1);
  const size_t rec0 = ((size_t)r * g.BH + bh) * g.N;  // record row of token 0 of this (b, h)
  const bool math_thread = tid < tcb::kIssuer;
  const int grp = lane >> 3, c8 = lane & 7;
  const int tok = 4 * warp + grp;  // the token of this lane group within a tile (math warps)

  if (tid == tcb::kIssuer) {
    mbar_init(bar_tab, 1);
    for (int i = 0; i < 3; ++i) {
      mbar_init(&bar_q[i], 1);
      mbar_init(&bar_g[i], 1);
      mbar_init(&bar_w[i], 1);
    }
    mbar_init(bar_mma, 1);
    *s_abort = 0;
    fence_barrier_init();
  }
  {
    float4* p4 = reinterpret_cast<float4*>(sm + tcb::OFF_P);
    for (int i = tid; i < 2 * (int)tcb::kPBuf / 16; i += tcb::kThreads) p4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, tcb::kTmemCols);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // everything above touched only this CTA's shared memory and TMEM: it overlaps the previous
  // kernel, whose outputs (tables, dW, dq of later rounds) are read from here on
  pdl_wait();
  pdl_trigger();
  const uint32_t tmem = *tmem_slot;
  uint32_t ph_mma = 0;
  // Scatter operands. fp16: as they are. bf16: as fp16 under the pair's power-of-two scales (the
  // q and grad_out tiles converted in place once loaded, each math thread its own 16-byte chunk,
  // the weights and coefficients one fp16 term), unless the pair's largest |q| or |grad_out|
  // exceeds 2^8: then bf16 operands with two terms per weight and coefficient.
  constexpr bool kBf16 = tcb::Fmt<T>::v == 1;
  bool f16ops = true;
  float sq = 1.f, sg = 1.f;  // operand scales of the q and grad_out tiles
  if constexpr (kBf16) {
    float* smax = reinterpret_cast<float*>(sm + tcb::OFF_MISC + 104);
    if (warp == 0) {
      float mq = bs.amax[(size_t)bh * 64 + lane], mg = bs.amax[(size_t)bh * 64 + 32 + lane];
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        mq = fmaxf(mq, __shfl_xor_sync(0xffffffffu, mq, o));
        mg = fmaxf(mg, __shfl_xor_sync(0xffffffffu, mg, o));
      }
      if (lane == 0) {
        smax[0] = mq;
        smax[1] = mg;
      }
    }
    __syncthreads();
    f16ops = smax[0] <= 256.f && smax[1] <= 256.f;  // false for inf / NaN maxima too
    if (f16ops) {
      sq = tcb::pow2i(tcb::scale_exp(smax[0]));
      sg = tcb::pow2i(tcb::scale_exp(smax[1]));
    }
  }
  const bool convert_tiles = kBf16 && f16ops;
  const uint32_t id_upd = idesc_f16(f16ops ? 0u : tcb::Fmt<T>::v, 128, 64, 1, 1);
  // the issuer's bookkeeping of asynchronous copies: the last tile issued / waited for
  int q_issued = -1, g_issued = -1, w_issued = -1, q_done = -1, g_done = -1, w_done = -1;
  bool tab_pending = false;
  auto load_q = [&](int j) {  // issuer
    const int s = j % 3;
    mbar_arrive_expect_tx(&bar_q[s], tcb::kTileBytes);
    tma_load_4d(sm + tcb::OFF_Q + s * tcb::kTileBytes, &qmap, 0, t_beg + j * kBT, h, b, &bar_q[s]);
    q_issued = j;
  };
  auto load_g = [&](int j) {  // issuer
    const int s = j % 3;
    mbar_arrive_expect_tx(&bar_g[s], tcb::kTileBytes);
    tma_load_4d(sm + tcb::OFF_G + s * tcb::kTileBytes, &gmap, 0, t_beg + j * kBT, h, b, &bar_g[s]);
    g_issued = j;
  };
  auto load_w = [&](int j) {  // issuer: the tile's softmax weights, 32 bytes per token
    const int s = j % 3;
    const int n = t_beg + j * kBT;
    const uint32_t bytes = (uint32_t)min(kBT, t_end - n) * 32u;
    mbar_arrive_expect_tx(&bar_w[s], bytes);
    bulk_g2s(sm + tcb::OFF_TW + s * kBT * 32, sv.w + (rec0 + n) * 8, bytes, &bar_w[s]);
    w_issued = j;
  };
  auto wait_copy = [&](uint64_t* bar, int j, int& done) {  // issuer
    if (tcb::timed_wait(bar, (j / 3) & 1)) {
      done = j;
    } else {
      atomicOr(&g_device_error, tcb::kErrWait);
      *s_abort = 1;
    }
  };
  if (tid == tcb::kIssuer) {
    mbar_arrive_expect_tx(bar_tab, tcb::kTables + 1024);
    bulk_g2s(sm, tables + (size_t)bh * tcb::kTables, tcb::kTables, bar_tab);
    bulk_g2s(sm + tcb::OFF_DW, dWpad + (size_t)bh * tcb::kSlotsPad, 1024, bar_tab);
    tab_pending = true;
    for (int j = 0; j < 2 && j < ntiles; ++j) {
      load_q(j);
      load_g(j);
      load_w(j);
    }
  }
  // every thread reads the tables: wait for them once
  if (!tcb::timed_wait(bar_tab, 0)) {
    atomicOr(&g_device_error, tcb::kErrWait);
    *s_abort = 1;
  } else if (tid == tcb::kIssuer) {
    tab_pending = false;
  }

  const uint8_t* tK = sm + tcb::OFF_K;
  const uint8_t* tV = sm + tcb::OFF_V;
  const uint8_t* tS = sm + tcb::OFF_DS;
  // D += P^T . B over a tile's 64 tokens (issuer): two 128-slot halves, four k-steps of 16 tokens
  auto issue_scatter = [&](uint32_t a_p, uint32_t a_b, uint32_t col, bool first_acc) {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh)
#pragma unroll
      for (int kk = 0; kk < kBT / 16; ++kk)
        mma_f16(tmem + col + 64 * hh,
                smem_desc(a_p + 2 * hh * tcb::kPBlock + kk * 2048, tcb::kPBlock, 1024, kSwizzle128B),
                smem_desc(a_b + kk * 2048, tcb::kTileBytes, 1024, kSwizzle128B), id_upd,
                (first_acc && kk == 0) ? 0u : 1u);
  };
  auto wait_mma = [&]() {
    if (tcb::timed_wait(bar_mma, ph_mma)) ph_mma ^= 1;
    else { atomicOr(&g_device_error, tcb::kErrWait); *s_abort = 1; }
    tc_fence_after();
  };
  auto p_addr = [&](int j) { return s_base + tcb::OFF_P + (j & 1) * tcb::kPBuf; };
  auto q_addr = [&](int j) { return s_base + tcb::OFF_Q + (j % 3) * tcb::kTileBytes; };
  auto g_addr = [&](int j) { return s_base + tcb::OFF_G + (j % 3) * tcb::kTileBytes; };
  auto p_entry = [&](int j, int t, int m) -> uint16_t* {  // P of tile j: token t, slot m
    return reinterpret_cast<uint16_t*>(sm + tcb::OFF_P + (j & 1) * tcb::kPBuf + (m >> 6) * tcb::kPBlock +
                                       sw128_offset(t, m & 63));
  };
  auto tix_of = [&](int j) { return reinterpret_cast<uint2*>(sm + tcb::OFF_TIX + (j & 1) * kBT * 8); };
  auto tw_of = [&](int j) { return reinterpret_cast<const float*>(sm + tcb::OFF_TW + (j % 3) * kBT * 32); };
  auto tgw_of = [&](int j) { return reinterpret_cast<float*>(sm + tcb::OFF_TGW + (j & 1) * kBT * 32); };
  auto fill_tgw = [&](int j) {  // dL/d weights of tile j (last round, when given)
    const int n = t_beg + j * kBT;
    const float* src = gw + ((size_t)bh * g.N + n) * kTopK;
    float* dst = tgw_of(j);
    for (int e = tid; e < min(kBT, t_end - n) * kTopK; e += tcb::kThreads) dst[(e / kTopK) * 8 + e % kTopK] = src[e];
  };

  // Scatter phases over P (64 tokens x 256 slots, one term per phase):
  //   fp16: dV += P^T.G (P = w) during the token math, then dK += P^T.Q (P = scale*da);
  //   bf16: weights and coefficients go in as two terms each (hi = rn(x), lo = rn(x - hi)),
  //         since bf16 alone rounds them to 2^-9: dV_hi during the math, then dV_lo, dK_hi, dK_lo.
  // The last phase is issued with the next tile's first (and is waited for with it).
  const int terms = f16ops ? 1 : 2;
  auto hi_bits = [&](float x) -> uint16_t { return f16ops ? tcb::bits<__half>(x) : tcb::bits<T>(x); };
  auto lo_bits = [](float x) -> uint16_t {
    const uint16_t hb = tcb::bits<T>(x);
    return tcb::bits<T>(x - Elem<T>::load(reinterpret_cast<const T*>(&hb)));
  };
  auto pick_of = [](uint2 pk, int j) -> int { return (int)(((j < 4 ? pk.x : pk.y) >> (8 * (j & 3))) & 0xffu); };
  auto last_phase = [&](int j) {  // issuer: the deferred last scatter of tile j (fp16 dK; bf16 dK_lo)
    issue_scatter(p_addr(j), q_addr(j), tcb::COL_DK, j == 0 && terms == 1);
  };
  // picks of this lane group's token of a tile
  auto fetch_ix = [&](int j) -> uint2 {
    uint2 v = make_uint2(0u, 0u);
    const int n = t_beg + j * kBT;
    if (math_thread && j < ntiles && tok < min(kBT, t_end - n)) v = reinterpret_cast<const uint2*>(sv.idx)[rec0 + n + tok];
    return v;
  };
  // dq of earlier rounds for this thread's token and head dims of a tile, read a tile ahead
  float4 pv0 = make_float4(0.f, 0.f, 0.f, 0.f), pv1 = pv0;
  auto fetch_prev = [&](int j) {
    pv0 = pv1 = make_float4(0.f, 0.f, 0.f, 0.f);
    const int n = t_beg + j * kBT;
    if (math_thread && !first && j < ntiles && tok < min(kBT, t_end - n)) {
      const float4* acc = reinterpret_cast<const float4*>(bs.dq + ((size_t)bh * g.N + n + tok) * g.D + 8 * c8);
      pv0 = acc[0];
      pv1 = acc[1];
    }
  };
  // Records of tile j into P[j & 1] (lane c8: pick c8): the entry of tile j-2 is cleared first.
  // Tile j-2's last scatter finished before tile j-1's first did, which every thread has waited for.
  int oslot0 = -1, oslot1 = -1;  // this lane's entry in P[0] / P[1] (-1: none)
  auto records = [&](int j, uint2 rix) {
    const int nn = min(kBT, t_end - (t_beg + j * kBT));
    const int os = (j & 1) ? oslot1 : oslot0;
    if (os >= 0) *p_entry(j, tok, os) = 0;
    __syncwarp();  // every old entry of the token is cleared before any new one is written
    int ns = -1;
    if (tok < nn && c8 < kTopK) {
      if (!tcb::timed_wait(&bar_w[j % 3], (j / 3) & 1)) {
        atomicOr(&g_device_error, tcb::kErrWait);
        *s_abort = 1;
      }
      ns = pick_of(rix, c8);
      *p_entry(j, tok, ns) = hi_bits(tw_of(j)[tok * 8 + c8]);
    }
    if (tok < nn && c8 == 0) tix_of(j)[tok] = rix;
    if (j & 1) oslot1 = ns;
    else oslot0 = ns;
  };

  // bf16 with fp16 operands: this thread's 16-byte chunk (row tok, chunk c8) of tile j's q and
  // grad_out, kept as loaded for the token math and written back as fp16 under the pair's scales
  uint4 qreg = make_uint4(0u, 0u, 0u, 0u), greg = qreg;
  auto convert = [&](int j) {  // math threads
    if (!tcb::timed_wait(&bar_q[j % 3], (j / 3) & 1) || !tcb::timed_wait(&bar_g[j % 3], (j / 3) & 1)) {
      atomicOr(&g_device_error, tcb::kErrWait);
      *s_abort = 1;
      return;
    }
    const uint32_t rw = (uint32_t)tok * 128 + (((uint32_t)c8 ^ (tok & 7)) << 4);
    uint4* pq = reinterpret_cast<uint4*>(sm + tcb::OFF_Q + (j % 3) * tcb::kTileBytes + rw);
    uint4* pg = reinterpret_cast<uint4*>(sm + tcb::OFF_G + (j % 3) * tcb::kTileBytes + rw);
    qreg = *pq;
    greg = *pg;
    *pq = tcb::bf16_to_f16_scaled(qreg, sq);
    *pg = tcb::bf16_to_f16_scaled(greg, sg);
  };

  fetch_prev(0);
  if (math_thread && ntiles > 0) records(0, fetch_ix(0));
  if (convert_tiles && math_thread && ntiles > 0) convert(0);
  if (gw && first && ntiles > 0) fill_tgw(0);
  uint2 rq = fetch_ix(1);  // picks for the next records
  if (tid == tcb::kIssuer && ntiles > 0) {
    wait_copy(&bar_q[0], 0, q_done);
    wait_copy(&bar_g[0], 0, g_done);
    wait_copy(&bar_w[0], 0, w_done);
  }

  bool stop = false;
  for (int tile = 0; tile < ntiles; ++tile) {
    const int n0 = t_beg + tile * kBT;
    const int nt = min(kBT, t_end - n0);
    fence_proxy_async_smem();
    tc_fence_before();
    if (__syncthreads_or(*s_abort != 0)) { stop = true; break; }  // one decision for all threads
    tc_fence_after();
    if (tid == tcb::kIssuer) {
      if (tile > 0) last_phase(tile - 1);
      issue_scatter(p_addr(tile), g_addr(tile), tcb::COL_DV, tile == 0);  // dV (first term)
      mma_commit(bar_mma);
      if (tile + 2 < ntiles) {  // buffers (tile+2) mod 3 were last read by tile-1's math and dV phases
        load_g(tile + 2);
        load_w(tile + 2);
      }
      if (!first && tile + 1 < ntiles) {  // next tile's earlier-round dq into L2
        const int nn0 = n0 + kBT;
        bulk_prefetch_l2(bs.dq + ((size_t)bh * g.N + nn0) * g.D, (uint32_t)(min(kBT, t_end - nn0) * g.D * 4));
      }
    }

    // ---- token math: 8 lanes per token (8 head dims per lane), 4 tokens per warp ----
    const uint8_t* sq_t = sm + tcb::OFF_Q + (tile % 3) * tcb::kTileBytes;
    const uint8_t* sgo = sm + tcb::OFF_G + (tile % 3) * tcb::kTileBytes;
    const uint2* tix = tix_of(tile);
    const float* tw = tw_of(tile);
    const float* tgw = tgw_of(tile);
    const bool live = tok < nt;                      // group-uniform
    const bool busy = math_thread && 4 * warp < nt;  // warp-uniform
    int ix[kTopK];
    float w[kTopK], c[kTopK];
    if (busy) {
      const int t = live ? tok : 0;
      const int n = n0 + t;
      const uint2 pk = tix[t];
#pragma unroll
      for (int j = 0; j < kTopK; ++j) ix[j] = pick_of(pk, j);
      const float4 w0 = reinterpret_cast<const float4*>(tw + t * 8)[0];
      const float4 w1 = reinterpret_cast<const float4*>(tw + t * 8)[1];
      w[0] = w0.x; w[1] = w0.y; w[2] = w0.z; w[3] = w0.w; w[4] = w1.x; w[5] = w1.y; w[6] = w1.z;
      // swizzled 128-byte rows of the TMA tiles: 16-byte chunk c8 of row t
      const uint32_t rw = (uint32_t)t * 128 + (((uint32_t)c8 ^ (t & 7)) << 4);
      const uint4 qv = convert_tiles ? qreg : *reinterpret_cast<const uint4*>(sq_t + rw);
      const uint4 gv = convert_tiles ? greg : *reinterpret_cast<const uint4*>(sgo + rw);
      float dq[8] = {pv0.x, pv0.y, pv0.z, pv0.w, pv1.x, pv1.y, pv1.z, pv1.w};
      float part[8];
#pragma unroll
      for (int j = 0; j < kTopK; ++j) {
        float a = tcb::dot8<T>(gv, *reinterpret_cast<const uint4*>(tV + ix[j] * 128 + 16 * c8), 0.f);
        if (has_slot_grad) {  // dS[i_j] enters both dw_j and dq
          const uint4 ds = *reinterpret_cast<const uint4*>(tS + ix[j] * 128 + 16 * c8);
          a = tcb::dot8<T>(qv, ds, a);
          tcb::axpy8<T>(w[j], ds, dq);
        }
        part[j] = a;
      }
      part[7] = 0.f;
      tcb::group8_sum8(part);
      float dw[kTopK], s = 0.f;
#pragma unroll
      for (int j = 0; j < kTopK; ++j) {
        dw[j] = part[j] + (has_slot_grad ? dWs[ix[j]] : 0.f);
        if (gw && first) dw[j] += tgw[t * 8 + j];
        s = fmaf(w[j], dw[j], s);
      }
#pragma unroll
      for (int j = 0; j < kTopK; ++j) {
        c[j] = g.scale * (w[j] * (dw[j] - s));
        tcb::axpy8<T>(c[j], *reinterpret_cast<const uint4*>(tK + ix[j] * 128 + 16 * c8), dq);
      }
      if (live) {
        if (r == 0) {
          uint4 o;
          uint16_t* oh = reinterpret_cast<uint16_t*>(&o);
#pragma unroll
          for (int i = 0; i < 8; ++i) oh[i] = tcb::bits<T>(dq[i]);
          *reinterpret_cast<uint4*>(row_ptr(gq, gqs, b, h, n) + 8 * c8) = o;
        } else {
          float4* acc = reinterpret_cast<float4*>(bs.dq + ((size_t)bh * g.N + n) * g.D + 8 * c8);
          acc[0] = make_float4(dq[0], dq[1], dq[2], dq[3]);
          acc[1] = make_float4(dq[4], dq[5], dq[6], dq[7]);
        }
      }
    }
    // the next tile's earlier-round dq, in flight during the scatter wait
    fetch_prev(tile + 1);
    wait_mma();  // tile-1's last scatter and this tile's first are done
    if (tid == tcb::kIssuer && tile + 2 < ntiles) load_q(tile + 2);  // its buffer was last read by tile-1's dK
    if (busy && live && c8 < kTopK) {  // P[tile & 1] takes the next term
      float wl = 0.f, cl = 0.f;
      int ml = 0;
#pragma unroll
      for (int j = 0; j < kTopK; ++j)
        if (c8 == j) { wl = w[j]; cl = c[j]; ml = ix[j]; }
      coef[tok * 8 + c8] = cl;
      *p_entry(tile, tok, ml) = terms == 1 ? hi_bits(cl) : lo_bits(wl);
    }
    // the next tile's weights into P[(tile+1) & 1] (free: tile-1's dK is done)
    if (math_thread && tile + 1 < ntiles) {
      records(tile + 1, rq);
      rq = fetch_ix(tile + 2);
    }
    if (gw && first && tile + 1 < ntiles) fill_tgw(tile + 1);  // its buffer was last read by tile-1's math

    // ---- bf16: dV_lo, dK_hi (the last phase, dK_lo, is issued with the next tile's first) ----
#pragma unroll 1
    for (int ph = 1; ph < 2 * terms - 1; ++ph) {
      const bool is_k = ph >= terms;
      if (ph >= 2 && math_thread && tok < nt && c8 < kTopK) {  // P takes the coefficient's high term
        *p_entry(tile, tok, pick_of(tix[tok], c8)) = hi_bits(coef[tok * 8 + c8]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      stop = __syncthreads_or(*s_abort != 0);
      tc_fence_after();
      if (stop) break;
      if (tid == tcb::kIssuer) {
        issue_scatter(p_addr(tile), is_k ? q_addr(tile) : g_addr(tile), is_k ? tcb::COL_DK : tcb::COL_DV,
                      tile == 0 && is_k && ph == terms);
        mma_commit(bar_mma);
      }
      wait_mma();
    }
    if (stop) break;
    if (terms == 2 && math_thread && tok < nt && c8 < kTopK)  // bf16: the coefficient's low term
      *p_entry(tile, tok, pick_of(tix[tok], c8)) = lo_bits(coef[tok * 8 + c8]);
    if (tid == tcb::kIssuer && tile + 1 < ntiles) {  // the next tile's copies (issued two tiles ago)
      wait_copy(&bar_q[(tile + 1) % 3], tile + 1, q_done);
      wait_copy(&bar_g[(tile + 1) % 3], tile + 1, g_done);
      wait_copy(&bar_w[(tile + 1) % 3], tile + 1, w_done);
    }
    if (convert_tiles && math_thread && tile + 1 < ntiles) convert(tile + 1);  // published by the next barrier
  }

  // the last tile's last scatter, once its P entries are written; every scatter finished before
  // TMEM is read (this also drains the MMAs of an aborted tile)
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid == tcb::kIssuer) {
    if (!stop && ntiles > 0) last_phase(ntiles - 1);
    mma_commit(bar_mma);
  }
  wait_mma();
  // ---- chunk partials of dK_r, dV_r (TMEM lanes are slots): warps 0-3 dV, 4-7 dK ----
  if (warp < 8 && !__any_sync(0xffffffffu, *s_abort != 0)) {
    const int quad = warp & 3;
    const uint32_t lb = (uint32_t)(32 * quad) << 16;
    const bool is_k = warp >= 4;
    float* dst_base = is_k ? bs.dKpart : bs.dVpart;
    const float unscale = 1.f / (is_k ? sq : sg);  // a power of two: exact
    const size_t po = (size_t)bh * g.bwd_chunks + chunk;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int m = 128 * hh + 32 * quad + lane;
      float a[32], c2[32];
      const uint32_t col = (is_k ? tcb::COL_DK : tcb::COL_DV) + 64 * hh;
      tmem_ld32(tmem + lb + col, a);
      tmem_ld32(tmem + lb + col + 32, c2);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        a[i] *= unscale;
        c2[i] *= unscale;
      }
      if (m < g.M) {  // chunk-major: a warp's store of one 4-column chunk covers 32 consecutive rows
        float4* dst = reinterpret_cast<float4*>(dst_base) + po * 16 * g.M + m;
#pragma unroll
        for (int i = 0; i < 8; ++i)
          dst[(size_t)i * g.M] = make_float4(a[4 * i], a[4 * i + 1], a[4 * i + 2], a[4 * i + 3]);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          dst[(size_t)(8 + i) * g.M] = make_float4(c2[4 * i], c2[4 * i + 1], c2[4 * i + 2], c2[4 * i + 3]);
      }
    }
  }
  if (tid == tcb::kIssuer) {  // copies still in flight after an abort: wait for them (bounded)
    if (tab_pending) tcb::timed_wait(bar_tab, 0);
    for (int j = q_done + 1; j <= q_issued; ++j) tcb::timed_wait(&bar_q[j % 3], (j / 3) & 1);
    for (int j = g_done + 1; j <= g_issued; ++j) tcb::timed_wait(&bar_g[j % 3], (j / 3) & 1);
    for (int j = w_done + 1; j <= w_issued; ++j) tcb::timed_wait(&bar_w[j % 3], (j / 3) & 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, tcb::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 tc_tensor_map_encoder();  // murm_tc.cu

template <typename T>
static bool make_rows_map(CUtensorMap* map, const Geom& g, const void* base, Strides3 st) {
  auto encode = tc_tensor_map_encoder();
  if (!encode) return false;
  const cuuint64_t esz = sizeof(T);
  cuuint64_t dims[4] = {(cuuint64_t)g.D, (cuuint64_t)g.N, (cuuint64_t)g.H, (cuuint64_t)g.B};
  cuuint64_t strides[3] = {(cuuint64_t)st.s[2] * esz, (cuuint64_t)st.s[1] * esz,
                           (cuuint64_t)(st.s[0] ? st.s[0] : 1) * esz};
  cuuint32_t box[4] = {64, tcb::kBTile, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt =
      tcb::Fmt<T>::v == 1 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return encode(map, dt, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool tc_backward_supported(const Geom& g, int dtype, const BwdPtrs& p) {
  if (dtype != MURM_F16 && dtype != MURM_BF16) return false;
  if (g.D != tcb::kD || g.R < 1) return false;
  for (int i = 0; i < 3; ++i)
    if ((p.qs.s[i] % 8) || (p.gos.s[i] % 8) || (p.gqs.s[i] % 8)) return false;
  if ((reinterpret_cast<uintptr_t>(p.q) | reinterpret_cast<uintptr_t>(p.go) | reinterpret_cast<uintptr_t>(p.gq)) & 15)
    return false;
  const char* force = getenv("MURM_FORCE_SIMT");
  return !(force && force[0] == '1');
}

size_t tc_bwd_tables_bytes(const Geom& g) {
  if (g.D != tcb::kD || g.dtype == MURM_F32) return 0;
  return (size_t)g.BH * (tcb::kTables + tcb::kSlotsPad * 4);
}

template <typename T>
cudaError_t bwd_tc(const Geom& g, const BwdPtrs& p, const Saved& sv, const BwdScratch& bs, cudaStream_t st) {
  CUtensorMap qmap, gmap;
  if (!make_rows_map<T>(&qmap, g, p.q, p.qs) || !make_rows_map<T>(&gmap, g, p.go, p.gos))
    return cudaErrorInvalidValue;
  if (cudaError_t e = smem_opt_in(k_bwd_tokens_tc<T>, tcb::kSmem)) return e;
  uint8_t* tables = bs.tables;
  float* dWpad = reinterpret_cast<float*>(tables + (size_t)g.BH * tcb::kTables);
  const int slot_blocks = (g.M + kSlotRows - 1) / kSlotRows;
  static_assert(tcb::kSlotsPad * 32 / 256 == 32, "32 blocks per pair: the token kernel reads 32 maxima of each");
  MURM_LAUNCH_PDL("bwd_tables", k_bwd_tables_last<T>, dim3(g.BH, tcb::kSlotsPad * 32 / 256), 256, 0, st, g, sv, tables, dWpad,
                  static_cast<const T*>(p.q), p.qs, static_cast<const T*>(p.go), p.gos, bs.amax);
  for (int r = g.R - 1; r >= 0; --r) {
    MURM_LAUNCH_PDL("bwd_tokens_tc", k_bwd_tokens_tc<T>, dim3(g.bwd_chunks, g.BH), tcb::kThreads, tcb::kSmem, st, g, r,
                qmap, gmap, static_cast<const T*>(p.q), p.qs, static_cast<const T*>(p.go), p.gos, p.gw,
                static_cast<T*>(p.gq), p.gqs, sv, bs, tables, dWpad);
    MURM_LAUNCH_PDL("bwd_slots", k_bwd_slots<T>, dim3(g.BH, slot_blocks), tcb::kRowLanes * kSlotHalo, 0, st, g, r, r < g.R - 1 ? 1 : 0, 1,
                sv, bs, tables, dWpad, static_cast<T*>(p.gsk), p.gsks, static_cast<T*>(p.gsv), p.gsvs);
  }
  return cudaGetLastError();
}

template cudaError_t bwd_tc<__half>(const Geom&, const BwdPtrs&, const Saved&, const BwdScratch&, cudaStream_t);
template cudaError_t bwd_tc<__nv_bfloat16>(const Geom&, const BwdPtrs&, const Saved&, const BwdScratch&,
                                           cudaStream_t);

}  // namespace murm
