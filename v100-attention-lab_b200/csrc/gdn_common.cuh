// Device helpers shared by the GDN kernels: problem constants, per-chunk
// vector layout, operand writers and the fp32 unit-lower-triangular inverse.
#pragma once
#include "tc.cuh"
#include "../../include/gdn_b200.h"

namespace gdn {

constexpr int kC = 64;    // chunk length
constexpr int kK = 128;   // key dim
constexpr int kV = 128;   // value dim
constexpr int kAStride = 68;  // fp32 row stride of the A/T work matrix (column 64 holds F_m)
constexpr int kVecN = 4;      // per-chunk vectors: b*log2(e) (cumsum), beta, e^b, e^(b_C - b)
enum : int { V_B2 = 0, V_BETA = 1, V_EB = 2, V_DD = 3 };

// Tracing: with -DGDN_TRACE the kernel records clock64() at fixed points of
// each role for every chunk of CTA 0 into P.trace[chunk * kTraceSlots + slot].
constexpr int kTraceSlots = 24;
#ifdef GDN_TRACE
#define GDN_TR(slot, chunk)                                                                  \
  do {                                                                                       \
    if (P.trace != nullptr && blockIdx.x == 0) P.trace[(chunk) * kTraceSlots + (slot)] = clock64(); \
  } while (0)
#else
#define GDN_TR(slot, chunk) \
  do {                      \
  } while (0)
#endif

// beta and g of one step as the kernels use them: zero past T (the padding
// rule of gdn_ref.py:102-114), g == 0 when no gate tensor is given (the
// DeltaNet recurrence), and the activations of bench_gdn.py:33-40 applied here
// when the inputs are logits (GDN_FLAG_BETA_SIGMOID, GDN_FLAG_G_LOGSIGMOID).
__device__ __forceinline__ float load_beta(const float* bp, long long off, bool valid, int flags) {
  if (!valid) return 0.f;
  const float x = bp[off];
  return (flags & GDN_FLAG_BETA_SIGMOID) ? 1.f / (1.f + expf(-x)) : x;
}
__device__ __forceinline__ float load_g(const float* gp, long long off, bool valid, int flags) {
  if (!valid || gp == nullptr) return 0.f;
  const float x = gp[off];
  // logsigmoid(x) = min(x, 0) - log(1 + e^{-|x|})
  return (flags & GDN_FLAG_G_LOGSIGMOID) ? fminf(x, 0.f) - log1pf(expf(-fabsf(x))) : x;
}

__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

template <typename OutT>
__device__ __forceinline__ void store_row(OutT* dst, const float* v, int n);

template <>
__device__ __forceinline__ void store_row<float>(float* dst, const float* v, int n) {
  for (int i = 0; i < n; i += 4) *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
}
template <>
__device__ __forceinline__ void store_row<__half>(__half* dst, const float* v, int n) {
  for (int i = 0; i < n; i += 8) {
    uint4 w;
    w.x = Cvt<__half>::pack(v[i], v[i + 1]);
    w.y = Cvt<__half>::pack(v[i + 2], v[i + 3]);
    w.z = Cvt<__half>::pack(v[i + 4], v[i + 5]);
    w.w = Cvt<__half>::pack(v[i + 6], v[i + 7]);
    *reinterpret_cast<uint4*>(dst + i) = w;
  }
}
template <>
__device__ __forceinline__ void store_row<__nv_bfloat16>(__nv_bfloat16* dst, const float* v, int n) {
  for (int i = 0; i < n; i += 8) {
    uint4 w;
    w.x = Cvt<__nv_bfloat16>::pack(v[i], v[i + 1]);
    w.y = Cvt<__nv_bfloat16>::pack(v[i + 2], v[i + 3]);
    w.z = Cvt<__nv_bfloat16>::pack(v[i + 4], v[i + 5]);
    w.w = Cvt<__nv_bfloat16>::pack(v[i + 6], v[i + 7]);
    *reinterpret_cast<uint4*>(dst + i) = w;
  }
}

// Write 32 fp32 values as fp16 into row r of a BV=32 (64-byte rows, SW64) or
// the first half of a BV=64 (128-byte rows, SW128) MN-major tile.
template <int BV>
__device__ __forceinline__ void st_row16(uint8_t* tile, uint32_t r, uint32_t c16_base, const float* v) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint4 w;
    w.x = Cvt<__half>::pack(v[8 * c + 0], v[8 * c + 1]);
    w.y = Cvt<__half>::pack(v[8 * c + 2], v[8 * c + 3]);
    w.z = Cvt<__half>::pack(v[8 * c + 4], v[8 * c + 5]);
    w.w = Cvt<__half>::pack(v[8 * c + 6], v[8 * c + 7]);
    const uint32_t off = (BV == 32) ? sw64_off(r, c16_base + c) : sw128_off(r, c16_base + c);
    *reinterpret_cast<uint4*>(tile + off) = w;
  }
}

// ------------------------------------------------------------------ the inverse
// T = (I + A)^-1 for the 64x64 strictly-lower A held in `am` (row stride
// kAStride), in place, by NTH = 128 or 256 threads (named barrier 1).  Eight 8x8
// diagonal blocks are inverted by column forward substitution; three
// doubling levels (8 -> 16 -> 32 -> 64) then apply
//     inv([[L0, 0], [X, L1]]) = [[inv(L0), 0], [-inv(L1) X inv(L0), inv(L1)]].
// The upper triangle of every block stays zero (the triangular factors' zero
// halves are skipped, not read).  Same result as the row-by-row forward
// substitution of gdn_triton.py:75-84 applied to the identity.
// Work items of one doubling level are 1 x 4 output strips (blk, row i, strip q).
// Phase 1 sums over m >= 4q only (inv(L0) is lower triangular), phase 2 over
// p <= i only (inv(L1) likewise); items are paired (q with N/4-1-q, i with
// N-1-i) so that every lane of a warp runs the same number of iterations.
template <int N, int NTH>
struct InvItems {
  static constexpr int NB = 64 / (2 * N), NQ = N / 4;
  static constexpr int PER = (NB * N * NQ + NTH - 1) / NTH;  // items per thread (1 or 2)
  __device__ static bool p1(int tid, int e, int& blk, int& i, int& q) {
    if constexpr (N == 32) {
      blk = 0;
      i = tid & 31;
      if constexpr (NTH == 256) {
        const int w = tid >> 5;  // warps w and w + 4 share a sub-partition: q and 7 - q
        q = w < 4 ? w : 11 - w;
      } else {
        q = e == 0 ? (tid >> 5) : NQ - 1 - (tid >> 5);
      }
      return true;
    } else if constexpr (N == 16) {
      blk = (tid >> 6) & 1; i = tid & 15; q = (tid >> 4) & 3;
      return tid < 128;
    } else {
      blk = (tid >> 4) & 3; i = tid & 7; q = (tid >> 3) & 1;
      return tid < 64;
    }
  }
  __device__ static bool p2(int tid, int e, int& blk, int& i, int& q) {
    if constexpr (N == 32) {
      blk = 0;
      q = tid & 7;
      if constexpr (NTH == 256) {
        const int w = tid >> 5, g = w < 4 ? w : 11 - w;  // row groups g and 7 - g per sub-partition
        i = 4 * g + ((tid & 31) >> 3);
      } else {
        i = e == 0 ? (tid >> 3) : N - 1 - (tid >> 3);
      }
      return true;
    } else if constexpr (N == 16) {
      blk = (tid >> 6) & 1; q = tid & 3; i = (tid >> 2) & 15;
      return tid < 128;
    } else {
      blk = (tid >> 4) & 3; q = tid & 1; i = (tid >> 1) & 7;
      return tid < 64;
    }
  }
};

__device__ __forceinline__ void fma4(float4& acc, float a, const float4& b) {
  acc.x = fmaf(a, b.x, acc.x);
  acc.y = fmaf(a, b.y, acc.y);
  acc.z = fmaf(a, b.z, acc.z);
  acc.w = fmaf(a, b.w, acc.w);
}

template <int N, int NTH>
__device__ __forceinline__ void inv_level(float* am, int tid) {
  using It = InvItems<N, NTH>;
  constexpr int S = kAStride;
  float4 acc[It::PER];
  // phase 1: Y = X inv(L0); X = rows N..2N-1 x cols 0..N-1 of each 2N block
#pragma unroll
  for (int e = 0; e < It::PER; ++e) {
    int blk, i, q;
    float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
    if (It::p1(tid, e, blk, i, q)) {
      const int o = blk * 2 * N;
      const float* xr = am + (o + N + i) * S + o;
#pragma unroll
      for (int m4 = 0; m4 < It::NQ; ++m4) {
        if (m4 >= q) {
          const float4 x = *reinterpret_cast<const float4*>(xr + 4 * m4);
          const float* t0 = am + (o + 4 * m4) * S + o + 4 * q;
          fma4(a0, x.x, *reinterpret_cast<const float4*>(t0));
          fma4(a1, x.y, *reinterpret_cast<const float4*>(t0 + S));
          fma4(a0, x.z, *reinterpret_cast<const float4*>(t0 + 2 * S));
          fma4(a1, x.w, *reinterpret_cast<const float4*>(t0 + 3 * S));
        }
      }
    }
    acc[e] = make_float4(a0.x + a1.x, a0.y + a1.y, a0.z + a1.z, a0.w + a1.w);
  }
  named_bar(1, NTH);
#pragma unroll
  for (int e = 0; e < It::PER; ++e) {
    int blk, i, q;
    if (It::p1(tid, e, blk, i, q)) {
      const int o = blk * 2 * N;
      *reinterpret_cast<float4*>(am + (o + N + i) * S + o + 4 * q) = acc[e];
    }
  }
  named_bar(1, NTH);
  // phase 2: T = -inv(L1) Y
#pragma unroll
  for (int e = 0; e < It::PER; ++e) {
    int blk, i, q;
    float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
    if (It::p2(tid, e, blk, i, q)) {
      const int o = blk * 2 * N;
      const float* tr = am + (o + N + i) * S + o + N;
#pragma unroll
      for (int p4 = 0; p4 < It::NQ; ++p4) {
        if (p4 <= (i >> 2)) {
          const float4 t = *reinterpret_cast<const float4*>(tr + 4 * p4);
          const float* y = am + (o + N + 4 * p4) * S + o + 4 * q;
          fma4(a0, t.x, *reinterpret_cast<const float4*>(y));
          fma4(a1, t.y, *reinterpret_cast<const float4*>(y + S));
          fma4(a0, t.z, *reinterpret_cast<const float4*>(y + 2 * S));
          fma4(a1, t.w, *reinterpret_cast<const float4*>(y + 3 * S));
        }
      }
    }
    acc[e] = make_float4(a0.x + a1.x, a0.y + a1.y, a0.z + a1.z, a0.w + a1.w);
  }
  named_bar(1, NTH);
#pragma unroll
  for (int e = 0; e < It::PER; ++e) {
    int blk, i, q;
    if (It::p2(tid, e, blk, i, q)) {
      const int o = blk * 2 * N;
      *reinterpret_cast<float4*>(am + (o + N + i) * S + o + 4 * q) =
          make_float4(-acc[e].x, -acc[e].y, -acc[e].z, -acc[e].w);
    }
  }
  named_bar(1, NTH);
}

// One doubling level with the intermediate Y = X inv(L0) in a scratch tile
// instead of in place over X, so each phase ends with a single barrier (the
// in-place form needs one between computing and writing back): 2 barriers per
// level instead of 4.  Same arithmetic, same order of operations.  `scr` holds
// (64 / 2N) blocks of N rows at a stride of N + 4 floats (at most 4.5 KB) and
// must not overlap `am`.
template <int N, int NTH>
__device__ __forceinline__ void inv_level_scr(float* am, float* scr, int tid) {
  using It = InvItems<N, NTH>;
  constexpr int S = kAStride;
  constexpr int SS = N + 4;
  // phase 1: Y = X inv(L0) -> scr; X = rows N..2N-1 x cols 0..N-1 of each 2N block
#pragma unroll
  for (int e = 0; e < It::PER; ++e) {
    int blk, i, q;
    if (It::p1(tid, e, blk, i, q)) {
      float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
      const int o = blk * 2 * N;
      const float* xr = am + (o + N + i) * S + o;
#pragma unroll
      for (int m4 = 0; m4 < It::NQ; ++m4) {
        if (m4 >= q) {
          const float4 x = *reinterpret_cast<const float4*>(xr + 4 * m4);
          const float* t0 = am + (o + 4 * m4) * S + o + 4 * q;
          fma4(a0, x.x, *reinterpret_cast<const float4*>(t0));
          fma4(a1, x.y, *reinterpret_cast<const float4*>(t0 + S));
          fma4(a0, x.z, *reinterpret_cast<const float4*>(t0 + 2 * S));
          fma4(a1, x.w, *reinterpret_cast<const float4*>(t0 + 3 * S));
        }
      }
      *reinterpret_cast<float4*>(scr + (blk * N + i) * SS + 4 * q) =
          make_float4(a0.x + a1.x, a0.y + a1.y, a0.z + a1.z, a0.w + a1.w);
    }
  }
  named_bar(1, NTH);
  // phase 2: T21 = -inv(L1) Y over X (X's last reader was phase 1)
#pragma unroll
  for (int e = 0; e < It::PER; ++e) {
    int blk, i, q;
    if (It::p2(tid, e, blk, i, q)) {
      float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
      const int o = blk * 2 * N;
      const float* tr = am + (o + N + i) * S + o + N;
      const float* yb = scr + (blk * N) * SS + 4 * q;
#pragma unroll
      for (int p4 = 0; p4 < It::NQ; ++p4) {
        if (p4 <= (i >> 2)) {
          const float4 t = *reinterpret_cast<const float4*>(tr + 4 * p4);
          const float* y = yb + (4 * p4) * SS;
          fma4(a0, t.x, *reinterpret_cast<const float4*>(y));
          fma4(a1, t.y, *reinterpret_cast<const float4*>(y + SS));
          fma4(a0, t.z, *reinterpret_cast<const float4*>(y + 2 * SS));
          fma4(a1, t.w, *reinterpret_cast<const float4*>(y + 3 * SS));
        }
      }
      *reinterpret_cast<float4*>(am + (o + N + i) * S + o + 4 * q) =
          make_float4(-(a0.x + a1.x), -(a0.y + a1.y), -(a0.z + a1.z), -(a0.w + a1.w));
    }
  }
  named_bar(1, NTH);
}

// The diagonal 8x8 blocks of (I + A)^-1 by column forward substitution
// (64 threads), in place.
__device__ __forceinline__ void invert_diag8(float* am, int ptid) {
  if (ptid < 64) {
    const int blk_id = ptid >> 3, c = ptid & 7;
    float* blk = am + (8 * blk_id) * kAStride + 8 * blk_id;
    float x[8];
#pragma unroll
    for (int m = 0; m < 8; ++m) x[m] = (m == c) ? 1.f : 0.f;
#pragma unroll
    for (int t = 1; t < 8; ++t) {
      float a0 = 0.f, a1 = 0.f;
#pragma unroll
      for (int m = 0; m < t; ++m) {
        if (m & 1)
          a1 = fmaf(blk[t * kAStride + m], x[m], a1);
        else
          a0 = fmaf(blk[t * kAStride + m], x[m], a0);
      }
      if (t > c) x[t] = -(a0 + a1);
    }
    __syncwarp();
#pragma unroll
    for (int t = 0; t < 8; ++t) blk[t * kAStride + c] = x[t];
  }
}

// T = (I + A)^-1 in place, as invert_unit_lower64, with the doubling levels'
// intermediates in `scr` (>= 4608 bytes, disjoint from am): 7 barriers, not 13.
template <int NTH>
__device__ __forceinline__ void invert_unit_lower64_scr(float* am, float* scr, int ptid) {
  invert_diag8(am, ptid);
  named_bar(1, NTH);
  inv_level_scr<8, NTH>(am, scr, ptid);
  inv_level_scr<16, NTH>(am, scr, ptid);
  inv_level_scr<32, NTH>(am, scr, ptid);
}

template <int NTH = 128>
__device__ __forceinline__ void invert_unit_lower64(float* am, int ptid) {
  if (ptid < 64) {
    const int blk_id = ptid >> 3, c = ptid & 7;
    float* blk = am + (8 * blk_id) * kAStride + 8 * blk_id;
    float x[8];
#pragma unroll
    for (int m = 0; m < 8; ++m) x[m] = (m == c) ? 1.f : 0.f;
#pragma unroll
    for (int t = 1; t < 8; ++t) {
      float a0 = 0.f, a1 = 0.f;
#pragma unroll
      for (int m = 0; m < t; ++m) {
        if (m & 1)
          a1 = fmaf(blk[t * kAStride + m], x[m], a1);
        else
          a0 = fmaf(blk[t * kAStride + m], x[m], a0);
      }
      if (t > c) x[t] = -(a0 + a1);
    }
    __syncwarp();
#pragma unroll
    for (int t = 0; t < 8; ++t) blk[t * kAStride + c] = x[t];
  }
  named_bar(1, NTH);
  inv_level<8, NTH>(am, ptid);
  inv_level<16, NTH>(am, ptid);
  inv_level<32, NTH>(am, ptid);
}

}  // namespace gdn
