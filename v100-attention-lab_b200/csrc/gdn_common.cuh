// Device helpers shared by the GDN kernels: problem constants, per-chunk
// vector layout, operand writers and the fp32 unit-lower-triangular inverse.
#pragma once
#include "tc.cuh"

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
// kAStride), in place, by the 128 prep threads (named barrier 1).  Eight 8x8
// diagonal blocks are inverted by column forward substitution; three
// doubling levels (8 -> 16 -> 32 -> 64) then apply
//     inv([[L0, 0], [X, L1]]) = [[inv(L0), 0], [-inv(L1) X inv(L0), inv(L1)]].
// The upper triangle of every block stays zero, so the block products can run
// over full index ranges.  Same result as the row-by-row forward substitution
// of gdn_triton.py:75-84 applied to the identity.
template <int N>
__device__ __forceinline__ void inv_level(float* am, int tid) {
  constexpr int NTH = 128;
  constexpr int NOUT = (64 / (2 * N)) * N * N;  // outputs per phase
  constexpr int PER = NOUT / NTH;               // outputs per thread
  float acc[PER];
  // phase 1: Y = X inv(L0), X = rows N..2N-1 x cols 0..N-1 of each 2N block
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    const int idx = tid + e * NTH;
    const int pr = idx / (N * N), rem = idx % (N * N);
    const int i = rem / N, j = rem % N, o = pr * 2 * N;
    const float* xr = am + (o + N + i) * kAStride + o;
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
    for (int m = 0; m < N; m += 4) {
      const float4 xv = *reinterpret_cast<const float4*>(xr + m);
      s0 = fmaf(xv.x, am[(o + m + 0) * kAStride + o + j], s0);
      s1 = fmaf(xv.y, am[(o + m + 1) * kAStride + o + j], s1);
      s2 = fmaf(xv.z, am[(o + m + 2) * kAStride + o + j], s2);
      s3 = fmaf(xv.w, am[(o + m + 3) * kAStride + o + j], s3);
    }
    acc[e] = (s0 + s1) + (s2 + s3);
  }
  named_bar(1, NTH);
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    const int idx = tid + e * NTH;
    const int pr = idx / (N * N), rem = idx % (N * N);
    am[(pr * 2 * N + N + rem / N) * kAStride + pr * 2 * N + rem % N] = acc[e];
  }
  named_bar(1, NTH);
  // phase 2: T = -inv(L1) Y
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    const int idx = tid + e * NTH;
    const int pr = idx / (N * N), rem = idx % (N * N);
    const int i = rem / N, j = rem % N, o = pr * 2 * N;
    const float* tr = am + (o + N + i) * kAStride + o + N;
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
    for (int p = 0; p < N; p += 4) {
      const float4 tv = *reinterpret_cast<const float4*>(tr + p);
      s0 = fmaf(tv.x, am[(o + N + p + 0) * kAStride + o + j], s0);
      s1 = fmaf(tv.y, am[(o + N + p + 1) * kAStride + o + j], s1);
      s2 = fmaf(tv.z, am[(o + N + p + 2) * kAStride + o + j], s2);
      s3 = fmaf(tv.w, am[(o + N + p + 3) * kAStride + o + j], s3);
    }
    acc[e] = -((s0 + s1) + (s2 + s3));
  }
  named_bar(1, NTH);
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    const int idx = tid + e * NTH;
    const int pr = idx / (N * N), rem = idx % (N * N);
    am[(pr * 2 * N + N + rem / N) * kAStride + pr * 2 * N + rem % N] = acc[e];
  }
  named_bar(1, NTH);
}

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
  named_bar(1, 128);
  inv_level<8>(am, ptid);
  inv_level<16>(am, ptid);
  inv_level<32>(am, ptid);
}

}  // namespace gdn
