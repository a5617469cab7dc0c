// Two-kernel chunked GDN forward for B200 (sm_100a).
//
// Per chunk of C = 64 steps (b = in-chunk cumsum of g, gdn_ref.py:76-99), the
// state update and the output are affine in the chunk-start state S = h^T
// (K x V):
//
//   S' = e^{b_C} S + N S + c            N = -Kbar^T W          (K x K)
//                                      c =  Kbar^T U          (K x V)
//   o  = Q' S + o_intra                 Q' = Qhat - P W        (C x K)
//                                      o_intra = P U          (C x V)
//
// with Kbar = e^{b_C - b} k, Qhat = e^{b} q, P = tril(Q K^T * e^{b_t - b_j}),
// W = T diag(beta e^b) K, U = T diag(beta) V, T = (I + A)^-1.  This is the
// reference's own two-GEMM state update h0 (e^{b_C} I - Wbar^T K) + Ubar^T K
// (gdn_ref.py:92-98) and its output u-form (gdn_ref.py:86-90) regrouped so
// that everything except one K x K by K x V product per chunk is independent
// of the state.
//
//   gdn_wy_kernel   chunk-parallel, one CTA per (b, h, chunk), two per SM:
//                   S = [K;Q]K^T -> A, P; T in fp32; W, U (U split hi + lo);
//                   then N, c, Q', o_intra on the tensor cores, stored from
//                   registers as a 96 KB packet of chunk-major fp16 images
//                   that the scan feeds to its tensor cores as they are.
//   gdn_scan_kernel one CTA per (b, h, 32-wide V slice), serial over chunks:
//                   one 128x128x32 product per chunk on the critical path
//                   (N S), plus Q' S off it; the state stays in registers.
//
// The packets are scratch memory (kPacketBytesPerChunk per (b, h, chunk));
// long sequences are processed in segments of chunks so the scratch stays
// bounded, the state being carried between segments.
#include "gdn_common.cuh"
#include "tmap.h"
#include "gdn_wy_scan.h"
#include "../../include/gdn_b200.h"

#include <cuda_runtime.h>

namespace gdn {

constexpr uint32_t kPacketBytes = uint32_t(kPacketBytesPerChunk);
// packet layout (bytes)
// Every piece is chunk-major: 16-byte chunk j (8 consecutive columns) of row r
// sits at (j * rows + r) * 16.  The prep writes it straight from the TMEM-row
// layout (a warp stores 32 consecutive rows of one chunk: 512 contiguous
// bytes), and for N and Q' it is the no-swizzle K-major operand layout of the
// scan's MMAs (8-row x 16-byte core matrices; next chunk = next K core matrix).
namespace pkt {
constexpr uint32_t kN = 0;        // N fp16, 128 x 128: 16 chunks x 128 rows
constexpr uint32_t kQ = 32768;    // Q' fp16, 64 x 128: 16 chunks x 64 rows
constexpr uint32_t kHdr = 49152;  // fp32 e^{b_C}
constexpr uint32_t kCs = 49408;   // c fp16, 4 V slices x (4 chunks x 128 rows)
constexpr uint32_t kOs = 82176;   // o_intra fp16, 4 V slices x (4 chunks x 64 rows)
static_assert(kOs + 4 * 4096 == kPacketBytesPerChunk, "packet size");
}  // namespace pkt

// =========================================================== prep kernel
namespace wy {
// warps 0-7: prep (warp w reads TMEM lane quarter w & 3 and takes column half w >> 2);
// warp 8: TMA + MMA
constexpr int kThreads = 288;
constexpr int kPrep = 256;
constexpr int kMmaWarp = 8;
// Column blocks of 64 elements (128-byte rows, 128B swizzle).  k0, k1, v0, v1
// sit 16 KB apart so that [K | V] is one N = 256 MN-major operand.
constexpr uint32_t k0 = 0, q0 = 8192, k1 = 16384, q1 = 24576;
constexpr uint32_t v0 = 32768, v1 = 49152;                     // later U_lo fp16
constexpr uint32_t p16 = 40960;    // P fp16, 64 x 128 B
constexpr uint32_t tw = 57344;     // [Tw_hi; Tb_hi] (input dtype): one M = 128 operand; later W fp16
constexpr uint32_t zz = 73728;     // [Tw_lo; Tb_lo]: one M = 128 operand; later U_hi fp16
constexpr uint32_t amat = 90112;   // fp32 A / T (64 x kAStride); later Kbar fp16
// Kbar = e^{b_C - b} k (fp16, two 64-column blocks, 128B swizzle) is written
// over A / T, dead after the T split: k's own buffer is then free for the
// next chunk's k as soon as epilogue A has read it.
constexpr uint32_t kbar = amat;
constexpr uint32_t vec = amat + 17408;  // 2 buffers (item parity) x kVecN x 64 fp32
constexpr uint32_t kVecBytes = kVecN * kC * 4;
constexpr uint32_t bars = vec + 2 * kVecBytes;
constexpr uint32_t misc = bars + 24 * 8;
constexpr uint32_t total = misc + 32;
constexpr uint32_t alloc = total + 1024;
static_assert(kC * kAStride * 4 <= 17408 && 2 * 8192 <= 17408, "A/T region");
static_assert(amat % 1024 == 0, "Kbar tiles are 1024-byte aligned");
static_assert(2 * (alloc + 1024) <= 233472, "two CTAs per SM");
// TMEM columns: S 0-63 (M=128); [W | Tw V ; Tb K | U] 0-255 (M=128: W = lanes 0-63 cols 0-127,
// U = lanes 64-127 cols 128-255); PW 0-127, PU 128-255 (M=64); N 0-127, c 128-255 (M=128).
// Packet pieces go from registers straight to global memory (chunk-major, so
// every warp store is 512 contiguous bytes): no staging, and nothing to drain
// before the CTA leaves.  The stores carry an L2 evict-last policy so that as
// many packets as fit are still in L2 when the scan reads them (the scan loads
// its private c / o_intra slices evict-first); measured 1.3 % per forward.
//
// The kernel is persistent: its CTAs claim items (chunks) in order from a
// counter in the workspace, one item ahead of the one they run, so the items in
// flight at any time are a contiguous range, as with one CTA per item, and
// no SM is left with a single CTA at the end.  Each mbarrier completes one phase per item
// (B_NSR / B_NSD an even number), so an item's phases have parity (item & 1).
// The next item's inputs are loaded while this one finishes, each as soon as
// its buffer is free: k after epilogue A (Kbar is out), q after epilogue C,
// v (later U_lo) after the N / c products; its S product (TMEM columns 0-63)
// is issued as soon as epilogue B has read those columns, while the rest of
// epilogue B runs.  Its g and beta are read and its vectors written (into the
// other of two buffers) right after this item's S product is issued, while the
// prep warps run the inverse, so neither the next S product nor the MMA
// warp's response to the epilogues waits on them (measured: vectors computed
// after the N / c issue kept the prep warps idle ~7.8k of ~30k cycles per item).
// B_STARTED keeps the MMA warp from completing the next item's B_VEC phase
// before every prep warp has waited on this item's.
enum {
  B_FULLK = 0,  // k landed
  B_FULLQ,      // q landed
  B_FULLV,      // v landed (first read by the W | U product)
  B_VEC,        // the item's cumsum / beta vectors written (MMA warp)
  B_STARTED,    // every prep warp has passed the item's B_VEC wait
  B_SFULL,
  B_TREADY,
  B_WUFULL,
  B_EPA,
  B_PFULL,
  B_EPC,
  B_NCFULL,
  B_EPB,        // epilogue B has read TMEM columns 0-63 (warps 0-3): the next S may go there
  B_NORM,
  B_NSR,
  B_NSD,
  B_DONE,
  B_COUNT
};
static_assert(B_COUNT <= 24, "barrier region");
}  // namespace wy

__device__ __forceinline__ uint4 pack8_f16(const float* x) {
  uint4 w;
  w.x = Cvt<__half>::pack(x[0], x[1]);
  w.y = Cvt<__half>::pack(x[2], x[3]);
  w.z = Cvt<__half>::pack(x[4], x[5]);
  w.w = Cvt<__half>::pack(x[6], x[7]);
  return w;
}

// Newton-Schulz alternative to invert_unit_lower64, after gdn_triton_v2.py:58-68:
// M = I + A and X = I - A as fp16 operands, then `iters` times
//     Y = 2I - M X,   X = X Y
// with fp16 operands and fp32 accumulation on the tensor cores (M=64, N=64,
// K=64; issued by the MMA warp, results in TMEM columns 0-63, row 16 w + l in
// lane 32 w + l).  The final X (fp32) replaces A in `am`.  Exact only when A^(2^(iters+1))
// vanishes (iters >= 5 for C = 64); the fp16 operands bound its accuracy.
// Called by NP = 256 threads (warp w: lane quarter w & 3, column half w >> 2).
template <int NP>
__device__ __forceinline__ bool ns_solve64(float* am, uint8_t* m16, uint8_t* x16, uint8_t* y16, uint32_t tmem,
                                           uint64_t* nsr, uint64_t* nsd, int iters, volatile int* abort_flag) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  {
    // M and X from A (rows rr, 16-byte chunks 2 cq, 2 cq + 1)
    const int rr = tid >> 2, cq = tid & 3;
    const float* arow = am + rr * kAStride;
#pragma unroll
    for (int c = 2 * cq; c < 2 * cq + 2; ++c) {
      float mv[8], xv[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int m = 8 * c + e;
        const float a = arow[m], d = (m == rr) ? 1.f : 0.f;
        mv[e] = d + a;
        xv[e] = d - a;
      }
      *reinterpret_cast<uint4*>(m16 + sw128_off(rr, c)) = pack8_f16(mv);
      *reinterpret_cast<uint4*>(x16 + sw128_off(rr, c)) = pack8_f16(xv);
    }
  }
  fence_async_smem();
  __syncwarp();
  if (lane == 0) mbar_arrive(nsr);
  const int lq = warp & 3, hc = warp >> 2;
  const int t = 16 * lq + (lane & 15);
  bool ok = true;
  for (int it = 0; it < iters; ++it) {
#pragma unroll 1
    for (int h = 0; h < 2; ++h) {
      ok = mbar_wait_warp(nsd, h & 1, abort_flag);  // phase 2 it + h
      if (bar_any(1, NP, !ok || *abort_flag)) return false;
      tc_fence_after();
      float x[32];
      tmem_ld32w(tmem_addr(tmem, lq * 32, 32 * hc), x);
      tc_fence_before();
      const bool last = (h == 1) && (it + 1 == iters);
      if (lane < 16) {
        if (h == 0) {
          // Y = 2I - M X
#pragma unroll
          for (int e = 0; e < 32; ++e) x[e] = ((32 * hc + e == t) ? 2.f : 0.f) - x[e];
        }
        if (last) {
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            *reinterpret_cast<float4*>(am + t * kAStride + 32 * hc + e) = make_float4(x[e], x[e + 1], x[e + 2], x[e + 3]);
        } else {
          uint8_t* dst = h == 0 ? y16 : x16;
#pragma unroll
          for (int c = 0; c < 4; ++c)
            *reinterpret_cast<uint4*>(dst + sw128_off(t, 4 * hc + c)) = pack8_f16(x + 8 * c);
        }
      }
      if (!last) {
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(nsr);
      }
    }
  }
  named_bar(1, NP);  // T visible in am to every thread
  return ok;
}

// Item order of the prep: the segment's chunks fall into blocks of P.blk_len
// consecutive chunks, taken last block first, head-major inside a block (one
// head's chunks run back to back, so its input rows and its packets are read and
// written in address order).  The packets written last are the ones still in
// L2 when the scan starts, and the scan starts at the segment's first chunks:
// with several blocks those are the first block's packets instead of the last
// heads' final chunks (T = 65536: 2.54 vs 2.59 ms per forward with 4 blocks).
// One block (blk_len >= NS) is plain head-major order: the kernel's kBlocked =
// false instantiation, which carries none of this code (its presence alone cost
// 0.8 % at T = 4096).
__device__ __forceinline__ void wy_item_blocked(const WyParams& P, int x, int& il, int& bh) {
  const int nbh = P.B * P.H;
  for (int lo = (P.NS - 1) / P.blk_len * P.blk_len; lo >= 0; lo -= P.blk_len) {
    const int n = min(P.NS - lo, P.blk_len);
    if (x < nbh * n) {
      bh = x / n;
      il = lo + (x - bh * n);
      return;
    }
    x -= nbh * n;
  }
  il = -1;  // past the last item
  bh = 0;
}

template <bool kBlocked>
__device__ __forceinline__ void wy_item(const WyParams& P, int x, int& il, int& bh) {
  if constexpr (kBlocked) {
    wy_item_blocked(P, x, il, bh);
  } else {
    il = x % P.NS;
    bh = x / P.NS;
  }
}

// g and beta of steps t0 + lane and t0 + lane + 32 of head (bb, hh), as the
// kernels use them (zero past T, gdn_ref.py:102-114; activations applied).
struct WyStepVals {
  float ga, gb, ba, bb;
};
__device__ __forceinline__ WyStepVals wy_step_vals(const WyParams& P, int bb, int hh, int t0, int lane) {
  const float* gp = P.g == nullptr ? nullptr : P.g + bb * P.sg_b + hh * P.sg_h;
  const float* bp = P.beta + bb * P.sb_b + hh * P.sb_h;
  const int ta = t0 + lane, tb = t0 + lane + 32;
  WyStepVals r;
  r.ga = load_g(gp, (long long)ta * P.sg_t, ta < P.T, P.flags);
  r.gb = load_g(gp, (long long)tb * P.sg_t, tb < P.T, P.flags);
  r.ba = load_beta(bp, (long long)ta * P.sb_t, ta < P.T, P.flags);
  r.bb = load_beta(bp, (long long)tb * P.sb_t, tb < P.T, P.flags);
  return r;
}

// In-chunk cumsum of g (log2 units), beta, e^b and e^{b_C - b} of one chunk
// into vec, from its WyStepVals.  Whole warp.
__device__ __forceinline__ void wy_vectors(const WyStepVals& sv, float* vec, int lane) {
  constexpr float kLog2e = 1.4426950408889634f;
  float xa = sv.ga * kLog2e;
  float xb = sv.gb * kLog2e;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const float ya = __shfl_up_sync(0xffffffffu, xa, d);
    const float yb = __shfl_up_sync(0xffffffffu, xb, d);
    if (lane >= d) {
      xa += ya;
      xb += yb;
    }
  }
  xb += __shfl_sync(0xffffffffu, xa, 31);
  const float bC = __shfl_sync(0xffffffffu, xb, 31);
  vec[V_B2 * kC + lane] = xa;
  vec[V_B2 * kC + lane + 32] = xb;
  vec[V_BETA * kC + lane] = sv.ba;
  vec[V_BETA * kC + lane + 32] = sv.bb;
  vec[V_EB * kC + lane] = fast_exp2(xa);
  vec[V_EB * kC + lane + 32] = fast_exp2(xb);
  vec[V_DD * kC + lane] = fast_exp2(bC - xa);
  vec[V_DD * kC + lane + 32] = fast_exp2(bC - xb);
}

// q/k L2 normalisation in the kernel (gdn_ref.py:24-25): every row of the raw
// q and k tiles divided by sqrt(sum of squares + 1e-6) in fp32, in place.
// Thread pair (2i, 2i+1) takes the two 64-column blocks of row i (k rows, then
// q rows).  Out of line: inlined, its registers pushed the rest of the kernel
// into spills (the kernel runs at 96 registers for two CTAs per SM).
template <typename InT>
__device__ __noinline__ void l2norm_qk_rows(uint8_t* sm, int ptid) {
  const int rr = ptid >> 1, half = ptid & 1, t = rr & 63;
  uint8_t* blk = sm + (rr < 64 ? wy::k0 : wy::q0) + half * 16384;
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const uint4 x = *reinterpret_cast<const uint4*>(blk + sw128_off(t, c));
    const uint32_t w4[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = Cvt<InT>::unpack(w4[e]);
      ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
    }
  }
  ss += __shfl_xor_sync(0xffffffffu, ss, 1);
  const float inv = 1.f / sqrtf(ss + 1e-6f);
  // second pass re-reads the row from shared memory rather than holding it
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const uint4 x = *reinterpret_cast<const uint4*>(blk + sw128_off(t, c));
    const uint32_t w4[4] = {x.x, x.y, x.z, x.w};
    uint32_t y4[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = Cvt<InT>::unpack(w4[e]);
      y4[e] = Cvt<InT>::pack(f.x * inv, f.y * inv);
    }
    *reinterpret_cast<uint4*>(blk + sw128_off(t, c)) = make_uint4(y4[0], y4[1], y4[2], y4[3]);
  }
}

template <typename InT, bool kBlocked>
__global__ void __launch_bounds__(wy::kThreads, 2) gdn_wy_kernel(const __grid_constant__ WyParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + wy::bars);
  uint32_t* tmem_base_p = reinterpret_cast<uint32_t*>(sm + wy::misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + wy::misc + 4);
  float* amat = reinterpret_cast<float*>(sm + wy::amat);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nitems = P.B * P.H * P.NS;
  // item of each parity slot, written by the MMA warp before its B_VEC arrival
  // (-1: no further item, the prep warps leave)
  volatile int* slot_item = reinterpret_cast<volatile int*>(sm + wy::misc + 8);

  if (warp == wy::kMmaWarp) {
    if (lane == 0) {
      for (int i = 0; i < wy::B_COUNT; ++i)
        mbar_init(&bars[i], (i == wy::B_TREADY || i == wy::B_EPA || i == wy::B_EPC || i == wy::B_NORM ||
                             i == wy::B_NSR || i == wy::B_STARTED)
                                ? wy::kPrep / 32
                                : (i == wy::B_EPB ? wy::kPrep / 64 : 1));
      *abort_flag = 0;
      fence_mbar_init();
    }
    tmem_alloc(tmem_base_p, 256);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_p;
  const uint32_t sb = smem_u32(sm);
  constexpr uint32_t kInBf16 = Cvt<InT>::kIsBf16;

  if (warp == wy::kMmaWarp) {
    // ------------------------------------------------ TMA, vectors and MMA issue (the whole warp; elect.sync inside)
    float* vec_buf = reinterpret_cast<float*>(sm + wy::vec);
    uint32_t nk = 0, nq = 0, nv = 0;  // loads issued on B_FULLK / B_FULLQ / B_FULLV
    auto load_k = [&](int t0, int hh, int bb) {
      if (lane == 0) {
        mbar_arrive_expect_tx(&bars[wy::B_FULLK], 16384);
        tma_load_4d(sm + wy::k0, &P.tm_k, &bars[wy::B_FULLK], 0, t0, hh, bb);
        tma_load_4d(sm + wy::k1, &P.tm_k, &bars[wy::B_FULLK], 64, t0, hh, bb);
      }
      ++nk;
    };
    auto load_q = [&](int t0, int hh, int bb) {
      if (lane == 0) {
        mbar_arrive_expect_tx(&bars[wy::B_FULLQ], 16384);
        tma_load_4d(sm + wy::q0, &P.tm_q, &bars[wy::B_FULLQ], 0, t0, hh, bb);
        tma_load_4d(sm + wy::q1, &P.tm_q, &bars[wy::B_FULLQ], 64, t0, hh, bb);
      }
      ++nq;
    };
    auto load_v = [&](int t0, int hh, int bb) {
      if (lane == 0) {
        mbar_arrive_expect_tx(&bars[wy::B_FULLV], 16384);
        tma_load_4d(sm + wy::v0, &P.tm_v, &bars[wy::B_FULLV], 0, t0, hh, bb);
        tma_load_4d(sm + wy::v1, &P.tm_v, &bars[wy::B_FULLV], 64, t0, hh, bb);
      }
      ++nv;
    };
    // Each CTA's first item is its blockIdx (no atomic on the path of the
    // first item, which all CTAs start at once); the items after the first
    // G are claimed one ahead from the segment's counter (zeroed before the
    // launch), so CTAs that run faster take more items and all finish together
    // (a fixed round-robin left one CTA per SM running the last items alone).
    auto claim = [&]() -> int {
      int x = 0;
      if (lane == 0) x = int(atomicAdd(P.work, 1u)) + int(gridDim.x);
      return __shfl_sync(0xffffffffu, x, 0);
    };
    bool ok = true;
    int cur = int(blockIdx.x);
    if (cur < nitems) {
      int il, bh;
      wy_item<kBlocked>(P, cur, il, bh);
      const int t0 = (P.c0 + il) * kC, hh = bh % P.H, bb = bh / P.H;
      // g and beta first: these small loads would otherwise queue behind
      // the whole grid's q / k / v tiles (measured: the first vectors took
      // ~9k cycles after the CTA started)
      const WyStepVals sv0 = wy_step_vals(P, bb, hh, t0, lane);
      load_k(t0, hh, bb);
      load_q(t0, hh, bb);
      load_v(t0, hh, bb);
      wy_vectors(sv0, vec_buf, lane);
    }
    if (lane == 0) slot_item[0] = cur < nitems ? cur : -1;
    __syncwarp();
    if (lane == 0) mbar_arrive(&bars[wy::B_VEC]);
    for (int it = 0; cur < nitems && ok; ++it) {
      const uint32_t ph = uint32_t(it) & 1u;
      ok = mbar_wait_warp(&bars[wy::B_FULLK], ph, abort_flag) && mbar_wait_warp(&bars[wy::B_FULLQ], ph, abort_flag);
      if (P.flags & GDN_FLAG_QK_L2NORM) ok = ok && mbar_wait_warp(&bars[wy::B_NORM], ph, abort_flag);
      if (it > 0) ok = ok && mbar_wait_warp(&bars[wy::B_EPB], ph ^ 1u, abort_flag);  // columns 0-63 read
      if (!ok) break;
      // S = [K;Q] K^T: M=128 (k rows then q rows), N=64, K=128
      tc_fence_after();
      const uint32_t id_s = idesc_f16(128, 64, kInBf16, 0, 0);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t a = sb + wy::k0 + (kk >> 2) * 16384 + (kk & 3) * 32;
        mma_f16_ss_warp(tmem, sdesc(a, 16, 1024, kSw128), sdesc(a, 16, 1024, kSw128), id_s, kk > 0);
      }
      mma_commit_warp(&bars[wy::B_SFULL]);
      // the next item, claimed after this S product is issued so that the
      // claim's atomic never delays it
      const int next = claim();
      const bool has_next = next < nitems;
      int nt0 = 0, nhh = 0, nbb = 0;
      if (has_next) {
        int nil, nbh;
        wy_item<kBlocked>(P, next, nil, nbh);
        nt0 = (P.c0 + nil) * kC;
        nhh = nbh % P.H;
        nbb = nbh / P.H;
        if (lane == 0) {  // the next item's inputs into L2 now; its loads start during this item
          tma_prefetch_4d(&P.tm_k, 0, nt0, nhh, nbb);
          tma_prefetch_4d(&P.tm_k, 64, nt0, nhh, nbb);
          tma_prefetch_4d(&P.tm_q, 0, nt0, nhh, nbb);
          tma_prefetch_4d(&P.tm_q, 64, nt0, nhh, nbb);
          tma_prefetch_4d(&P.tm_v, 0, nt0, nhh, nbb);
          tma_prefetch_4d(&P.tm_v, 64, nt0, nhh, nbb);
        }
      }
      {
        // the next item (or the end) for the prep warps, with its vectors in
        // the other buffer, while they run A / P and the inverse: that buffer's
        // previous item read it for the last time in its epilogue C, and
        // B_STARTED says every prep warp has waited on this item's B_VEC phase
        WyStepVals nsv = {0.f, 0.f, 0.f, 0.f};
        if (has_next) nsv = wy_step_vals(P, nbb, nhh, nt0, lane);
        ok = mbar_wait_warp(&bars[wy::B_STARTED], ph, abort_flag);
        if (!ok) break;
        if (has_next) wy_vectors(nsv, vec_buf + (ph ^ 1u) * (wy::kVecBytes / 4), lane);
        if (lane == 0) slot_item[ph ^ 1u] = has_next ? next : -1;
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[wy::B_VEC]);
      }
      // Newton-Schulz solve (gdn_triton_v2.py:58-68): per iteration M X, then X (2I - M X),
      // fp16 operands written by the prep warps: M at tw, X at tw + 8 KB, 2I - M X at zz
      const int ns_iters = (P.flags >> GDN_FLAG_NS_ITERS_SHIFT) & 15;
      if (P.flags & GDN_FLAG_SOLVER_NS) {
        const uint32_t id_ns = idesc_f16(64, 64, 0, 0, 1);
        for (int nit = 0; nit < ns_iters && ok; ++nit) {
#pragma unroll 1
          for (int h = 0; h < 2 && ok; ++h) {
            ok = mbar_wait_warp(&bars[wy::B_NSR], h & 1, abort_flag);  // phase 2 nit + h
            if (!ok) break;
            tc_fence_after();
            const uint32_t a = sb + wy::tw + (h ? 8192 : 0), b = sb + (h ? wy::zz : wy::tw + 8192);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_f16_ss_warp(tmem, sdesc(a + kk * 32, 16, 1024, kSw128), sdesc(b + kk * 2048, 8192, 1024, kSw128),
                              id_ns, kk > 0);
            mma_commit_warp(&bars[wy::B_NSD]);
          }
        }
      }
      ok = ok && mbar_wait_warp(&bars[wy::B_TREADY], ph, abort_flag) &&
           mbar_wait_warp(&bars[wy::B_FULLV], ph, abort_flag);
      if (!ok) break;
      // ([Tw_hi; Tb_hi] + [Tw_lo; Tb_lo]) [K | V] (M=128, N=256, K=64 twice):
      // W = lanes 0-63 x cols 0-127, U = lanes 64-127 x cols 128-255.  Both T
      // operands are split hi + lo in the input dtype: with bf16 inputs one
      // 8-bit-mantissa copy of T alone costs ~1e-3 on the final state when g is
      // small (slow decay keeps every chunk's error).
      tc_fence_after();
      const uint32_t id_wu = idesc_f16(128, 256, kInBf16, 0, 1);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        mma_f16_ss_warp(tmem, sdesc(sb + (kk < 4 ? wy::tw : wy::zz) + (kk & 3) * 32, 16, 1024, kSw128),
                        sdesc(sb + wy::k0 + (kk & 3) * 2048, 16384, 1024, kSw128), id_wu, kk > 0);
      mma_commit_warp(&bars[wy::B_WUFULL]);
      ok = mbar_wait_warp(&bars[wy::B_EPA], ph, abort_flag);
      if (!ok) break;
      if (has_next) load_k(nt0, nhh, nbb);  // epilogue A has read k and written Kbar elsewhere
      // P W -> cols 0-127, P (U_hi + U_lo) -> cols 128-255  (M=64, N=128, K=64; B MN-major)
      tc_fence_after();
      const uint32_t id_p = idesc_f16(64, 128, 0, 0, 1);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        mma_f16_ss_warp(tmem, sdesc(sb + wy::p16 + kk * 32, 16, 1024, kSw128),
                        sdesc(sb + wy::tw + kk * 2048, 8192, 1024, kSw128), id_p, kk > 0);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        mma_f16_ss_warp(tmem + 128, sdesc(sb + wy::p16 + (kk & 3) * 32, 16, 1024, kSw128),
                        kk < 4 ? sdesc(sb + wy::zz + (kk & 3) * 2048, 8192, 1024, kSw128)
                               : sdesc(sb + wy::v0 + (kk & 3) * 2048, 16384, 1024, kSw128),
                        id_p, kk > 0);
      mma_commit_warp(&bars[wy::B_PFULL]);
      ok = mbar_wait_warp(&bars[wy::B_EPC], ph, abort_flag);
      if (!ok) break;
      // Kbar^T W -> cols 0-127, Kbar^T (U_hi + U_lo) -> cols 128-255  (M=128, N=128, K=64; A and B MN-major)
      tc_fence_after();
      const uint32_t id_n = idesc_f16(128, 128, 0, 1, 1);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        mma_f16_ss_warp(tmem, sdesc(sb + wy::kbar + kk * 2048, 8192, 1024, kSw128),
                        sdesc(sb + wy::tw + kk * 2048, 8192, 1024, kSw128), id_n, kk > 0);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        mma_f16_ss_warp(tmem + 128, sdesc(sb + wy::kbar + (kk & 3) * 2048, 8192, 1024, kSw128),
                        kk < 4 ? sdesc(sb + wy::zz + (kk & 3) * 2048, 8192, 1024, kSw128)
                               : sdesc(sb + wy::v0 + (kk & 3) * 2048, 16384, 1024, kSw128),
                        id_n, kk > 0);
      mma_commit_warp(&bars[wy::B_NCFULL]);
      if (has_next) {
        load_q(nt0, nhh, nbb);  // epilogue C was the last reader of q
        // v's buffer holds U_lo until the N / c products complete
        ok = mbar_wait_warp(&bars[wy::B_NCFULL], ph, abort_flag);
        if (!ok) break;
        load_v(nt0, nhh, nbb);
      }
      cur = next;
    }
    if (!ok && lane == 0) *abort_flag = 1;
    __syncwarp();
    if (!ok) {
      // a failed wait: let the loads in flight land before the CTA releases its smem
      if (lane == 0) {
        volatile int never = 0;
        if (nk) mbar_wait(&bars[wy::B_FULLK], (nk - 1) & 1, &never);
        if (nq) mbar_wait(&bars[wy::B_FULLQ], (nq - 1) & 1, &never);
        if (nv) mbar_wait(&bars[wy::B_FULLV], (nv - 1) & 1, &never);
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------ prep (warps 0-7)
    constexpr int NP = wy::kPrep;
    const int ptid = tid;                     // 0..255
    const int lq = warp & 3, hc = warp >> 2;  // TMEM lane quarter, column half
    const int r = (lq << 5) | lane;           // TMEM lane = row of an M=128 accumulator
    for (int it = 0;; ++it) {
      const uint32_t ph = uint32_t(it) & 1u;
      bool ok = mbar_wait_warp(&bars[wy::B_VEC], ph, abort_flag);
      if (bar_any(1, NP, !ok || *abort_flag)) break;
      const int x = slot_item[ph];
      if (x < 0) break;  // the same value for every prep warp: no further item
      int il, bh;
      wy_item<kBlocked>(P, x, il, bh);
      uint8_t* const pkg = P.packets + (size_t(bh) * P.NS + il) * kPacketBytes;
      const float* vec = reinterpret_cast<const float*>(sm + wy::vec + ph * wy::kVecBytes);
      if (lane == 0) mbar_arrive(&bars[wy::B_STARTED]);
      const float b2first = vec[V_B2 * kC], b2last = vec[V_B2 * kC + kC - 1];
      const float ref = 0.5f * (b2first + b2last);
      const bool prod_form = (b2first - b2last) < 200.f;
      if (ptid < 64) amat[ptid * kAStride + 64] = fast_exp2(ref - vec[V_B2 * kC + ptid]);
      named_bar(2, NP);
      if (P.flags & GDN_FLAG_QK_L2NORM) {
        // raw q and k normalised in place before any product reads them
        if (mbar_wait_warp(&bars[wy::B_FULLK], ph, abort_flag) && mbar_wait_warp(&bars[wy::B_FULLQ], ph, abort_flag)) {
          l2norm_qk_rows<InT>(sm, ptid);
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[wy::B_NORM]);
      }
      ok = mbar_wait_warp(&bars[wy::B_SFULL], ph, abort_flag);
      if (bar_any(1, NP, !ok || *abort_flag)) break;
      {
        tc_fence_after();
        // rows 0-63: A[t][m] = beta_t exp(b_t - b_m) (k_t.k_m), m < t   (TMEM lanes 0-63 = K K^T)
        // rows 64-127: P[t][m] = exp(b_t - b_m) (q_t.k_m), m <= t      (lanes 64-127 = Q K^T)
        const int t = r & 63;
        const float b2t = vec[V_B2 * kC + t];
        const float et = fast_exp2(b2t - ref);
        const float bt = (r < 64) ? vec[V_BETA * kC + t] : 1.f;
        float* arow = amat + t * kAStride;
        uint8_t* pimg = sm + wy::p16;
#pragma unroll 1
        for (int cg = 2 * hc; cg < 2 * hc + 2; ++cg) {
          float sv[16];
          tmem_ld16w(tmem_addr(tmem, lq * 32, cg * 16), sv);
          float x[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int m = cg * 16 + e;
            const float dec = prod_form ? et * amat[m * kAStride + 64] : fast_exp2(b2t - vec[V_B2 * kC + m]);
            const bool keep = (r < 64) ? (m < t) : (m <= t);
            x[e] = keep ? bt * dec * sv[e] : 0.f;
          }
          if (r < 64) {
#pragma unroll
            for (int e = 0; e < 16; e += 4)
              *reinterpret_cast<float4*>(arow + cg * 16 + e) = make_float4(x[e], x[e + 1], x[e + 2], x[e + 3]);
          } else {
            *reinterpret_cast<uint4*>(pimg + sw128_off(t, 2 * cg)) = pack8_f16(x);
            *reinterpret_cast<uint4*>(pimg + sw128_off(t, 2 * cg + 1)) = pack8_f16(x + 8);
          }
        }
        tc_fence_before();
        named_bar(1, NP);
        if (P.flags & GDN_FLAG_SOLVER_NS)
          ok = ns_solve64<NP>(amat, sm + wy::tw, sm + wy::tw + 8192, sm + wy::zz, tmem, &bars[wy::B_NSR],
                              &bars[wy::B_NSD], (P.flags >> GDN_FLAG_NS_ITERS_SHIFT) & 15, abort_flag);
        else
          // T = (I + A)^-1 in place; the doubling intermediates go to the
          // T operand buffer, unused until the split below
          invert_unit_lower64_scr<NP>(amat, reinterpret_cast<float*>(sm + wy::tw), ptid);
        if (!ok) break;  // uniform: ns_solve64 decides through bar_any
        // Tw = T diag(beta e^b), Tb = T diag(beta), each split hi + lo in the input dtype:
        // [Tw_hi; Tb_hi] and [Tw_lo; Tb_lo]
        {
          const int rr = ptid >> 2, cq = ptid & 3;
          const float* trow = amat + rr * kAStride;
          uint8_t* twh = sm + wy::tw;
          uint8_t* tbh = sm + wy::tw + 8192;
          uint8_t* twl = sm + wy::zz;
          uint8_t* tbl = sm + wy::zz + 8192;
#pragma unroll
          for (int c = 2 * cq; c < 2 * cq + 2; ++c) {
            uint32_t wh[4], wl[4], hi[4], lo[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int m = 8 * c + 2 * e;
              const float tb0 = trow[m] * vec[V_BETA * kC + m], tb1 = trow[m + 1] * vec[V_BETA * kC + m + 1];
              const float tw0 = tb0 * vec[V_EB * kC + m], tw1 = tb1 * vec[V_EB * kC + m + 1];
              wh[e] = Cvt<InT>::pack(tw0, tw1);
              const float2 wf = Cvt<InT>::unpack(wh[e]);
              wl[e] = Cvt<InT>::pack(tw0 - wf.x, tw1 - wf.y);
              hi[e] = Cvt<InT>::pack(tb0, tb1);
              const float2 hf = Cvt<InT>::unpack(hi[e]);
              lo[e] = Cvt<InT>::pack(tb0 - hf.x, tb1 - hf.y);
            }
            const uint32_t off = sw128_off(rr, c);
            *reinterpret_cast<uint4*>(twh + off) = make_uint4(wh[0], wh[1], wh[2], wh[3]);
            *reinterpret_cast<uint4*>(twl + off) = make_uint4(wl[0], wl[1], wl[2], wl[3]);
            *reinterpret_cast<uint4*>(tbh + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
            *reinterpret_cast<uint4*>(tbl + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
          }
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[wy::B_TREADY]);
        // A / T is dead from here; epilogue A writes Kbar over it once the W | U
        // product, issued after every warp's B_TREADY arrival, has completed
      }
      // ---- epilogue A: rows 0-63 W -> fp16 [t][k] (over [Tw; Tb_hi]); rows 64-127 U -> fp16
      //      hi (over [Tw_lo; Tb_lo]) and lo (over v); and Kbar = e^{b_C - b_t} k fp16 (over A / T)
      ok = mbar_wait_warp(&bars[wy::B_WUFULL], ph, abort_flag);
      if (ok) {
        tc_fence_after();
        const int t = r & 63;
        const bool isw = r < 64;
#pragma unroll 1
        for (int c0 = 64 * hc; c0 < 64 * hc + 64; c0 += 32) {
          float x[32];
          tmem_ld32w(tmem_addr(tmem, lq * 32, (isw ? 0 : 128) + c0), x);
          const uint32_t chunk0 = (c0 & 63) >> 3;
          if (isw) {
            uint8_t* dst = sm + wy::tw + (c0 >> 6) * 8192;
#pragma unroll
            for (int c = 0; c < 4; ++c)
              *reinterpret_cast<uint4*>(dst + sw128_off(t, chunk0 + c)) = pack8_f16(x + 8 * c);
          } else {
            uint8_t* dhi = sm + wy::zz + (c0 >> 6) * 8192;
            uint8_t* dlo = sm + wy::v0 + (c0 >> 6) * 16384;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              float hi[8], lo[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                hi[e] = __half2float(__float2half_rn(x[8 * c + e]));
                lo[e] = x[8 * c + e] - hi[e];
              }
              const uint32_t off = sw128_off(t, chunk0 + c);
              *reinterpret_cast<uint4*>(dhi + off) = pack8_f16(hi);
              *reinterpret_cast<uint4*>(dlo + off) = pack8_f16(lo);
            }
          }
        }
        if (isw) {
          // Kbar, both 64-column blocks of row t, by the W-row warps only: the
          // U-row warps carry the hi / lo split above, the larger share
          const float dd = vec[V_DD * kC + t];
#pragma unroll
          for (int b = 0; b < 2; ++b) {
            const uint8_t* ks = sm + (b ? wy::k1 : wy::k0);
            uint8_t* kd = sm + wy::kbar + b * 8192;
#pragma unroll
            for (int c = 4 * hc; c < 4 * hc + 4; ++c) {
              const uint4 x = *reinterpret_cast<const uint4*>(ks + sw128_off(t, c));
              const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
              uint32_t ys[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 f = Cvt<InT>::unpack(xs[e]);
                ys[e] = Cvt<__half>::pack(f.x * dd, f.y * dd);
              }
              *reinterpret_cast<uint4*>(kd + sw128_off(t, c)) = make_uint4(ys[0], ys[1], ys[2], ys[3]);
            }
          }
        }
        fence_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[wy::B_EPA]);
      }
      // ---- epilogue C: Q' = e^{b_t} q_t - (P W)_t and o_intra = P U (M=64: row 16 lq + l in
      //      lane 32 lq + l, l < 16), straight to the packet; e^{b_C}
      ok = ok && mbar_wait_warp(&bars[wy::B_PFULL], ph, abort_flag);
      if (bar_any(1, NP, !ok || *abort_flag)) break;  // uniform: named barriers follow
      {
        tc_fence_after();
        const int t = 16 * lq + (lane & 15);
        const float eb = vec[V_EB * kC + t];
        const uint64_t keep = l2_policy_evict_last();  // packets: keep in L2 for the scan
#pragma unroll 1
        for (int c0 = 64 * hc; c0 < 64 * hc + 64; c0 += 32) {
          float pw[32];
          tmem_ld32w(tmem_addr(tmem, lq * 32, c0), pw);
          if (lane < 16) {
            const uint8_t* qrow = sm + wy::q0 + (c0 >> 6) * 16384;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const uint4 x = *reinterpret_cast<const uint4*>(qrow + sw128_off(t, ((c0 & 63) >> 3) + c));
              const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
              float y[8];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 f = Cvt<InT>::unpack(xs[e]);
                y[2 * e] = fmaf(eb, f.x, -pw[8 * c + 2 * e]) * P.scale;
                y[2 * e + 1] = fmaf(eb, f.y, -pw[8 * c + 2 * e + 1]) * P.scale;
              }
              const int j = (c0 >> 3) + c;  // 16-byte chunk of the 128 Q' columns
              st_global_hint(pkg + pkt::kQ + (j * 64 + t) * 16, pack8_f16(y), keep);
            }
          }
        }
#pragma unroll 1
        for (int c0 = 64 * hc; c0 < 64 * hc + 64; c0 += 32) {
          float ou[32];
          tmem_ld32w(tmem_addr(tmem, lq * 32, 128 + c0), ou);
          if (lane < 16) {
            uint8_t* dst = pkg + pkt::kOs + (c0 >> 5) * 4096;  // V slice c0 / 32
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              float sc8[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) sc8[e] = ou[8 * c + e] * P.scale;
              st_global_hint(dst + (c * 64 + t) * 16, pack8_f16(sc8), keep);
            }
          }
        }
        if (ptid == 0) *reinterpret_cast<float*>(pkg + pkt::kHdr) = vec[V_EB * kC + kC - 1];
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[wy::B_EPC]);
      }
      // ---- epilogue B: N = -(Kbar^T W) and c = Kbar^T U (row k1 = TMEM lane)
      ok = mbar_wait_warp(&bars[wy::B_NCFULL], ph, abort_flag);
      if (bar_any(1, NP, !ok || *abort_flag)) break;
      {
        tc_fence_after();
        const uint64_t keep = l2_policy_evict_last();
#pragma unroll 1
        for (int c0 = 64 * hc; c0 < 64 * hc + 64; c0 += 32) {
          float n[32];
          tmem_ld32w(tmem_addr(tmem, lq * 32, c0), n);
#pragma unroll
          for (int e = 0; e < 32; ++e) n[e] = -n[e];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int j = (c0 >> 3) + c;  // 16-byte chunk of the 128 N columns
            st_global_hint(pkg + pkt::kN + (j * 128 + r) * 16, pack8_f16(n + 8 * c), keep);
          }
        }
        if (hc == 0) {  // columns 0-63 read: the next item's S product may overwrite them
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars[wy::B_EPB]);
        }
#pragma unroll 1
        for (int c0 = 64 * hc; c0 < 64 * hc + 64; c0 += 32) {
          float cv[32];
          tmem_ld32w(tmem_addr(tmem, lq * 32, 128 + c0), cv);
          uint8_t* dst = pkg + pkt::kCs + (c0 >> 5) * 8192;  // V slice c0 / 32
#pragma unroll
          for (int c = 0; c < 4; ++c) st_global_hint(dst + (c * 128 + r) * 16, pack8_f16(cv + 8 * c), keep);
        }
        tc_fence_before();
      }
    }
  }
  __syncthreads();
  if (warp == wy::kMmaWarp) {
    if (lane == 0 && *abort_flag && P.status != nullptr) atomicOr(P.status, 1 << GDN_ERR_TIMEOUT);
    __syncwarp();
    // every issued MMA completes before TMEM is released (same elected lane as the MMAs)
    mma_commit_warp(&bars[wy::B_DONE]);
    if (lane == 0) {
      volatile int never = 0;
      mbar_wait(&bars[wy::B_DONE], 0, &never);
    }
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// =========================================================== scan kernel
namespace sc {
// warps 0-3: state chain + output rows (TMEM lane quarters), warp 4: ring A loads,
// warp 5: every tcgen05.mma of the CTA, warp 6: ring B loads
constexpr int kThreads = 224;
// ring B is freed only once the output rows of its chunk are out, two chunks
// after the chunk's state update, hence the deeper ring
constexpr int kStagesA = 2, kStagesB = 4;
// ring A slot: N (32 KB), free once N S of its chunk completed
// ring B slot: [Q' 16 KB | hdr] (one bulk copy), this CTA's c and o_intra slices
constexpr uint32_t kSlotA = 32768;
constexpr uint32_t kOffQ = 0, kOffHdr = 16384, kOffC = 17408, kOffO = 25600;
constexpr uint32_t kSlotB = 29696;
constexpr uint32_t ringA = 0;
constexpr uint32_t ringB = kStagesA * kSlotA;
constexpr int kSBufs = 3;                   // S fp16 [k][v] MN-major SW64, 8 KB each
constexpr uint32_t s16 = ringB + kStagesB * kSlotB;
constexpr uint32_t bars = s16 + kSBufs * 8192;
constexpr uint32_t misc = bars + 24 * 8;
constexpr uint32_t total = misc + 32;
constexpr uint32_t alloc = total + 1024;
static_assert(alloc <= 232448, "shared memory budget exceeded");
static_assert(kOffO + 4096 <= kSlotB && kOffHdr + 256 <= kOffC && kSlotB % 1024 == 0, "slot layout");
static_assert(pkt::kQ + 16384 == pkt::kHdr, "Q' and hdr adjacent in the packet");
// TMEM: N S (M=128, 32 cols) and Q' S (M=64) in 3 rotating buffers.  The output
// product of chunk c is issued once S'(c+1) is ready (the last one once S'(c)
// is); the chain warps read chunk c-3 out of the same buffer before that.
constexpr uint32_t kTmN = 0, kTmO = 32;
constexpr int kOBufs = 3;
static_assert(kTmO + kOBufs * 32 <= 128, "TMEM columns");
enum {
  B_FULLA = 0,    // [2] N landed
  B_FULLB = 2,    // [4] Q', hdr, c, o_intra landed
  B_EMPTYA = 6,   // [2] N S of the slot's chunk complete (MMA commit)
  B_EMPTYB = 8,   // [4] output MMA commit + 4 chain warps
  B_DN = 12,      // N S of the current chunk complete (and every earlier product)
  B_DO = 13,      // [3] Q' S of a chunk complete
  B_SREADY = 16,  // S16 of the next chunk written (4 chain warps)
  B_DONE = 17,
  B_COUNT = 18
};
}  // namespace sc

// Chunk c's products are issued in the order N S(c), then Q' S(c-1): the chain
// product never queues behind an output product, and the output product of
// chunk c-1 runs while the chain warps update the state with N S(c).
template <typename OutT>
__global__ void __launch_bounds__(sc::kThreads, 1) gdn_scan_kernel(const __grid_constant__ ScanParams P) {
  constexpr int BV = 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + sc::bars);
  uint32_t* tmem_base_p = reinterpret_cast<uint32_t*>(sm + sc::misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + sc::misc + 4);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int NT = P.NS;
  const int slice = blockIdx.x % P.nslice;
  const int bh = blockIdx.x / P.nslice;
  const int hh = bh % P.H, bb = bh / P.H;
  const int v0 = slice * BV;
  const uint32_t sb = smem_u32(sm);

  if (tid == 0) {
    for (int i = 0; i < sc::B_COUNT; ++i) {
      const bool emptyb = i >= sc::B_EMPTYB && i < sc::B_EMPTYB + sc::kStagesB;
      mbar_init(&bars[i], emptyb ? 5 : (i == sc::B_SREADY ? 4 : 1));
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 4) {
    tmem_alloc(tmem_base_p, 128);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_p;

  if (warp == 4 || warp == 6) {
    // ================================================================ producers (ring A: N, ring B: the rest)
    const bool ra = warp == 4;
    const int fullb = ra ? sc::B_FULLA : sc::B_FULLB;
    const int emptyb = ra ? sc::B_EMPTYA : sc::B_EMPTYB;
    const int nst = ra ? sc::kStagesA : sc::kStagesB;
    int issued = 0;
    for (int i = 0; i < NT; ++i) {
      const int s = i % nst;
      if (i >= nst && !mbar_wait_warp(&bars[emptyb + s], ((i / nst) - 1) & 1, abort_flag)) break;
      if (lane == 0) {
        uint64_t* fb = &bars[fullb + s];
        const uint8_t* pk = P.packets + (size_t(bh) * P.NS + i) * kPacketBytes;
        if (ra) {
          mbar_arrive_expect_tx(fb, 32768);
          bulk_load(sm + sc::ringA + s * sc::kSlotA, pk + pkt::kN, 32768, fb);
          GDN_TR(0, i);
          // ring B is freed a chunk later than ring A: pull its pieces of chunk
          // i + 2 (and the N of chunk i + 3) into L2 now, so its loads hit L2
          if (i + 2 < NT) {
            const uint8_t* pf = pk + 2 * size_t(kPacketBytes);
            bulk_prefetch_l2(pf + pkt::kQ, 16640);
            bulk_prefetch_l2(pf + pkt::kCs + slice * 8192, 8192);
            bulk_prefetch_l2(pf + pkt::kOs + slice * 4096, 4096);
          }
          if (i + 3 < NT) bulk_prefetch_l2(pk + 3 * size_t(kPacketBytes) + pkt::kN, 32768);
        } else {
          uint8_t* st = sm + sc::ringB + s * sc::kSlotB;
          mbar_arrive_expect_tx(fb, 16640 + 8192 + 4096);
          bulk_load(st + sc::kOffQ, pk + pkt::kQ, 16640, fb);
          // this slice's c and o_intra are read by this CTA only: first out of L2
          const uint64_t once = l2_policy_evict_first();
          bulk_load_hint(st + sc::kOffC, pk + pkt::kCs + slice * 8192, 8192, fb, once);
          bulk_load_hint(st + sc::kOffO, pk + pkt::kOs + slice * 4096, 4096, fb, once);
        }
      }
      issued = i + 1;
    }
    if (lane == 0) {
      // let every issued copy land before the CTA exits
      volatile int never = 0;
      for (int i = (issued > nst ? issued - nst : 0); i < issued; ++i)
        mbar_wait(&bars[fullb + i % nst], (i / nst) & 1, &never);
    }
    __syncwarp();
  } else if (warp == 5) {
    // ================================================================ MMA issue (whole warp, elect.sync)
    const uint32_t id_n = idesc_f16(128, BV, 0, 0, 1);
    const uint32_t id_o = idesc_f16(64, BV, 0, 0, 1);
    auto issue_out = [&](int c) -> bool {
      const int s = c % sc::kStagesB;
      if (!mbar_wait_warp(&bars[sc::B_FULLB + s], (c / sc::kStagesB) & 1, abort_flag)) return false;
      tc_fence_after();
      const uint32_t st = sb + sc::ringB + s * sc::kSlotB;
      const uint32_t sbuf = sb + sc::s16 + (c % sc::kSBufs) * 8192;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        mma_f16_ss_warp(tmem + sc::kTmO + (c % sc::kOBufs) * BV, sdesc(st + sc::kOffQ + kk * 2048, 1024, 128, kSwNone),
                        sdesc(sbuf + kk * 1024, 8192, 512, kSw64), id_o, kk > 0);
      mma_commit_warp(&bars[sc::B_DO + c % sc::kOBufs]);
      mma_commit_warp(&bars[sc::B_EMPTYB + s]);
      return true;
    };
    bool okm = true;
    for (int c = 0; c < NT && okm; ++c) {
      const int s = c % sc::kStagesA;
      // descriptors first: after S' is ready only the issue itself remains
      const uint32_t st = sb + sc::ringA + s * sc::kSlotA;
      const uint32_t sbuf = sb + sc::s16 + (c % sc::kSBufs) * 8192;
      uint64_t ad[8], bd[8];
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        ad[kk] = sdesc(st + kk * 4096, 2048, 128, kSwNone);
        bd[kk] = sdesc(sbuf + kk * 1024, 8192, 512, kSw64);
      }
      okm = mbar_wait_warp(&bars[sc::B_FULLA + s], (c / sc::kStagesA) & 1, abort_flag);
      if (lane == 0) GDN_TR(5, c);
      okm = okm && mbar_spin_warp(&bars[sc::B_SREADY], c & 1, abort_flag);
      if (!okm) break;
      tc_fence_after();
      if (lane == 0) GDN_TR(1, c);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) mma_f16_ss_warp(tmem + sc::kTmN, ad[kk], bd[kk], id_n, kk > 0);
      mma_commit_warp(&bars[sc::B_DN]);
      mma_commit_warp(&bars[sc::B_EMPTYA + s]);
      if (lane == 0) GDN_TR(6, c);
      if (c > 0) okm = issue_out(c - 1);
      if (lane == 0) GDN_TR(7, c);
    }
    if (okm && NT > 0) okm = issue_out(NT - 1);
    if (!okm && lane == 0) *abort_flag = 1;
    // issued MMAs complete before TMEM is released (same elected lane as the MMAs)
    mma_commit_warp(&bars[sc::B_DONE]);
    if (lane == 0) {
      volatile int never = 0;
      mbar_wait(&bars[sc::B_DONE], 0, &never);
    }
    __syncwarp();
  } else {
    // ================================================================ chain (thread r = row k of S)
    const int r = tid;
    const size_t hbase = (size_t(bb) * P.H + hh) * kV * kK;
    float S[BV];
    if (P.h0 != nullptr) {
#pragma unroll
      for (int j = 0; j < BV; ++j) S[j] = P.h0[hbase + size_t(v0 + j) * kK + r];
    } else {
#pragma unroll
      for (int j = 0; j < BV; ++j) S[j] = 0.f;
    }
    // output rows of chunk c: o = Q' S + o_intra (gdn_ref.py:86-90); rows t = 16 w + l (l < 16).
    // ov holds Q' S(c), read out of TMEM beforehand.
    auto finish_out = [&](int c, float* ov) {
      const int s = c % sc::kStagesB;
      const int t = 16 * warp + lane;
      const int tg = (P.c0 + c) * kC + t;
      const uint8_t* st = sm + sc::ringB + s * sc::kSlotB;
      if (lane < 16 && tg < P.T) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 x = *reinterpret_cast<const uint4*>(st + sc::kOffO + (q * 64 + t) * 16);
          const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = Cvt<__half>::unpack(xs[e]);
            ov[8 * q + 2 * e] += f.x;
            ov[8 * q + 2 * e + 1] += f.y;
          }
        }
        OutT* dst = reinterpret_cast<OutT*>(P.o) + bb * P.so_b + (long long)tg * P.so_t + hh * P.so_h + v0;
        store_row<OutT>(dst, ov, BV);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[sc::B_EMPTYB + s]);
    };
    auto out_rows = [&](int c) -> bool {
      if (!mbar_wait_warp(&bars[sc::B_DO + c % sc::kOBufs], (c / sc::kOBufs) & 1, abort_flag)) return false;
      tc_fence_after();
      float ov[BV];
      tmem_ld32w(tmem_addr(tmem + sc::kTmO + (c % sc::kOBufs) * BV, warp * 32, 0), ov);
      tc_fence_before();
      finish_out(c, ov);
      return true;
    };
    st_row16<BV>(sm + sc::s16, r, 0, S);
    fence_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(&bars[sc::B_SREADY]);
    bool ok = true;
    for (int i = 0; i < NT; ++i) {
      const int s = i % sc::kStagesB;
      const uint8_t* st = sm + sc::ringB + s * sc::kSlotB;
      ok = mbar_wait_warp(&bars[sc::B_FULLB + s], (i / sc::kStagesB) & 1, abort_flag);
      if (!ok) break;
      float cv[BV];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 x = *reinterpret_cast<const uint4*>(st + sc::kOffC + (q * 128 + r) * 16);
        const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = Cvt<__half>::unpack(xs[e]);
          cv[8 * q + 2 * e] = f.x;
          cv[8 * q + 2 * e + 1] = f.y;
        }
      }
      const float gam = *reinterpret_cast<const float*>(st + sc::kOffHdr);
      ok = mbar_spin_warp(&bars[sc::B_DN], i & 1, abort_flag);
      if (!ok) break;
      tc_fence_after();
      if (r == 0) GDN_TR(2, i);
      // Q' S(i - 2) is read out of TMEM here, with N S(i): it was issued
      // before N S(i) by the same thread, so B_DN covers it too.  The chain
      // warps then read no TMEM while N S(i + 1) runs.
      float d[BV], ov[BV];
      if (i >= 2)
        tmem_ld32x2w(tmem_addr(tmem + sc::kTmN, warp * 32, 0), d,
                     tmem_addr(tmem + sc::kTmO + ((i - 2) % sc::kOBufs) * BV, warp * 32, 0), ov);
      else
        tmem_ld32w(tmem_addr(tmem + sc::kTmN, warp * 32, 0), d);
      tc_fence_before();
      // S' = e^{b_C} S + N S + c   (gdn_ref.py:92-98, regrouped)
#pragma unroll
      for (int j = 0; j < BV; ++j) S[j] = fmaf(gam, S[j], d[j] + cv[j]);
      if (i + 1 < NT) {
        st_row16<BV>(sm + sc::s16 + ((i + 1) % sc::kSBufs) * 8192, r, 0, S);
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[sc::B_SREADY]);
      }
      if (r == 0) GDN_TR(3, i);
      if (i >= 2) finish_out(i - 2, ov);
      if (r == 0) GDN_TR(4, i);
    }
    for (int c = NT >= 2 ? NT - 2 : 0; ok && c < NT; ++c) ok = out_rows(c);
    if (ok && P.ht != nullptr) {
#pragma unroll
      for (int j = 0; j < BV; ++j) P.ht[hbase + size_t(v0 + j) * kK + r] = S[j];
    }
    if (!ok) *abort_flag = 1;
  }
  __syncthreads();
  if (*abort_flag && tid == 0 && P.status != nullptr) atomicOr(P.status, 1 << GDN_ERR_TIMEOUT);
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

// ------------------------------------------------------------------ launchers
template <typename InT, bool kBlocked>
int launch_wy(const WyParams& p, int grid, cudaStream_t s) {
  auto kern = gdn_wy_kernel<InT, kBlocked>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(wy::alloc)) != cudaSuccess)
      return GDN_ERR_CUDA;
    configured[dev] = true;
  }
  kern<<<grid, wy::kThreads, wy::alloc, s>>>(p);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_CUDA;
}

template <typename OutT>
int launch_scan(const ScanParams& p, int grid, cudaStream_t s) {
  auto kern = gdn_scan_kernel<OutT>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sc::alloc)) != cudaSuccess)
      return GDN_ERR_CUDA;
    configured[dev] = true;
  }
  kern<<<grid, sc::kThreads, sc::alloc, s>>>(p);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_CUDA;
}

int run_wy(int in_bf16, const WyParams& p, int num_sms, cudaStream_t s) {
  const long long items = (long long)p.B * p.H * p.NS;
  const int grid = int(items < 2LL * num_sms ? items : 2LL * num_sms);
  if (grid < 1) return GDN_OK;
  if (p.blk_len < p.NS)
    return in_bf16 ? launch_wy<__nv_bfloat16, true>(p, grid, s) : launch_wy<__half, true>(p, grid, s);
  return in_bf16 ? launch_wy<__nv_bfloat16, false>(p, grid, s) : launch_wy<__half, false>(p, grid, s);
}

int run_scan(int out_dtype, const ScanParams& p, int grid, cudaStream_t s) {
  if (out_dtype == GDN_DTYPE_F32) return launch_scan<float>(p, grid, s);
  if (out_dtype == GDN_DTYPE_F16) return launch_scan<__half>(p, grid, s);
  return launch_scan<__nv_bfloat16>(p, grid, s);
}

}  // namespace gdn
