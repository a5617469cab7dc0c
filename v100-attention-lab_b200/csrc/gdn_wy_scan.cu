// Two-kernel chunked GDN forward for B200 (sm_100a):
//
//   gdn_wy_kernel   chunk-parallel WY/UT preparation, one CTA per (b, h, chunk),
//                   two CTAs per SM.  Everything state-independent and
//                   V-independent is done once per chunk here:
//                     S = [K;Q]K^T, A and P (gdn_ref.py:76-80, :87-88),
//                     T = (I+A)^-1 in fp32, W = T diag(beta e^b) K (gdn_ref.py:85),
//                   and written to a 40 KB "packet" in the exact shared-memory
//                   image the scan kernel feeds to its tensor cores:
//                     [W fp16 (2 x 8 KB) | Tb_hi | P fp16 | Tb_lo]  (8 KB each)
//                   with Tb = T diag(beta) split hi + lo in the input dtype.
//   gdn_scan_kernel one CTA per (b, h, 32-wide V slice), serial over chunks:
//                   U = Tb V (gdn_ref.py:84), u = U - W h^T, h = e^{b_C} h +
//                   Kbar^T u, o = Qhat h^T + P u; q and k are scaled and
//                   converted to fp16 in place in the stage buffers.
//
// The packets are scratch memory of 40 KB per (b, h, chunk); long sequences
// are processed in segments of chunks so the scratch stays bounded, the
// state being carried between segments (gdn_ref.py semantics are unchanged).
#include "gdn_common.cuh"
#include "tmap.h"
#include "gdn_wy_scan.h"
#include "../../include/gdn_b200.h"

#include <cuda_runtime.h>

namespace gdn {

constexpr uint32_t kPacketBytes = 40960;
// packet offsets
constexpr uint32_t kPkW0 = 0, kPkW1 = 8192, kPkTbHi = 16384, kPkP = 24576, kPkTbLo = 32768;

// =========================================================== WY/UT prep kernel
namespace wy {
constexpr int kThreads = 160;  // warps 0-3: prep (TMEM lanes 0-127), warp 4: TMA + MMA
constexpr uint32_t kq = 0;          // [k;q] stacked: 2 col-blocks x (64 k rows | 64 q rows) x 128 B
constexpr uint32_t tw = 32768;      // Tw (input dtype), 64 rows x 128 B
constexpr uint32_t pk = 40960;      // packet image, 40 KB
constexpr uint32_t amat = 81920;    // fp32 A / T, 64 x kAStride
constexpr uint32_t vec = amat + kC * kAStride * 4;
constexpr uint32_t bars = vec + kVecN * kC * 4;
constexpr uint32_t misc = bars + 8 * 8;
constexpr uint32_t total = misc + 32;
constexpr uint32_t alloc = total + 1024;
constexpr uint32_t kTmS = 0, kTmW = 64;  // TMEM columns (W is M=64: 128 columns)
enum { B_FULL = 0, B_SFULL, B_TREADY, B_WFULL, B_DONE, B_COUNT };
}  // namespace wy

template <typename InT>
__global__ void __launch_bounds__(wy::kThreads, 2) gdn_wy_kernel(const __grid_constant__ WyParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + wy::bars);
  uint32_t* tmem_base_p = reinterpret_cast<uint32_t*>(sm + wy::misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + wy::misc + 4);
  float* vec = reinterpret_cast<float*>(sm + wy::vec);
  float* amat = reinterpret_cast<float*>(sm + wy::amat);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int il = blockIdx.x % P.NS;      // chunk within the segment
  const int bh = blockIdx.x / P.NS;
  const int hh = bh % P.H, bb = bh / P.H;
  const int chunk = P.c0 + il;
  const int t0 = chunk * kC;

  if (tid == 0) {
    for (int i = 0; i < wy::B_COUNT; ++i) mbar_init(&bars[i], i == wy::B_TREADY ? 4 : 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 4) {
    tmem_alloc(tmem_base_p, 256);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_p;
  const uint32_t sb = smem_u32(sm);

  if (warp == 4) {
    if (lane == 0) {
      mbar_arrive_expect_tx(&bars[wy::B_FULL], 32768);
      tma_load_4d(sm + wy::kq, &P.tm_k, &bars[wy::B_FULL], 0, t0, hh, bb);
      tma_load_4d(sm + wy::kq + 8192, &P.tm_q, &bars[wy::B_FULL], 0, t0, hh, bb);
      tma_load_4d(sm + wy::kq + 16384, &P.tm_k, &bars[wy::B_FULL], 64, t0, hh, bb);
      tma_load_4d(sm + wy::kq + 24576, &P.tm_q, &bars[wy::B_FULL], 64, t0, hh, bb);
    }
    // in-chunk cumsum of g (log2 units) and beta; zero past T (gdn_ref.py:102-114)
    constexpr float kLog2e = 1.4426950408889634f;
    const float* gp = P.g + bb * P.sg_b + hh * P.sg_h;
    const float* bp = P.beta + bb * P.sb_b + hh * P.sb_h;
    const int ta = t0 + lane, tb = t0 + lane + 32;
    float xa = (ta < P.T) ? gp[(long long)ta * P.sg_t] * kLog2e : 0.f;
    float xb = (tb < P.T) ? gp[(long long)tb * P.sg_t] * kLog2e : 0.f;
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
    vec[V_B2 * kC + lane] = xa;
    vec[V_B2 * kC + lane + 32] = xb;
    vec[V_BETA * kC + lane] = (ta < P.T) ? bp[(long long)ta * P.sb_t] : 0.f;
    vec[V_BETA * kC + lane + 32] = (tb < P.T) ? bp[(long long)tb * P.sb_t] : 0.f;
    vec[V_EB * kC + lane] = fast_exp2(xa);
    vec[V_EB * kC + lane + 32] = fast_exp2(xb);
  }
  __syncthreads();  // vec visible

  constexpr uint32_t kInBf16 = Cvt<InT>::kIsBf16;
  bool ok = true;
  if (warp == 4) {
    if (lane == 0) {
      ok = mbar_wait(&bars[wy::B_FULL], 0, abort_flag);
      if (ok) {
        tc_fence_after();
        const uint32_t id_s = idesc_f16(128, 64, kInBf16, 0, 0);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t a = sb + wy::kq + (kk >> 2) * 16384 + (kk & 3) * 32;
          mma_f16_ss(tmem + wy::kTmS, sdesc(a, 16, 1024, kSw128), sdesc(a, 16, 1024, kSw128), id_s, kk > 0);
        }
        mma_commit(&bars[wy::B_SFULL]);
        ok = mbar_wait(&bars[wy::B_TREADY], 0, abort_flag);
      }
      if (ok) {
        tc_fence_after();
        // W = Tw K: M=64 (Tw rows), N=128 (d), K=64 (j); B = k tile read MN-major
        const uint32_t id_w = idesc_f16(64, 128, kInBf16, 0, 1);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f16_ss(tmem + wy::kTmW, sdesc(sb + wy::tw + kk * 32, 16, 1024, kSw128),
                     sdesc(sb + wy::kq + kk * 2048, 16384, 1024, kSw128), id_w, kk > 0);
        mma_commit(&bars[wy::B_WFULL]);
      }
      if (!ok) *abort_flag = 1;
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- prep (warps 0-3)
    const int ptid = tid;  // 0..127 = TMEM lane
    const float b2first = vec[V_B2 * kC], b2last = vec[V_B2 * kC + kC - 1];
    const float ref = 0.5f * (b2first + b2last);
    const bool prod_form = (b2first - b2last) < 200.f;
    if (ptid < 64) amat[ptid * kAStride + 64] = fast_exp2(ref - vec[V_B2 * kC + ptid]);
    named_bar(2, 128);
    ok = mbar_wait_warp(&bars[wy::B_SFULL], 0, abort_flag);
    if (!bar_any(1, 128, !ok || *abort_flag)) {
      tc_fence_after();
      // rows 0-63: A[t][m] = beta_t exp(b_t - b_m) (k_t.k_m), m < t   (TMEM lanes 0-63 = K K^T)
      // rows 64-127: P[t][m] = exp(b_t - b_m) (q_t.k_m), m <= t      (lanes 64-127 = Q K^T)
      const int t = ptid & 63;
      const float b2t = vec[V_B2 * kC + t];
      const float et = fast_exp2(b2t - ref);
      const float bt = (ptid < 64) ? vec[V_BETA * kC + t] : 1.f;
      float* arow = amat + t * kAStride;
      uint8_t* pimg = sm + wy::pk + kPkP;
#pragma unroll 1
      for (int cg = 0; cg < 4; ++cg) {
        float s[16];
        tmem_ld16w(tmem_addr(tmem + wy::kTmS, warp * 32, cg * 16), s);
        float x[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int m = cg * 16 + e;
          const float dec = prod_form ? et * amat[m * kAStride + 64] : fast_exp2(b2t - vec[V_B2 * kC + m]);
          const bool keep = (ptid < 64) ? (m < t) : (m <= t);
          x[e] = keep ? bt * dec * s[e] : 0.f;
        }
        if (ptid < 64) {
#pragma unroll
          for (int e = 0; e < 16; e += 4)
            *reinterpret_cast<float4*>(arow + cg * 16 + e) = make_float4(x[e], x[e + 1], x[e + 2], x[e + 3]);
        } else {
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            uint4 w;
            w.x = Cvt<__half>::pack(x[8 * h2 + 0], x[8 * h2 + 1]);
            w.y = Cvt<__half>::pack(x[8 * h2 + 2], x[8 * h2 + 3]);
            w.z = Cvt<__half>::pack(x[8 * h2 + 4], x[8 * h2 + 5]);
            w.w = Cvt<__half>::pack(x[8 * h2 + 6], x[8 * h2 + 7]);
            *reinterpret_cast<uint4*>(pimg + sw128_off(t, 2 * cg + h2)) = w;
          }
        }
      }
      tc_fence_before();
      named_bar(1, 128);
      invert_unit_lower64(amat, ptid);  // T = (I + A)^-1 in place
      // Tw = T diag(beta e^b) -> tw (MMA operand); Tb = T diag(beta) -> packet hi + lo
      {
        const int r = ptid >> 1, half = ptid & 1;
        const float* trow = amat + r * kAStride;
        uint8_t* twp = sm + wy::tw;
        uint8_t* hip = sm + wy::pk + kPkTbHi;
        uint8_t* lop = sm + wy::pk + kPkTbLo;
#pragma unroll 1
        for (int c = 4 * half; c < 4 * half + 4; ++c) {
          uint32_t ww[4], hi[4], lo[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int m = 8 * c + 2 * e;
            const float tb0 = trow[m] * vec[V_BETA * kC + m], tb1 = trow[m + 1] * vec[V_BETA * kC + m + 1];
            ww[e] = Cvt<InT>::pack(tb0 * vec[V_EB * kC + m], tb1 * vec[V_EB * kC + m + 1]);
            hi[e] = Cvt<InT>::pack(tb0, tb1);
            const float2 hf = Cvt<InT>::unpack(hi[e]);
            lo[e] = Cvt<InT>::pack(tb0 - hf.x, tb1 - hf.y);
          }
          *reinterpret_cast<uint4*>(twp + sw128_off(r, c)) = make_uint4(ww[0], ww[1], ww[2], ww[3]);
          *reinterpret_cast<uint4*>(hip + sw128_off(r, c)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
          *reinterpret_cast<uint4*>(lop + sw128_off(r, c)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[wy::B_TREADY]);
      // W (M=64 layout: row 16w + l in TMEM lane 32w + l, l < 16) -> fp16 packet image
      ok = mbar_wait_warp(&bars[wy::B_WFULL], 0, abort_flag);
      if (ok) {
        tc_fence_after();
        const int r = 16 * warp + (lane & 15);
#pragma unroll 1
        for (int c0 = 0; c0 < 128; c0 += 32) {
          float w[32];
          tmem_ld32w(tmem_addr(tmem + wy::kTmW, warp * 32, c0), w);
          if (lane < 16) {
            uint8_t* wimg = sm + wy::pk + (c0 >= 64 ? kPkW1 : kPkW0);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              uint4 y;
              y.x = Cvt<__half>::pack(w[8 * c + 0], w[8 * c + 1]);
              y.y = Cvt<__half>::pack(w[8 * c + 2], w[8 * c + 3]);
              y.z = Cvt<__half>::pack(w[8 * c + 4], w[8 * c + 5]);
              y.w = Cvt<__half>::pack(w[8 * c + 6], w[8 * c + 7]);
              *reinterpret_cast<uint4*>(wimg + sw128_off(r, ((c0 & 63) >> 3) + c)) = y;
            }
          }
        }
        tc_fence_before();
        fence_async_smem();
      }
    } else {
      ok = false;
    }
    if (!ok) *abort_flag = 1;
  }
  __syncthreads();
  if (tid == 128) {
    if (!*abort_flag) {
      // the whole packet image -> global in one bulk copy
      uint8_t* dst = P.packets + (size_t(bh) * P.NS + il) * kPacketBytes;
      asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
                   "r"(sb + wy::pk), "r"(kPacketBytes)
                   : "memory");
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    } else {
      // a failed wait: let the TMA load land before the CTA releases its smem
      volatile int never = 0;
      mbar_wait(&bars[wy::B_FULL], 0, &never);
      if (P.status != nullptr) atomicOr(P.status, 1 << GDN_ERR_TIMEOUT);
    }
    // every issued MMA completes before TMEM is released
    mma_commit(&bars[wy::B_DONE]);
    volatile int never = 0;
    mbar_wait(&bars[wy::B_DONE], 0, &never);
  }
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// =========================================================== scan kernel
namespace sc {
constexpr int kThreads = 384;
// stage layout (76 KB): per column block cb: [W16 | q->Qhat | k->Kbar] x 8 KB,
// then the v slice, then [Tb_hi | P | Tb_lo]
constexpr uint32_t kStage = 77824;             // 76 KB
constexpr uint32_t kCb = 24576;                // column-block stride
constexpr uint32_t kOffQ = 8192, kOffK = 16384;
constexpr uint32_t kOffV = 49152;              // v slice (4 KB for BV=32)
constexpr uint32_t kOffTp = 53248;             // [Tb_hi | P | Tb_lo], 24 KB
constexpr uint32_t st0 = 0, st1 = kStage;
constexpr uint32_t ht16 = 2 * kStage;          // 155648: h^T fp16, 128 rows x 64 B
constexpr uint32_t u16 = ht16 + 8192;          // u fp16, 64 rows x 64 B
constexpr uint32_t vec = u16 + 4096;           // 4 chunks x kVecN x 64 fp32
constexpr uint32_t bars = vec + 4 * kVecN * kC * 4;
constexpr uint32_t misc = bars + 32 * 8;
constexpr uint32_t total = misc + 32;
constexpr uint32_t alloc = total + 1024;
static_assert(alloc <= 232448, "shared memory budget exceeded");
// TMEM columns (BV = 32)
constexpr uint32_t kTmU0 = 0, kTmU1 = 32, kTmD1 = 64, kTmD2 = 96, kTmD3 = 128;
enum {
  B_FULL = 0,   // [2]
  B_EMPTY = 2,  // [2]
  B_VEC = 4,    // [4]
  B_CVT = 8,    // [2]
  B_UFULL = 10, // [2]
  B_UFREE = 12, // [2]
  B_D1 = 14,
  B_D2 = 15,
  B_DONE = 16,   // U issuer drain
  B_DONE2 = 17,  // chain issuer drain
  B_COUNT = 18
};
}  // namespace sc

template <typename InT, typename OutT>
__global__ void __launch_bounds__(sc::kThreads, 1) gdn_scan_kernel(const __grid_constant__ ScanParams P) {
  constexpr int BV = 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + sc::bars);
  uint32_t* tmem_base_p = reinterpret_cast<uint32_t*>(sm + sc::misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + sc::misc + 4);
  float* vecs = reinterpret_cast<float*>(sm + sc::vec);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int NT = P.NS;
  const int slice = blockIdx.x % P.nslice;
  const int bh = blockIdx.x / P.nslice;
  const int hh = bh % P.H, bb = bh / P.H;
  const int v0 = slice * BV;
  const uint32_t sb = smem_u32(sm);

  if (tid == 0) {
    const uint32_t counts[sc::B_COUNT] = {1, 1, 2, 2, 32, 32, 32, 32, 4, 4, 1, 1, 2, 2, 1, 1, 1, 1};
    for (int i = 0; i < sc::B_COUNT; ++i) mbar_init(&bars[i], counts[i]);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&P.tm_q);
    prefetch_tmap(&P.tm_k);
    prefetch_tmap(&P.tm_v);
  }
  if (warp == 1) {
    tmem_alloc(tmem_base_p, 256);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_p;
  auto stage = [&](int i) -> uint32_t { return (i & 1) ? sc::st1 : sc::st0; };

  if (warp == 0) {
    // ================================================================ producer
    constexpr float kLog2e = 1.4426950408889634f;
    const float* gp = P.g + bb * P.sg_b + hh * P.sg_h;
    int issued = 0;
    for (int i = 0; i < NT; ++i) {
      const int s = i & 1;
      if (i >= 2 && !mbar_wait_warp(&bars[sc::B_EMPTY + s], ((i >> 1) - 1) & 1, abort_flag)) break;
      const int t0 = (P.c0 + i) * kC;
      if (lane == 0) {
        uint8_t* st = sm + stage(i);
        uint64_t* fb = &bars[sc::B_FULL + s];
        mbar_arrive_expect_tx(fb, 32768 + 4096 + kPacketBytes);
        tma_load_4d(st + sc::kOffQ, &P.tm_q, fb, 0, t0, hh, bb);
        tma_load_4d(st + sc::kOffK, &P.tm_k, fb, 0, t0, hh, bb);
        tma_load_4d(st + sc::kCb + sc::kOffQ, &P.tm_q, fb, 64, t0, hh, bb);
        tma_load_4d(st + sc::kCb + sc::kOffK, &P.tm_k, fb, 64, t0, hh, bb);
        tma_load_4d(st + sc::kOffV, &P.tm_v, fb, v0, t0, hh, bb);
        const uint8_t* pk = P.packets + (size_t(bh) * P.NS + i) * kPacketBytes;
        const uint32_t fbs = smem_u32(fb);
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                smem_u32(st)),
            "l"(pk + kPkW0), "r"(8192u), "r"(fbs)
            : "memory");
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                smem_u32(st + sc::kCb)),
            "l"(pk + kPkW1), "r"(8192u), "r"(fbs)
            : "memory");
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                smem_u32(st + sc::kOffTp)),
            "l"(pk + kPkTbHi), "r"(24576u), "r"(fbs)
            : "memory");
      }
      issued = i + 1;
      const int ta = t0 + lane, tb = t0 + lane + 32;
      float xa = (ta < P.T) ? gp[(long long)ta * P.sg_t] * kLog2e : 0.f;
      float xb = (tb < P.T) ? gp[(long long)tb * P.sg_t] * kLog2e : 0.f;
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
      // vec[i & 3] is free: chunk i-4's readers finished before EMPTY(i-2) completed
      float* vec = vecs + (i & 3) * kVecN * kC;
      vec[V_B2 * kC + lane] = xa;
      vec[V_B2 * kC + lane + 32] = xb;
      vec[V_EB * kC + lane] = fast_exp2(xa);
      vec[V_EB * kC + lane + 32] = fast_exp2(xb);
      vec[V_DD * kC + lane] = fast_exp2(bC - xa);
      vec[V_DD * kC + lane + 32] = fast_exp2(bC - xb);
      mbar_arrive(&bars[sc::B_VEC + (i & 3)]);
    }
    if (lane == 0) {
      volatile int never = 0;
      for (int i = (issued > 2 ? issued - 2 : 0); i < issued; ++i)
        mbar_wait(&bars[sc::B_FULL + (i & 1)], (i >> 1) & 1, &never);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ================================================================ U = Tb V
    if (lane == 0) {
      constexpr uint32_t kInBf16 = Cvt<InT>::kIsBf16;
      const uint32_t id_u = idesc_f16(128, BV, kInBf16, 0, 1);
      bool okm = true;
      for (int i = 0; i < NT && okm; ++i) {
        const int s = i & 1;
        okm = mbar_wait(&bars[sc::B_FULL + s], (i >> 1) & 1, abort_flag) &&
              (i < 2 || mbar_wait(&bars[sc::B_UFREE + s], ((i >> 1) - 1) & 1, abort_flag));
        if (!okm) break;
        tc_fence_after();
        const uint32_t tp = sb + stage(i) + sc::kOffTp;
        const uint32_t vt = sb + stage(i) + sc::kOffV;
        // rows 0-63 of A: Tb_hi (k-steps 0-3), Tb_lo (k-steps 4-7); U lands in lanes 0-63
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_f16_ss(tmem + (s ? sc::kTmU1 : sc::kTmU0),
                     sdesc(tp + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024, kSw128),
                     sdesc(vt + (kk & 3) * 1024, 8192, 512, kSw64), id_u, kk > 0);
        mma_commit(&bars[sc::B_UFULL + s]);
        mma_commit(&bars[sc::B_EMPTY + s]);
      }
      if (!okm) *abort_flag = 1;
      mma_commit(&bars[sc::B_DONE]);
      volatile int never = 0;
      mbar_wait(&bars[sc::B_DONE], 0, &never);
    }
    __syncwarp();
  } else if (warp >= 4 && warp < 8) {
    // ================================================================ convert in place
    // thread: row r of q (half 0) or of k (half 1); Qhat = e^{b_t} q_t, Kbar = e^{b_C - b_t} k_t (fp16)
    const int ct = tid - 128, r = ct & 63, isk = ct >> 6;
    for (int i = 0; i < NT; ++i) {
      const int s = i & 1;
      if (!mbar_wait_warp(&bars[sc::B_FULL + s], (i >> 1) & 1, abort_flag)) break;
      if (!mbar_wait_warp(&bars[sc::B_VEC + (i & 3)], (i >> 2) & 1, abort_flag)) break;
      const float* vec = vecs + (i & 3) * kVecN * kC;
      const float sc_ = isk ? vec[V_DD * kC + r] : vec[V_EB * kC + r];
      uint8_t* base = sm + stage(i) + (isk ? sc::kOffK : sc::kOffQ);
#pragma unroll 1
      for (int cc = 0; cc < 16; ++cc) {
        uint8_t* p = base + (cc >> 3) * sc::kCb + sw128_off(r, cc & 7);
        const uint4 x = *reinterpret_cast<const uint4*>(p);
        const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
        uint32_t ys[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = Cvt<InT>::unpack(xs[e]);
          ys[e] = Cvt<__half>::pack(f.x * sc_, f.y * sc_);
        }
        *reinterpret_cast<uint4*>(p) = make_uint4(ys[0], ys[1], ys[2], ys[3]);
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[sc::B_CVT + s]);
    }
  } else if (warp >= 8) {
    // ================================================================ chain
    // Thread r owns row d = r of h^T in fp32 registers (TMEM lane r).
    //   D1 = [W; Qhat] h^T   lanes 0-63: W h^T, lanes 64-127: Qhat h^T   (issued by r = 0)
    //   u  = U - W h^T       (U in lanes 0-63)
    //   D2 = Kbar^T u, D3 = [* ; P] u  (P u in lanes 64-127)            (issued by r = 0)
    //   h  = e^{b_C} h + D2,  o = Qhat h^T + P u
    const int r = tid - 256;
    const int wq = warp - 8;
    const uint32_t id_1 = idesc_f16(128, BV, 0, 0, 1);
    const uint32_t id_2 = idesc_f16(128, BV, 0, 1, 1);
    float h[BV];
    const size_t hbase = (size_t(bb) * P.H + hh) * kV * kK;
    if (P.h0 != nullptr) {
#pragma unroll
      for (int j = 0; j < BV; ++j) h[j] = P.h0[hbase + size_t(v0 + j) * kK + r];
    } else {
#pragma unroll
      for (int j = 0; j < BV; ++j) h[j] = 0.f;
    }
    bool ok = true;
    auto issue_d1 = [&](int c) -> bool {
      const int s = c & 1;
      if (!mbar_wait(&bars[sc::B_FULL + s], (c >> 1) & 1, abort_flag)) return false;
      if (!mbar_wait(&bars[sc::B_CVT + s], (c >> 1) & 1, abort_flag)) return false;
      tc_fence_after();
      const uint32_t st = sb + stage(c);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        mma_f16_ss(tmem + sc::kTmD1, sdesc(st + (kk >> 2) * sc::kCb + (kk & 3) * 32, 16, 1024, kSw128),
                   sdesc(sb + sc::ht16 + kk * 1024, 8192, 512, kSw64), id_1, kk > 0);
      mma_commit(&bars[sc::B_D1]);
      return true;
    };
    st_row16<BV>(sm + sc::ht16, r, 0, h);
    fence_async_smem();
    if (!bar_any(3, 128, false) && r == 0 && NT > 0) {
      if (!issue_d1(0)) *abort_flag = 1;
    }
    for (int i = 0; i < NT; ++i) {
      const int s = i & 1;
      ok = mbar_wait_warp(&bars[sc::B_D1], i & 1, abort_flag);
      if (ok) tc_fence_after();
      float y[BV];
      if (r < 64) {
        ok = ok && mbar_wait_warp(&bars[sc::B_UFULL + s], (i >> 1) & 1, abort_flag);
        if (ok) {
          tc_fence_after();
          float x[BV], uu[BV];
          tmem_ld32w(tmem_addr(tmem + sc::kTmD1, wq * 32, 0), x);
          tmem_ld32w(tmem_addr(tmem + (s ? sc::kTmU1 : sc::kTmU0), wq * 32, 0), uu);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars[sc::B_UFREE + s]);
#pragma unroll
          for (int j = 0; j < BV; ++j) uu[j] -= x[j];  // u = U - W h^T   (gdn_ref.py:86)
          st_row16<BV>(sm + sc::u16, r, 0, uu);
          fence_async_smem();
        }
        if (!bar_any(4, 64, !ok) && r == 0) {
          tc_fence_after();
          const uint32_t st = sb + stage(i);
          const uint32_t tp = st + sc::kOffTp;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_f16_ss(tmem + sc::kTmD2, sdesc(st + sc::kOffK + kk * 2048, sc::kCb, 1024, kSw128),
                       sdesc(sb + sc::u16 + kk * 1024, 8192, 512, kSw64), id_2, kk > 0);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_f16_ss(tmem + sc::kTmD3, sdesc(tp + kk * 32, 16, 1024, kSw128),
                       sdesc(sb + sc::u16 + kk * 1024, 8192, 512, kSw64), id_1, kk > 0);
          mma_commit(&bars[sc::B_D2]);
          mma_commit(&bars[sc::B_EMPTY + s]);
        }
      } else if (ok) {
        tmem_ld32w(tmem_addr(tmem + sc::kTmD1, wq * 32, 0), y);
      }
      ok = ok && mbar_wait_warp(&bars[sc::B_D2], i & 1, abort_flag) &&
           mbar_wait_warp(&bars[sc::B_VEC + (i & 3)], (i >> 2) & 1, abort_flag);
      if (ok) {
        tc_fence_after();
        float dh[BV];
        tmem_ld32w(tmem_addr(tmem + sc::kTmD2, wq * 32, 0), dh);
        const float gam = vecs[(i & 3) * kVecN * kC + V_EB * kC + kC - 1];  // e^{b_C}
#pragma unroll
        for (int j = 0; j < BV; ++j) h[j] = fmaf(gam, h[j], dh[j]);  // h' = e^{b_C} h + Kbar^T u
        if (i + 1 < NT) st_row16<BV>(sm + sc::ht16, r, 0, h);
        float z[BV];
        tmem_ld32w(tmem_addr(tmem + sc::kTmD3, wq * 32, 0), z);
        const int t = (P.c0 + i) * kC + (r - 64);
        if (r >= 64 && t < P.T) {
#pragma unroll
          for (int j = 0; j < BV; ++j) z[j] += y[j];  // o = Qhat h^T + P u   (gdn_ref.py:89-90)
          OutT* dst = reinterpret_cast<OutT*>(P.o) + bb * P.so_b + (long long)t * P.so_t + hh * P.so_h + v0;
          store_row<OutT>(dst, z, BV);
        }
        tc_fence_before();
        fence_async_smem();
      }
      if (bar_any(3, 128, !ok || *abort_flag)) {
        ok = false;
        break;
      }
      if (r == 0 && i + 1 < NT && !issue_d1(i + 1)) *abort_flag = 1;
    }
    if (ok && P.ht != nullptr) {
#pragma unroll
      for (int j = 0; j < BV; ++j) P.ht[hbase + size_t(v0 + j) * kK + r] = h[j];
    }
    if (!ok) *abort_flag = 1;
    if (r == 0) {
      // chain MMAs complete before TMEM is released
      mma_commit(&bars[sc::B_DONE2]);
      volatile int never = 0;
      mbar_wait(&bars[sc::B_DONE2], 0, &never);
    }
  }
  __syncthreads();
  if (*abort_flag && tid == 0 && P.status != nullptr) atomicOr(P.status, 1 << GDN_ERR_TIMEOUT);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// ------------------------------------------------------------------ launchers
template <typename InT>
int launch_wy(const WyParams& p, int grid, cudaStream_t s) {
  auto kern = gdn_wy_kernel<InT>;
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

template <typename InT, typename OutT>
int launch_scan(const ScanParams& p, int grid, cudaStream_t s) {
  auto kern = gdn_scan_kernel<InT, OutT>;
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

int run_wy(int in_bf16, const WyParams& p, int grid, cudaStream_t s) {
  return in_bf16 ? launch_wy<__nv_bfloat16>(p, grid, s) : launch_wy<__half>(p, grid, s);
}

int run_scan(int in_bf16, int out_dtype, const ScanParams& p, int grid, cudaStream_t s) {
  if (in_bf16) {
    if (out_dtype == GDN_DTYPE_F32) return launch_scan<__nv_bfloat16, float>(p, grid, s);
    if (out_dtype == GDN_DTYPE_F16) return launch_scan<__nv_bfloat16, __half>(p, grid, s);
    return launch_scan<__nv_bfloat16, __nv_bfloat16>(p, grid, s);
  }
  if (out_dtype == GDN_DTYPE_F32) return launch_scan<__half, float>(p, grid, s);
  if (out_dtype == GDN_DTYPE_F16) return launch_scan<__half, __half>(p, grid, s);
  return launch_scan<__half, __nv_bfloat16>(p, grid, s);
}

}  // namespace gdn
