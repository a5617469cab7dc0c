// Fused chunked Gated DeltaNet forward for B200 (sm_100a).
//
// One CTA owns one (batch, head, V-slice) and walks the sequence chunk by
// chunk, like the reference's program map (gdn_triton.py:42-54), but every
// contraction runs on tcgen05 tensor cores with fp32 TMEM accumulators, all
// operand tiles arrive by TMA, and the chunk-local preparation of chunk i+1
// overlaps the serial state update of chunk i through warp specialisation:
//
//   warp 0      TMA producer: q/k/v tiles, beta/g, in-chunk cumsum of g
//   warp 1      MMA issuer (one thread, non-blocking event loop)
//   warps 2-3   convert: Qhat = exp(b) q and Kbar = exp(b_C - b) k to fp16
//   warps 4-7   prep: A and P from S = [K;Q] K^T, T = (I+A)^-1 in fp32,
//               the split operands of W = T diag(beta e^b) K and
//               U = T diag(beta) V, and W to fp16
//   warps 8-11  chain: u = U - W h^T, h = e^{b_C} h + Kbar^T u (fp32 state in
//               registers), o = Qhat h^T + P u
//
// Per chunk (C = 64, K = V = 128, slice width BV) the tensor-core work is
//   S   = [K; Q] K^T              M=128 N=64  K=128   (gdn_ref.py:77, :87)
//   W   = Tw K                    M=128 N=128 K=64    (gdn_ref.py:85)
//   U   = (Tb_hi + Tb_lo) V       M=128 N=BV  K=128   (gdn_ref.py:84)
//   D1  = [Qhat; W] h^T           M=128 N=BV  K=128   (gdn_ref.py:86, :90)
//   D2  = Kbar^T u                M=128 N=BV  K=64    (gdn_ref.py:92-98, folded)
//   D3  = P u                     M=128 N=BV  K=64    (gdn_ref.py:87-89)
// The state update uses the identity h' = e^{b_C} h + (e^{b_C-b} u)^T K, which
// is the reference's h (e^{b_C} I - Wbar^T K) + Ubar^T K with the h Wbar^T K
// term folded into u; it needs one GEMM per chunk instead of two.
//
// Precision: S, W and U take the input dtype (fp16 or bf16) as operands
// (products of input values are exact in fp32); U uses a hi+lo split of
// T diag(beta) so it carries ~16 significant bits.  The state-side GEMMs
// (D1, D2, D3) take fp16 operands with fp32 accumulation, the same choice the
// reference makes for its state casts (gdn_triton.py:87, :93-94, :101-106).
// The state itself stays fp32 for the whole sequence.
#include "gdn_common.cuh"
#include "tmap.h"
#include "gdn_wy_scan.h"
#include "../../include/gdn_b200.h"

#include <cuda_runtime.h>
#include <cstdio>
#include <cstring>

namespace gdn {

constexpr int kThreads = 384;

// ------------------------------------------------------------------ layout
template <int BV>
struct Layout {
  // 1024-aligned swizzled tiles
  static constexpr uint32_t kq0 = 0;            // [k;q] stage 0: 2 col-blocks x (64 k rows | 64 q rows) x 128 B
  static constexpr uint32_t kq1 = 32768;        // stage 1
  static constexpr uint32_t ahat0 = 65536;      // [Qhat; W16] buffer 0 (2 col-blocks x 128 rows x 128 B)
  static constexpr uint32_t ahat1 = 98304;
  static constexpr uint32_t tstk = 131072;      // [Tw | Tb_hi] (cb0), [P1 | Tb_lo] (cb1)
  static constexpr uint32_t p1 = tstk + 16384;  // P buffer 1 lives in the unused rows of Tstack cb1
  static constexpr uint32_t p0 = 163840;        // P buffer 0 (its M=128 tail rows read Kbar: ignored lanes)
  static constexpr uint32_t kbar = 172032;      // Kbar: 2 d-blocks x 64 rows x 128 B
  static constexpr uint32_t vt0 = 188416;       // v slice stage 0: 64 rows x BV*2 B
  static constexpr uint32_t vt_bytes = kC * BV * 2;
  static constexpr uint32_t vt1 = vt0 + ((vt_bytes + 1023) / 1024) * 1024;
  static constexpr uint32_t ht16 = vt1 + ((vt_bytes + 1023) / 1024) * 1024;  // h^T fp16: 128 rows x BV*2 B
  static constexpr uint32_t u16 = ht16 + ((kK * BV * 2 + 1023) / 1024) * 1024;  // u fp16: 64 rows x BV*2 B
  static constexpr uint32_t amat = u16 + ((kC * BV * 2 + 1023) / 1024) * 1024;  // fp32 A / T
  static constexpr uint32_t vec = amat + kC * kAStride * 4;  // 4 chunks x {b2, beta, e^b, e^(b_C-b)} x 64
  static constexpr uint32_t bars = vec + 4 * kVecN * kC * 4;
  static constexpr uint32_t nbars = 40;
  static constexpr uint32_t misc = bars + nbars * 8;
  static constexpr uint32_t total = misc + 64;
  static constexpr uint32_t alloc = total + 1024;  // slack for 1024-B alignment of the base
  static_assert(alloc <= 232448, "shared memory budget exceeded");
  // swizzle of the BV-wide MN-major tiles (v, h^T, u)
  static constexpr uint32_t bv_swz = (BV == 32) ? kSw64 : kSw128;
  static constexpr uint32_t bv_sbo = (BV == 32) ? 512 : 1024;  // 8 rows x row bytes
};

// TMEM columns
constexpr uint32_t kTmS = 0;      // 64 cols
constexpr uint32_t kTmW = 64;     // 128 cols
constexpr uint32_t kTmU0 = 192;   // 2 x BV cols
template <int BV>
struct TmemCols {
  static constexpr uint32_t u0 = kTmU0, u1 = kTmU0 + BV;
  static constexpr uint32_t d1 = kTmU0 + 2 * BV, d2 = d1 + BV, d3 = d2 + BV;
  static constexpr uint32_t total = d3 + BV;
  static constexpr uint32_t alloc = total <= 256 ? 256 : 512;
};

// barrier indices
enum Bar : int {
  B_FULL = 0,        // [2]
  B_EMPTY = 2,       // [2]
  B_VEC = 4,         // [4]
  B_SFULL = 8,
  B_SFREE = 9,
  B_TREADY = 10,
  B_TFREE = 11,
  B_PFREE = 12,      // [2]
  B_WFULL = 14,
  B_WFREE = 15,
  B_UFULL = 16,      // [2]
  B_UFREE = 18,      // [2]
  B_AFULL = 20,      // [2]
  B_AFREE = 22,      // [2]
  B_KFULL = 24,
  B_KFREE = 25,
  B_HFULL = 26,
  B_D1 = 27,
  B_U16 = 28,
  B_D2 = 29,
  B_DONE = 30,
  B_COUNT = 31
};

struct FwdParams {
  CUtensorMap tm_q, tm_k, tm_v;
  const float* beta;
  const float* g;
  const float* h0;
  float* ht;
  void* o;
  float* w_out;  // prep-only mode
  float* u_out;
  int* status;
  long long* trace;  // per-chunk role timestamps of CTA 0 (GDN_TRACE builds only)
  long long sb_b, sb_t, sb_h;
  long long sg_b, sg_t, sg_h;
  long long so_b, so_t, so_h;
  int B, T, H, NT, nslice;
  float scale;  // multiplies o (q scaled)
  int flags;    // GDN_FLAG_BETA_SIGMOID / GDN_FLAG_G_LOGSIGMOID
};

// ------------------------------------------------------------------ kernel
// Abort protocol: every wait is bounded (tc.cuh).  A role that gives up sets
// the CTA abort flag and leaves its loop; the others see the flag within a
// few polls.  Roles that use CTA-wide or warp-collective instructions make
// the decision uniform first (warp votes, bar.red.or in the prep group), so
// no thread is ever left at a barrier its peers skipped.
template <int BV, typename InT, typename OutT, bool kPrepOnly>
__global__ void __launch_bounds__(kThreads, 1) gdn_fwd_kernel(const __grid_constant__ FwdParams P) {
  using L = Layout<BV>;
  using TC = TmemCols<BV>;
  static_assert(BV == 32, "this build implements 32-column V slices");
  extern __shared__ uint8_t smem_raw[];
  // 1024-B aligned base for the swizzled tiles.  Offsetting the __shared__
  // array itself (not an integer round trip) keeps the shared address space
  // visible to the compiler, so every access below is an LDS/STS.
  uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::bars);
  uint32_t* tmem_base_p = reinterpret_cast<uint32_t*>(sm + L::misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + L::misc + 4);
  float* vecs = reinterpret_cast<float*>(sm + L::vec);  // [4][kVecN][64]
  float* amat = reinterpret_cast<float*>(sm + L::amat);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int NT = P.NT;
  const int slice = blockIdx.x % P.nslice;
  const int bh = blockIdx.x / P.nslice;
  const int hh = bh % P.H, bb = bh / P.H;
  const int v0 = slice * BV;

  if (tid == 0) {
    const uint32_t counts[B_COUNT] = {1, 1, 3, 3, 32, 32, 32, 32, 1, 4, 4, 1, 1, 1, 1, 2,
                                      1, 1, 2, 2, 6, 6, 1, 1, 2, 1, 4, 1, 2, 1, 1};
    for (int i = 0; i < B_COUNT; ++i) mbar_init(&bars[i], counts[i]);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&P.tm_q);
    prefetch_tmap(&P.tm_k);
    prefetch_tmap(&P.tm_v);
  }
  if (warp == 1) {
    tmem_alloc(tmem_base_p, TC::alloc);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_p;

  if (warp == 0) {
    // ================================================================ producer
    constexpr float kLog2e = 1.4426950408889634f;
    const float* gp = P.g == nullptr ? nullptr : P.g + bb * P.sg_b + hh * P.sg_h;
    const float* bp = P.beta + bb * P.sb_b + hh * P.sb_h;
    int issued = 0;
    for (int i = 0; i < NT; ++i) {
      const int s = i & 1;
      if (i >= 2 && !mbar_wait_warp(&bars[B_EMPTY + s], ((i >> 1) - 1) & 1, abort_flag)) break;
      const int t0 = i * kC;
      if (lane == 0) {
        uint8_t* kq = sm + (s ? L::kq1 : L::kq0);
        uint8_t* vt = sm + (s ? L::vt1 : L::vt0);
        mbar_arrive_expect_tx(&bars[B_FULL + s], 32768 + L::vt_bytes);
        tma_load_4d(kq, &P.tm_k, &bars[B_FULL + s], 0, t0, hh, bb);
        tma_load_4d(kq + 8192, &P.tm_q, &bars[B_FULL + s], 0, t0, hh, bb);
        tma_load_4d(kq + 16384, &P.tm_k, &bars[B_FULL + s], 64, t0, hh, bb);
        tma_load_4d(kq + 24576, &P.tm_q, &bars[B_FULL + s], 64, t0, hh, bb);
        tma_load_4d(vt, &P.tm_v, &bars[B_FULL + s], v0, t0, hh, bb);
        GDN_TR(0, i);
      }
      issued = i + 1;
      // beta and the in-chunk cumsum of g (log2 units); zero past T, which is
      // the padding rule of gdn_ref.py:102-114 (beta = g = 0).
      const int ta = t0 + lane, tb = t0 + lane + 32;
      float xa = load_g(gp, (long long)ta * P.sg_t, ta < P.T, P.flags) * kLog2e;
      float xb = load_g(gp, (long long)tb * P.sg_t, tb < P.T, P.flags) * kLog2e;
      const float ba = load_beta(bp, (long long)ta * P.sb_t, ta < P.T, P.flags);
      const float bbv = load_beta(bp, (long long)tb * P.sb_t, tb < P.T, P.flags);
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
      // vec[i & 3] is free: chunk i-4's readers finished before EMPTY(i-2) completed
      const float bC = __shfl_sync(0xffffffffu, xb, 31);
      float* vec = vecs + (i & 3) * kVecN * kC;
      vec[V_B2 * kC + lane] = xa;
      vec[V_B2 * kC + lane + 32] = xb;
      vec[V_BETA * kC + lane] = ba;
      vec[V_BETA * kC + lane + 32] = bbv;
      vec[V_EB * kC + lane] = fast_exp2(xa);
      vec[V_EB * kC + lane + 32] = fast_exp2(xb);
      vec[V_DD * kC + lane] = fast_exp2(bC - xa);
      vec[V_DD * kC + lane + 32] = fast_exp2(bC - xb);
      mbar_arrive(&bars[B_VEC + (i & 3)]);
    }
    // every issued TMA load must land before the CTA exits
    if (lane == 0) {
      volatile int never = 0;
      for (int i = (issued > 2 ? issued - 2 : 0); i < issued; ++i)
        mbar_wait(&bars[B_FULL + (i & 1)], (i >> 1) & 1, &never);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ================================================================ MMA issuer (prep GEMMs)
    // The chain GEMMs (D1, D2, D3) are issued by the chain warps themselves so the
    // serial path never waits for this thread's polling loop.
    if (lane == 0) {
      constexpr uint32_t kInBf16 = Cvt<InT>::kIsBf16;
      const uint32_t id_s = idesc_f16(128, 64, kInBf16, 0, 0);
      const uint32_t id_w = idesc_f16(128, 128, kInBf16, 0, 1);
      const uint32_t id_u = idesc_f16(128, BV, kInBf16, 0, 1);
      const uint32_t sb = smem_u32(sm);
      // In-order: S(0), then per chunk i: W/U(i), S(i+1).  All waits suspend in
      // hardware (try_wait), so this thread takes no issue slots while idle.
      auto issue_s = [&](int c) -> bool {
        if (!mbar_wait(&bars[B_FULL + (c & 1)], (c >> 1) & 1, abort_flag)) return false;
        if (c > 0 && !mbar_wait(&bars[B_SFREE], (c - 1) & 1, abort_flag)) return false;
        tc_fence_after();
        const uint32_t kq = sb + ((c & 1) ? L::kq1 : L::kq0);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t a = kq + (kk >> 2) * 16384 + (kk & 3) * 32;
          mma_f16_ss(tmem + kTmS, sdesc(a, 16, 1024, kSw128), sdesc(a, 16, 1024, kSw128), id_s, kk > 0);
        }
        mma_commit(&bars[B_SFULL]);
        GDN_TR(1, c);
        return true;
      };
      bool okm = issue_s(0);
      for (int i = 0; i < NT && okm; ++i) {
        okm = mbar_wait(&bars[B_TREADY], i & 1, abort_flag) &&
              (i == 0 || mbar_wait(&bars[B_WFREE], (i - 1) & 1, abort_flag)) &&
              (i < 2 || mbar_wait(&bars[B_UFREE + (i & 1)], ((i >> 1) - 1) & 1, abort_flag));
        if (!okm) break;
        tc_fence_after();
        const uint32_t kq = sb + ((i & 1) ? L::kq1 : L::kq0);
        const uint32_t vt = sb + ((i & 1) ? L::vt1 : L::vt0);
        const uint32_t ts = sb + L::tstk;
        // W = [Tw; Tb_hi] K: lanes 0-63 hold W.  B = the k tile read MN-major
        // (d blocks of 64 are 16 KB apart in the stacked [k;q] layout).
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f16_ss(tmem + kTmW, sdesc(ts + kk * 32, 16, 1024, kSw128), sdesc(kq + kk * 2048, 16384, 1024, kSw128),
                     id_w, kk > 0);
        // U = [Tw | *; Tb_hi | Tb_lo] [V; V]: lanes 64-127 hold Tb_hi V + Tb_lo V.
        const uint32_t ucol = (i & 1) ? TC::u1 : TC::u0;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_f16_ss(tmem + ucol, sdesc(ts + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024, kSw128),
                     sdesc(vt + (kk & 3) * 2 * L::bv_sbo, 8192, L::bv_sbo, L::bv_swz), id_u, kk > 0);
        mma_commit(&bars[B_WFULL]);
        mma_commit(&bars[B_UFULL + (i & 1)]);
        mma_commit(&bars[B_TFREE]);
        mma_commit(&bars[B_EMPTY + (i & 1)]);
        GDN_TR(2, i);
        if (i + 1 < NT) okm = issue_s(i + 1);
      }
      if (!okm) *abort_flag = 1;
      // every issued MMA must complete before TMEM is released
      mma_commit(&bars[B_DONE]);
      volatile int never = 0;
      mbar_wait(&bars[B_DONE], 0, &never);
    }
    __syncwarp();
  } else if (warp == 2 || warp == 3) {
    const int t = tid - 64;  // chunk row 0..63
    for (int i = 0; i < NT; ++i) {
      const int s = i & 1, p = i & 1;
      if (!mbar_wait_warp(&bars[B_FULL + s], (i >> 1) & 1, abort_flag)) break;
      if (!mbar_wait_warp(&bars[B_VEC + (i & 3)], (i >> 2) & 1, abort_flag)) break;
      const float* vec = vecs + (i & 3) * kVecN * kC;
      const uint8_t* kq = sm + (s ? L::kq1 : L::kq0);
      if (!kPrepOnly) {
        // Qhat = exp(b_t) q_t -> rows 0-63 of Ahat[p]
        if (i >= 2 && !mbar_wait_warp(&bars[B_AFREE + p], ((i >> 1) - 1) & 1, abort_flag)) break;
        const float eb = vec[V_EB * kC + t];
        uint8_t* ah = sm + (p ? L::ahat1 : L::ahat0);
#pragma unroll 1
        for (int cc = 0; cc < 16; ++cc) {
          const int cb = cc >> 3, c = cc & 7;
          {
            const uint4 x = *reinterpret_cast<const uint4*>(kq + cb * 16384 + 8192 + sw128_off(t, c));
            const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
            uint32_t ys[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = Cvt<InT>::unpack(xs[e]);
              ys[e] = Cvt<__half>::pack(f.x * eb, f.y * eb);
            }
            *reinterpret_cast<uint4*>(ah + cb * 16384 + sw128_off(t, c)) = make_uint4(ys[0], ys[1], ys[2], ys[3]);
          }
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[B_AFULL + p]);
        if (t == 0) GDN_TR(5, i);
        // Kbar = exp(b_C - b_t) k_t -> Kbar (2 d-blocks x 64 rows)
        if (i >= 1 && !mbar_wait_warp(&bars[B_KFREE], (i - 1) & 1, abort_flag)) break;
        const float dd = vec[V_DD * kC + t];
        uint8_t* kb = sm + L::kbar;
#pragma unroll 1
        for (int cc = 0; cc < 16; ++cc) {
          const int cb = cc >> 3, c = cc & 7;
          {
            const uint4 x = *reinterpret_cast<const uint4*>(kq + cb * 16384 + sw128_off(t, c));
            const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
            uint32_t ys[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = Cvt<InT>::unpack(xs[e]);
              ys[e] = Cvt<__half>::pack(f.x * dd, f.y * dd);
            }
            *reinterpret_cast<uint4*>(kb + cb * 8192 + sw128_off(t, c)) = make_uint4(ys[0], ys[1], ys[2], ys[3]);
          }
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[B_KFULL]);
        if (t == 0) GDN_TR(6, i);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[B_EMPTY + s]);
    }
  } else if (warp >= 4 && warp < 8) {
    // ================================================================ prep
    // Threads 0-63 own row t of A (TMEM lanes 0-63 = K K^T rows); threads
    // 64-127 own row t of P (lanes 64-127 = Q K^T rows).  Decisions that gate
    // barriers are made uniform with bar.red.or (bar_any).
    const int ptid = tid - 128;
    const int wl = warp - 4;
    bool ok = true;
    for (int i = 0; i < NT; ++i) {
      const int p = i & 1;
      // checkpoint: also orders the previous chunk's reads of amat before new writes
      if (bar_any(1, 128, !ok || *abort_flag)) break;
      ok = mbar_wait_warp(&bars[B_VEC + (i & 3)], (i >> 2) & 1, abort_flag) &&
           mbar_wait_warp(&bars[B_SFULL], i & 1, abort_flag) &&
           (ptid < 64 || kPrepOnly || i < 2 ||
            mbar_wait_warp(&bars[B_PFREE + p], ((i >> 1) - 1) & 1, abort_flag));
      if (bar_any(1, 128, !ok || *abort_flag)) break;
      tc_fence_after();
      if (ptid == 0) GDN_TR(7, i);
      const float* vec = vecs + (i & 3) * kVecN * kC;
      // exp(b_t - b_m) = E_t F_m with E_t = 2^(b2_t - ref), F_m = 2^(ref - b2_m), valid
      // while the in-chunk log2 range stays below 200 (no fp32 overflow); otherwise
      // each factor is a direct exp2 of the difference.
      const float b2first = vec[V_B2 * kC], b2last = vec[V_B2 * kC + kC - 1];
      const float ref = 0.5f * (b2first + b2last);
      const bool prod_form = (b2first - b2last) < 200.f;
      if (ptid < 64) amat[ptid * kAStride + 64] = fast_exp2(ref - vec[V_B2 * kC + ptid]);
      named_bar(2, 128);
      {
        const int t = ptid & 63;
        const float b2t = vec[V_B2 * kC + t];
        const float et = fast_exp2(b2t - ref);
        const float bt = (ptid < 64) ? vec[V_BETA * kC + t] : 1.f;
        float* arow = amat + t * kAStride;
        uint8_t* pb = sm + (p ? L::p1 : L::p0);
#pragma unroll 1
        for (int cg = 0; cg < 4; ++cg) {
          float s[16];
          tmem_ld16w(tmem_addr(tmem + kTmS, wl * 32, cg * 16), s);
          float x[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int m = cg * 16 + e;
            const float dec = prod_form ? et * amat[m * kAStride + 64] : fast_exp2(b2t - vec[V_B2 * kC + m]);
            // A[t][m] = beta_t exp(b_t - b_m) (k_t . k_m), m < t     (gdn_ref.py:76-80)
            // P[t][m] = exp(b_t - b_m) (q_t . k_m),        m <= t    (gdn_ref.py:87-88)
            const bool keep = (ptid < 64) ? (m < t) : (m <= t);
            x[e] = keep ? bt * dec * s[e] : 0.f;
          }
          if (ptid < 64) {
#pragma unroll
            for (int e = 0; e < 16; e += 4)
              *reinterpret_cast<float4*>(arow + cg * 16 + e) = make_float4(x[e], x[e + 1], x[e + 2], x[e + 3]);
          } else if (!kPrepOnly) {
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
              uint4 w;
              w.x = Cvt<__half>::pack(x[8 * h2 + 0], x[8 * h2 + 1]);
              w.y = Cvt<__half>::pack(x[8 * h2 + 2], x[8 * h2 + 3]);
              w.z = Cvt<__half>::pack(x[8 * h2 + 4], x[8 * h2 + 5]);
              w.w = Cvt<__half>::pack(x[8 * h2 + 6], x[8 * h2 + 7]);
              *reinterpret_cast<uint4*>(pb + sw128_off(t, 2 * cg + h2)) = w;
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[B_SFREE]);
        if (ptid >= 64 && !kPrepOnly) {
          fence_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars[B_AFULL + p]);
        }
      }
      if (ptid == 0) GDN_TR(17, i);
      named_bar(1, 128);
      if (ptid == 0) GDN_TR(8, i);
      invert_unit_lower64(amat, ptid);  // T = (I + A)^-1 in place
      if (ptid == 0) GDN_TR(9, i);
      // Tstack: Tw = T diag(beta e^b) (input dtype), Tb = T diag(beta) as hi + lo
      ok = (i == 0) || mbar_wait_warp(&bars[B_TFREE], (i - 1) & 1, abort_flag);
      if (ok) {
        const int t = ptid >> 1, half = ptid & 1;
        const float* trow = amat + t * kAStride;
        uint8_t* ts = sm + L::tstk;
#pragma unroll 1
        for (int c = 4 * half; c < 4 * half + 4; ++c) {
          uint32_t ww[4], hi[4], lo[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int m = 8 * c + 2 * e;
            const float tb0 = trow[m] * vec[V_BETA * kC + m], tb1 = trow[m + 1] * vec[V_BETA * kC + m + 1];
            const float tw0 = tb0 * vec[V_EB * kC + m], tw1 = tb1 * vec[V_EB * kC + m + 1];
            ww[e] = Cvt<InT>::pack(tw0, tw1);
            hi[e] = Cvt<InT>::pack(tb0, tb1);
            const float2 hf = Cvt<InT>::unpack(hi[e]);
            lo[e] = Cvt<InT>::pack(tb0 - hf.x, tb1 - hf.y);
          }
          *reinterpret_cast<uint4*>(ts + sw128_off(t, c)) = make_uint4(ww[0], ww[1], ww[2], ww[3]);
          *reinterpret_cast<uint4*>(ts + sw128_off(64 + t, c)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
          *reinterpret_cast<uint4*>(ts + 16384 + sw128_off(64 + t, c)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[B_TREADY]);
        if (ptid == 0) GDN_TR(10, i);
      }
      // W (fp32, TMEM lanes 0-63) -> fp16 rows 64-127 of Ahat[p] (or to global in prep-only mode)
      if (ok && ptid < 64) {
        ok = mbar_wait_warp(&bars[B_WFULL], i & 1, abort_flag);
        if (ok && !kPrepOnly && i >= 2) ok = mbar_wait_warp(&bars[B_AFREE + p], ((i >> 1) - 1) & 1, abort_flag);
        if (ok) {
          tc_fence_after();
          const int t = ptid;
          uint8_t* ah = sm + (p ? L::ahat1 : L::ahat0);
#pragma unroll 1
          for (int c0 = 0; c0 < 128; c0 += 32) {
            float w[32];
            tmem_ld32w(tmem_addr(tmem + kTmW, wl * 32, c0), w);
            if (kPrepOnly) {
              if (slice == 0) store_row<float>(P.w_out + ((size_t(bh) * NT + i) * kC + t) * kK + c0, w, 32);
            } else {
              const int cb = c0 >> 6;
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                uint4 y;
                y.x = Cvt<__half>::pack(w[8 * c + 0], w[8 * c + 1]);
                y.y = Cvt<__half>::pack(w[8 * c + 2], w[8 * c + 3]);
                y.z = Cvt<__half>::pack(w[8 * c + 4], w[8 * c + 5]);
                y.w = Cvt<__half>::pack(w[8 * c + 6], w[8 * c + 7]);
                *reinterpret_cast<uint4*>(ah + cb * 16384 + sw128_off(64 + t, ((c0 & 63) >> 3) + c)) = y;
              }
            }
          }
          tc_fence_before();
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive(&bars[B_WFREE]);
            if (!kPrepOnly) mbar_arrive(&bars[B_AFULL + p]);
          }
          if (ptid == 0) GDN_TR(11, i);
        }
      }
    }
    if (!ok) *abort_flag = 1;
  } else {
    // ================================================================ chain
    // Thread r owns row d = r of h^T (all BV columns of this slice) in fp32
    // registers and TMEM lane r.  Per chunk:
    //   D1 = [Qhat; W] h^T                 (issued by r = 0)
    //   u  = U - W h^T      (rows 64-127 of D1 / the U accumulator)
    //   D2 = Kbar^T u, D3 = P u            (issued by r = 64)
    //   h  = e^{b_C} h + D2,  o = Qhat h^T + P u
    // Named barriers carry the abort decision (bar.red.or), so every thread
    // reaches the same barriers and leaves together.
    const int r = tid - 256;  // TMEM lane = state row d (0..127)
    const int wq = warp - 8;  // TMEM lane quarter of this warp
    const uint32_t sb = smem_u32(sm);
    const uint32_t id_1 = idesc_f16(128, BV, 0, 0, 1);
    const uint32_t id_2 = idesc_f16(128, BV, 0, 1, 1);
    const uint32_t id_3 = idesc_f16(128, BV, 0, 0, 1);
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
    // issue D1 for chunk c once h^T(c) is in shared memory (caller synchronised)
    auto issue_d1 = [&](int c) -> bool {
      if (!mbar_wait(&bars[B_AFULL + (c & 1)], (c >> 1) & 1, abort_flag)) return false;
      tc_fence_after();
      const uint32_t ab = sb + ((c & 1) ? L::ahat1 : L::ahat0);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        mma_f16_ss(tmem + TC::d1, sdesc(ab + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024, kSw128),
                   sdesc(sb + L::ht16 + kk * 2 * L::bv_sbo, 8192, L::bv_sbo, L::bv_swz), id_1, kk > 0);
      mma_commit(&bars[B_D1]);
      mma_commit(&bars[B_AFREE + (c & 1)]);
      GDN_TR(3, c);
      return true;
    };
    if (kPrepOnly) {
      for (int i = 0; i < NT && ok; ++i) {
        const int p = i & 1;
        if (r >= 64) {
          ok = mbar_wait_warp(&bars[B_UFULL + p], (i >> 1) & 1, abort_flag);
          if (!ok) break;
          tc_fence_after();
          float uu[32];
          tmem_ld32w(tmem_addr(tmem + (p ? TC::u1 : TC::u0), wq * 32, 0), uu);
          tc_fence_before();
          store_row<float>(P.u_out + ((size_t(bh) * NT + i) * kC + (r - 64)) * kV + v0, uu, BV);
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars[B_UFREE + p]);
        }
      }
    } else {
      st_row16<BV>(sm + L::ht16, r, 0, h);
      fence_async_smem();
      if (!bar_any(3, 128, false) && r == 0) {
        if (!issue_d1(0)) *abort_flag = 1;
      }
      for (int i = 0; i < NT; ++i) {
        const int p = i & 1;
        ok = mbar_wait_warp(&bars[B_D1], i & 1, abort_flag);
        if (ok) tc_fence_after();
        if (ok && r == 0) GDN_TR(12, i);
        float y[BV];
        if (r >= 64) {
          ok = ok && mbar_wait_warp(&bars[B_UFULL + p], (i >> 1) & 1, abort_flag);
          if (ok) {
            tc_fence_after();
            float x[BV], uu[BV];
            tmem_ld32w(tmem_addr(tmem + TC::d1, wq * 32, 0), x);
            tmem_ld32w(tmem_addr(tmem + (p ? TC::u1 : TC::u0), wq * 32, 0), uu);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars[B_UFREE + p]);
#pragma unroll
            for (int j = 0; j < BV; ++j) uu[j] -= x[j];  // u = U - W h^T   (gdn_ref.py:86)
            st_row16<BV>(sm + L::u16, r - 64, 0, uu);
            fence_async_smem();
          }
          if (r == 64) GDN_TR(13, i);
          // D2 = Kbar^T u and D3 = P u, each accumulator's k-steps issued back to back
          if (!bar_any(4, 64, !ok) && r == 64) {
            if (mbar_wait(&bars[B_KFULL], i & 1, abort_flag) &&
                mbar_wait(&bars[B_AFULL + p], (i >> 1) & 1, abort_flag)) {
              tc_fence_after();
              const uint32_t pb = sb + (p ? L::p1 : L::p0);
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                mma_f16_ss(tmem + TC::d2, sdesc(sb + L::kbar + kk * 2048, 8192, 1024, kSw128),
                           sdesc(sb + L::u16 + kk * 2 * L::bv_sbo, 8192, L::bv_sbo, L::bv_swz), id_2, kk > 0);
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                mma_f16_ss(tmem + TC::d3, sdesc(pb + kk * 32, 16, 1024, kSw128),
                           sdesc(sb + L::u16 + kk * 2 * L::bv_sbo, 8192, L::bv_sbo, L::bv_swz), id_3, kk > 0);
              mma_commit(&bars[B_D2]);
              mma_commit(&bars[B_KFREE]);
              mma_commit(&bars[B_PFREE + p]);
              GDN_TR(4, i);
            } else {
              *abort_flag = 1;
            }
          }
        } else if (ok) {
          tmem_ld32w(tmem_addr(tmem + TC::d1, wq * 32, 0), y);
        }
        ok = ok && mbar_wait_warp(&bars[B_D2], i & 1, abort_flag) &&
             mbar_wait_warp(&bars[B_VEC + (i & 3)], (i >> 2) & 1, abort_flag);
        if (ok) {
          tc_fence_after();
          if (r == 0) GDN_TR(14, i);
          float dh[BV];
          tmem_ld32w(tmem_addr(tmem + TC::d2, wq * 32, 0), dh);
          const float gam = vecs[(i & 3) * kVecN * kC + V_EB * kC + kC - 1];  // e^{b_C}
#pragma unroll
          for (int j = 0; j < BV; ++j) h[j] = fmaf(gam, h[j], dh[j]);  // h' = e^{b_C} h + Kbar^T u
          if (i + 1 < NT) st_row16<BV>(sm + L::ht16, r, 0, h);
          float z[BV];
          tmem_ld32w(tmem_addr(tmem + TC::d3, wq * 32, 0), z);
          const int t = i * kC + r;
          if (r < 64 && t < P.T) {
#pragma unroll
            for (int j = 0; j < BV; ++j) z[j] = (z[j] + y[j]) * P.scale;  // o = Qhat h^T + P u   (gdn_ref.py:89-90)
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
        if (r == 0) GDN_TR(15, i);
        if (r == 0 && i + 1 < NT && !issue_d1(i + 1)) *abort_flag = 1;
      }
    }
    if (ok && P.ht != nullptr) {
#pragma unroll
      for (int j = 0; j < BV; ++j) P.ht[hbase + size_t(v0 + j) * kK + r] = h[j];
    }
    if (!ok) *abort_flag = 1;
  }

  __syncthreads();
  if (*abort_flag && tid == 0 && P.status != nullptr) atomicOr(P.status, 1 << GDN_ERR_TIMEOUT);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TC::alloc);
  }
}


// ------------------------------------------------------------------ host side
namespace {

constexpr int kMaxDevices = 64;

bool device_is_sm100(int* dev_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  static int cached[kMaxDevices] = {0};  // 0 unknown, 1 yes, 2 no
  if (dev < 0 || dev >= kMaxDevices) return false;
  if (cached[dev] == 0) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    cached[dev] = (major == 10 && minor == 0) ? 1 : 2;
  }
  *dev_out = dev;
  return cached[dev] == 1;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int elem_size(int dt) { return dt == GDN_DTYPE_F32 ? 4 : 2; }

int validate(const gdn_fwd_args* a, bool need_out) {
  if (a == nullptr || a->abi_version != GDN_B200_ABI_VERSION) return GDN_ERR_INVALID_ARGUMENT;
  if (a->B < 1 || a->T < 1 || a->H < 1 || a->K < 1 || a->V < 1) return GDN_ERR_INVALID_ARGUMENT;
  if (!a->q || !a->k || !a->v || !a->beta) return GDN_ERR_INVALID_ARGUMENT;  // g may be NULL (g == 0)
  {
    const int known = GDN_FLAG_QK_L2NORM | GDN_FLAG_BETA_SIGMOID | GDN_FLAG_G_LOGSIGMOID | GDN_FLAG_SOLVER_NS |
                      GDN_FLAG_NS_ITERS(15);
    if (a->flags & ~known) return GDN_ERR_INVALID_ARGUMENT;
    const int iters = (a->flags >> GDN_FLAG_NS_ITERS_SHIFT) & 15;
    if ((a->flags & GDN_FLAG_SOLVER_NS) ? iters == 0 : iters != 0) return GDN_ERR_INVALID_ARGUMENT;
  }
  if (!(a->scale == a->scale) || a->scale > 3.0e38f || a->scale < -3.0e38f) return GDN_ERR_INVALID_ARGUMENT;
  if (need_out && !a->o) return GDN_ERR_INVALID_ARGUMENT;
  if (a->in_dtype != GDN_DTYPE_F16 && a->in_dtype != GDN_DTYPE_BF16) {
    return (a->in_dtype == GDN_DTYPE_F32) ? GDN_ERR_UNSUPPORTED : GDN_ERR_INVALID_ARGUMENT;
  }
  if (need_out && a->out_dtype != GDN_DTYPE_F16 && a->out_dtype != GDN_DTYPE_BF16 && a->out_dtype != GDN_DTYPE_F32)
    return GDN_ERR_INVALID_ARGUMENT;
  if (a->K != kK || a->V != kV || a->chunk_size != kC) return GDN_ERR_UNSUPPORTED;
  if (a->block_v != 0 && a->block_v != 32) return GDN_ERR_UNSUPPORTED;
  if ((long long)a->B * a->H * (kV / 32) > 0x7fffffffLL) return GDN_ERR_UNSUPPORTED;
  // TMA: 16-byte aligned bases and strides for q, k, v
  const void* in[3] = {a->q, a->k, a->v};
  const int64_t* st[3] = {a->q_stride, a->k_stride, a->v_stride};
  for (int i = 0; i < 3; ++i) {
    if (!aligned16(in[i])) return GDN_ERR_ALIGNMENT;
    for (int j = 0; j < 3; ++j) {
      if (st[i][j] <= 0 || (st[i][j] * 2) % 16 != 0) return GDN_ERR_ALIGNMENT;
    }
  }
  if (need_out) {
    const int es = elem_size(a->out_dtype);
    if (!aligned16(a->o)) return GDN_ERR_ALIGNMENT;
    for (int j = 0; j < 3; ++j)
      if (a->o_stride[j] <= 0 || (a->o_stride[j] * es) % 16 != 0) return GDN_ERR_ALIGNMENT;
  }
  for (int j = 0; j < 3; ++j)
    if (a->beta_stride[j] < 0 || a->g_stride[j] < 0) return GDN_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(a->h0) & 3u) || (reinterpret_cast<uintptr_t>(a->ht) & 3u))
    return GDN_ERR_ALIGNMENT;
  return GDN_OK;
}

bool make_input_map(CUtensorMap* m, const gdn_fwd_args* a, const void* base, const int64_t* stride, int inner,
                    int box_inner, CUtensorMapSwizzle swz) {
  const CUtensorMapDataType dt =
      a->in_dtype == GDN_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const uint64_t dims[4] = {uint64_t(inner), uint64_t(a->T), uint64_t(a->H), uint64_t(a->B)};
  const uint64_t strides[3] = {uint64_t(stride[1]) * 2, uint64_t(stride[2]) * 2, uint64_t(stride[0]) * 2};
  const uint32_t box[4] = {uint32_t(box_inner), uint32_t(kC), 1, 1};
  return make_tmap(m, dt, 4, base, dims, strides, box, swz);
}

template <int BV, typename InT, typename OutT, bool kPrep>
int launch_t(const FwdParams& p, int grid, cudaStream_t stream, int dev) {
  static bool configured[kMaxDevices] = {false};
  auto kern = gdn_fwd_kernel<BV, InT, OutT, kPrep>;
  if (!configured[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(Layout<BV>::alloc)) !=
        cudaSuccess)
      return GDN_ERR_CUDA;
    configured[dev] = true;
  }
  kern<<<grid, kThreads, Layout<BV>::alloc, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_CUDA;
}

template <typename InT, bool kPrep>
int launch_out(const gdn_fwd_args* a, const FwdParams& p, int grid, cudaStream_t s, int dev) {
  if (kPrep) return launch_t<32, InT, float, true>(p, grid, s, dev);
  switch (a->out_dtype) {
    case GDN_DTYPE_F32: return launch_t<32, InT, float, false>(p, grid, s, dev);
    case GDN_DTYPE_F16: return launch_t<32, InT, __half, false>(p, grid, s, dev);
    case GDN_DTYPE_BF16: return launch_t<32, InT, __nv_bfloat16, false>(p, grid, s, dev);
  }
  return GDN_ERR_INVALID_ARGUMENT;
}

#ifdef GDN_TRACE
long long* g_trace = nullptr;
long long* g_trace_wy = nullptr;
#endif

// Two-kernel path: per segment of chunks, the WY/UT prep kernel writes one
// packet per (b, h, chunk) into the workspace and the scan kernel consumes
// them; the state is carried between segments through ht (or the
// workspace's state area when the caller does not want ht).
int run_two_kernel(const gdn_fwd_args* a, void* stream, uint64_t per_chunk, uint64_t state_bytes) {
  constexpr int BV = 32;
  const int NT = (a->T + kC - 1) / kC;
  uint8_t* ws = static_cast<uint8_t*>(a->workspace);
  unsigned int* work = reinterpret_cast<unsigned int*>(ws);
  float* state = a->ht != nullptr ? a->ht : reinterpret_cast<float*>(ws + kWorkspaceHeaderBytes);
  uint8_t* packets = ws + kWorkspaceHeaderBytes + state_bytes;
  const int ns_max = int((a->workspace_bytes - kWorkspaceHeaderBytes - state_bytes) / per_chunk);
  WyParams wp;
  ScanParams sp;
  memset(&wp, 0, sizeof(wp));
  memset(&sp, 0, sizeof(sp));
  if (!make_input_map(&wp.tm_q, a, a->q, a->q_stride, kK, 64, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_input_map(&wp.tm_k, a, a->k, a->k_stride, kK, 64, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_input_map(&wp.tm_v, a, a->v, a->v_stride, kV, 64, CU_TENSOR_MAP_SWIZZLE_128B))
    return GDN_ERR_CUDA;
  wp.beta = a->beta;
  wp.g = a->g;
  wp.status = sp.status = a->status;
  wp.packets = packets;
  wp.work = work;
  sp.packets = packets;
  wp.sb_b = a->beta_stride[0];
  wp.sb_t = a->beta_stride[1];
  wp.sb_h = a->beta_stride[2];
  wp.sg_b = a->g_stride[0];
  wp.sg_t = a->g_stride[1];
  wp.sg_h = a->g_stride[2];
  wp.scale = a->scale == 0.f ? 1.f : a->scale;
  wp.flags = a->flags;
  sp.so_b = a->o_stride[0];
  sp.so_t = a->o_stride[1];
  sp.so_h = a->o_stride[2];
  sp.o = a->o;
  sp.ht = state;
  wp.B = sp.B = a->B;
  wp.T = sp.T = a->T;
  wp.H = sp.H = a->H;
  sp.nslice = kV / BV;
  int nsm = 0;
  {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || nsm < 1)
      return GDN_ERR_CUDA;
  }
#ifdef GDN_TRACE
  sp.trace = g_trace;
  wp.trace = g_trace_wy;
#endif
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int in_bf16 = a->in_dtype == GDN_DTYPE_BF16;
  for (int c0 = 0; c0 < NT; c0 += ns_max) {
    const int ns = (NT - c0 < ns_max) ? NT - c0 : ns_max;
    wp.c0 = sp.c0 = c0;
    wp.NS = sp.NS = ns;
    // blocks of >= 64 chunks, at most 4 (measured: 4 blocks for 340-chunk
    // segments, T = 65536; one block below 128 chunks, configs 2 and 4)
    const int nblk = ns / 64 < 1 ? 1 : (ns / 64 > 4 ? 4 : ns / 64);
    wp.blk_len = (ns + nblk - 1) / nblk;
    sp.h0 = (c0 == 0) ? a->h0 : state;
    // the prep claims its items from this counter
    if (cudaMemsetAsync(work, 0, sizeof(unsigned int), s) != cudaSuccess) return GDN_ERR_CUDA;
    int rc = run_wy(in_bf16, wp, nsm, s);
    if (rc != GDN_OK) return rc;
    rc = run_scan(a->out_dtype, sp, a->B * a->H * sp.nslice, s);
    if (rc != GDN_OK) return rc;
  }
  return GDN_OK;
}

int run(const gdn_fwd_args* a, float* w_out, float* u_out, void* stream, bool prep) {
  const int rc = validate(a, !prep);
  if (rc != GDN_OK) return rc;
  int dev = 0;
  if (!device_is_sm100(&dev)) return GDN_ERR_NO_DEVICE;
  if (prep && (w_out == nullptr || u_out == nullptr)) return GDN_ERR_INVALID_ARGUMENT;
  constexpr int BV = 32;
  if (!prep && a->workspace != nullptr) {
    const uint64_t per_chunk = uint64_t(a->B) * a->H * kPacketBytesPerChunk;
    const uint64_t state_bytes = uint64_t(a->B) * a->H * kV * kK * 4;
    if ((reinterpret_cast<uintptr_t>(a->workspace) & 255u) == 0 &&
        a->workspace_bytes >= kWorkspaceHeaderBytes + state_bytes + per_chunk)
      return run_two_kernel(a, stream, per_chunk, state_bytes);
  }
  // the single fused kernel (and the WY/UT-only mode) reads q and k as given and
  // solves with the exact blocked inverse
  if (a->flags & (GDN_FLAG_QK_L2NORM | GDN_FLAG_SOLVER_NS)) return GDN_ERR_UNSUPPORTED;
  FwdParams p;
  memset(&p, 0, sizeof(p));
  if (!make_input_map(&p.tm_q, a, a->q, a->q_stride, kK, 64, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_input_map(&p.tm_k, a, a->k, a->k_stride, kK, 64, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !make_input_map(&p.tm_v, a, a->v, a->v_stride, kV, BV, CU_TENSOR_MAP_SWIZZLE_64B))
    return GDN_ERR_CUDA;
  p.beta = a->beta;
  p.g = a->g;
  p.h0 = a->h0;
  p.ht = prep ? nullptr : a->ht;
  p.o = a->o;
  p.w_out = w_out;
  p.u_out = u_out;
  p.status = a->status;
#ifdef GDN_TRACE
  p.trace = g_trace;
#endif
  p.sb_b = a->beta_stride[0];
  p.sb_t = a->beta_stride[1];
  p.sb_h = a->beta_stride[2];
  p.sg_b = a->g_stride[0];
  p.sg_t = a->g_stride[1];
  p.sg_h = a->g_stride[2];
  p.so_b = a->o_stride[0];
  p.so_t = a->o_stride[1];
  p.so_h = a->o_stride[2];
  p.B = a->B;
  p.T = a->T;
  p.H = a->H;
  p.NT = (a->T + kC - 1) / kC;
  p.nslice = kV / BV;
  p.scale = a->scale == 0.f ? 1.f : a->scale;
  p.flags = a->flags;
  const int grid = a->B * a->H * p.nslice;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a->in_dtype == GDN_DTYPE_BF16)
    return prep ? launch_out<__nv_bfloat16, true>(a, p, grid, s, dev) : launch_out<__nv_bfloat16, false>(a, p, grid, s, dev);
  return prep ? launch_out<__half, true>(a, p, grid, s, dev) : launch_out<__half, false>(a, p, grid, s, dev);
}

}  // namespace

// Argument checks of gdn_fwd_sm100, for entry points that wrap it and must
// report an invalid or unsupported request before their own checks.
int validate_fwd_args(const gdn_fwd_args* a) { return validate(a, true); }
}  // namespace gdn

namespace gdn {
// Diagnostic: one CTA waits on an mbarrier that nothing arrives at, through
// the same bounded wait the forward kernel uses, and reports the expiry.
__global__ void wait_timeout_probe_kernel(int* status, long long limit_cycles) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const bool ok = mbar_wait_warp(&bar, 0, &abort_flag, limit_cycles);
  if (!ok && threadIdx.x == 0) atomicOr(status, 1 << GDN_ERR_TIMEOUT);
}
}  // namespace gdn

extern "C" int gdn_selftest_wait_timeout(int* status, long long limit_cycles, void* stream) {
  if (status == nullptr || limit_cycles <= 0) return GDN_ERR_INVALID_ARGUMENT;
  int dev = 0;
  if (!gdn::device_is_sm100(&dev)) return GDN_ERR_NO_DEVICE;
  gdn::wait_timeout_probe_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status, limit_cycles);
  return cudaGetLastError() == cudaSuccess ? GDN_OK : GDN_ERR_CUDA;
}

extern "C" int gdn_fwd_sm100(const gdn_fwd_args* args, void* stream) {
  return gdn::run(args, nullptr, nullptr, stream, false);
}

extern "C" int gdn_wy_prep_sm100(const gdn_fwd_args* args, float* W, float* U, void* stream) {
  return gdn::run(args, W, U, stream, true);
}

extern "C" const char* gdn_status_string(int code) {
  switch (code) {
    case GDN_OK: return "ok";
    case GDN_ERR_INVALID_ARGUMENT: return "invalid argument (pointer, shape, stride or dtype)";
    case GDN_ERR_UNSUPPORTED: return "unsupported configuration (this build: K=V=128, chunk_size=64, fp16/bf16 inputs)";
    case GDN_ERR_ALIGNMENT: return "tensor base or stride is not 16-byte aligned";
    case GDN_ERR_CUDA: return "CUDA runtime error";
    case GDN_ERR_TIMEOUT: return "device-side wait timed out (kernel aborted)";
    case GDN_ERR_NO_DEVICE: return "current device is not sm_100 (B200)";
    case GDN_ERR_SCRATCH_LIMIT: return "request too large for the fixed no-alloc scratch (256+B*H*(98560+V*K*4) bytes)";
  }
  return "unknown status";
}

extern "C" int gdn_abi_version(void) { return GDN_B200_ABI_VERSION; }

extern "C" uint64_t gdn_fwd_workspace_bytes(const gdn_fwd_args* a) {
  if (a == nullptr || a->B < 1 || a->H < 1 || a->T < 1 || a->chunk_size != gdn::kC) return 0;
  const uint64_t nt = (uint64_t(a->T) + gdn::kC - 1) / gdn::kC;
  return gdn::kWorkspaceHeaderBytes +
         uint64_t(a->B) * a->H * (nt * gdn::kPacketBytesPerChunk + uint64_t(gdn::kV) * gdn::kK * 4);
}

#ifdef GDN_TRACE
// Trace builds only: device buffer of NT * 16 int64 timestamps for CTA 0.
extern "C" void gdn_set_trace_buffer(long long* buf) { gdn::g_trace = buf; }
extern "C" void gdn_set_trace_buffer_wy(long long* buf) { gdn::g_trace_wy = buf; }
#endif
