/*
 * gdn_b200.h -- C ABI of the B200 (sm_100a) chunked Gated DeltaNet forward.
 *
 * This is the drop-in boundary for the reference's forward entry point
 *
 *     gdn_chunk_fwd(q, k, v, beta, g) -> (o, h_final)
 *         gdn_triton.py:113-140   (123123213weqw/v100-attention-lab)
 *     gdn_chunk_fwd_v2(q, k, v, beta, g, C, BV, num_warps, num_stages, iters)
 *         gdn_triton_v2.py:92-117
 *
 * with the semantics of gdn_ref.py:28-45 (step recurrence) and
 * gdn_ref.py:48-99 (chunked UT form), extended by the initial state h0
 * that gdn_ref accepts but the reference kernels ignore (gdn_triton.py:52).
 *
 * Plain C: device pointers, element strides and sizes; no framework types.
 * Every entry point returns a gdn_status code; nothing throws.
 */
#ifndef GDN_B200_H_
#define GDN_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GDN_B200_ABI_VERSION 3

/* Element types (q/k/v inputs, o output). */
enum gdn_dtype {
  GDN_DTYPE_F32 = 0,
  GDN_DTYPE_F16 = 1,
  GDN_DTYPE_BF16 = 2
};

/* Status codes returned by every entry point and written to args->status. */
enum gdn_status {
  GDN_OK = 0,
  GDN_ERR_INVALID_ARGUMENT = 1, /* bad pointer, shape, stride or dtype       */
  GDN_ERR_UNSUPPORTED = 2,      /* valid request this build does not handle  */
  GDN_ERR_ALIGNMENT = 3,        /* base/stride not 16-byte aligned (TMA)     */
  GDN_ERR_CUDA = 4,             /* a CUDA runtime call failed                */
  GDN_ERR_TIMEOUT = 5,          /* a device-side bounded wait expired        */
  GDN_ERR_NO_DEVICE = 6,        /* no sm_100 device is current               */
  GDN_ERR_SCRATCH_LIMIT = 7     /* request too large for the fixed scratch   */
};

/*
 * Input preparation done inside the kernel (gdn_fwd_args.flags), replacing
 * the caller-side steps of bench_gdn.py:33-40 / gdn_ref.py:24-25:
 *   GDN_FLAG_QK_L2NORM     q and k are raw: every row is divided by
 *                          sqrt(sum of squares + 1e-6) in fp32 before use
 *   GDN_FLAG_BETA_SIGMOID  beta holds logits: beta = sigmoid(beta)
 *   GDN_FLAG_G_LOGSIGMOID  g holds logits: g = logsigmoid(g)
 * Only the two-kernel path (a workspace is given) applies GDN_FLAG_QK_L2NORM;
 * the fused kernel returns GDN_ERR_UNSUPPORTED for it.
 */
#define GDN_FLAG_QK_L2NORM 1
#define GDN_FLAG_BETA_SIGMOID 2
#define GDN_FLAG_G_LOGSIGMOID 4
/*
 * Solver of (I + A)^-1 per chunk.  Default: exact, fp32 (blocked forward
 * substitution, the role of gdn_triton.py:75-84).  GDN_FLAG_SOLVER_NS selects
 * the Newton-Schulz iteration of gdn_triton_v2.py:58-68 (fp16 tensor-core
 * products, approximate) with GDN_FLAG_NS_ITERS(n) iterations, 1 <= n <= 15;
 * two-kernel path only.
 */
#define GDN_FLAG_SOLVER_NS 8
#define GDN_FLAG_NS_ITERS_SHIFT 8
#define GDN_FLAG_NS_ITERS(n) ((int32_t)(n) << GDN_FLAG_NS_ITERS_SHIFT)

/*
 * Arguments of one forward call.  Shapes follow the reference
 * (gdn_triton.py:116-117, gdn_ref.py:11-14):
 *   q, k  [B, T, H, K]   in_dtype     (last dim contiguous)
 *   v     [B, T, H, V]   in_dtype     (last dim contiguous)
 *   beta  [B, T, H]      float32
 *   g     [B, T, H]      float32      (log decay, <= 0), or NULL for g == 0
 *                                    (no decay: the DeltaNet recurrence)
 *   h0    [B, H, V, K]   float32      contiguous, or NULL for a zero state
 *   o     [B, T, H, V]   out_dtype    (last dim contiguous)
 *   ht    [B, H, V, K]   float32      contiguous, or NULL to skip the store
 * Strides are in elements, for the (b, t, h) dimensions.
 * T need not be a multiple of chunk_size: the tail chunk is zero-padded on
 * the device with the padding rule of gdn_ref.py:102-114 (q=k=v=0, beta=0,
 * g=0), so o[t >= T] is never written and the state is unaffected.
 */
typedef struct gdn_fwd_args {
  int32_t abi_version; /* must be GDN_B200_ABI_VERSION */
  int32_t B, T, H, K, V;
  int32_t chunk_size; /* C: 64 */
  int32_t in_dtype;   /* GDN_DTYPE_F16 or GDN_DTYPE_BF16 */
  int32_t out_dtype;  /* GDN_DTYPE_F16, GDN_DTYPE_BF16 or GDN_DTYPE_F32 */
  int32_t block_v;    /* V columns per CTA (32 or 64); 0 = choose */
  const void* q;
  int64_t q_stride[3];
  const void* k;
  int64_t k_stride[3];
  const void* v;
  int64_t v_stride[3];
  const float* beta;
  int64_t beta_stride[3];
  const float* g;
  int64_t g_stride[3];
  const float* h0;
  void* o;
  int64_t o_stride[3];
  float* ht;
  int32_t* status; /* optional device int; the kernel ORs error bits into it */
  /* Scratch for the two-kernel path (see gdn_fwd_workspace_bytes).  NULL or
   * too small for one chunk per (b, h): the single fused kernel runs instead. */
  void* workspace;
  uint64_t workspace_bytes;
  /* o is computed with q scaled by `scale` (the FLA convention); 0 means 1,
   * the reference's behaviour (gdn_ref.py:45 reads q unscaled). */
  float scale;
  int32_t flags; /* GDN_FLAG_* */
} gdn_fwd_args;

/*
 * Launch the chunked GDN forward on `stream` (a cudaStream_t; NULL is the
 * legacy default stream).  Asynchronous: returns after the launch(es).
 * Replaces gdn_chunk_fwd (gdn_triton.py:113) / gdn_chunk_fwd_v2
 * (gdn_triton_v2.py:92); the caller owns and allocates o and ht, as the
 * reference allocates them inside its wrapper (gdn_triton.py:126-127).
 *
 * With a workspace it runs two kernels per segment of chunks: the
 * chunk-parallel WY/UT preparation (96.25 KB of operands per (b, h, chunk) in the
 * workspace) and the state scan; segments are sized to the workspace and the
 * state is carried between them.  Without one it runs the single fused kernel.
 */
int gdn_fwd_sm100(const gdn_fwd_args* args, void* stream);

/*
 * Workspace bytes that let gdn_fwd_sm100 run the whole sequence as one
 * segment: 256 + B*H*ceil(T/C)*98560 + B*H*V*K*4 (a 256-byte header for the
 * prep kernel's work counter, which each call zeroes itself, and the state
 * carried between segments).  Any smaller workspace of at least
 * 256 + B*H*(98560 + V*K*4) bytes works with more segments.  Its contents need
 * no initialisation.  Returns 0 for invalid arguments.
 */
uint64_t gdn_fwd_workspace_bytes(const gdn_fwd_args* args);

/*
 * Allocation-free variant of gdn_fwd_sm100, for callers that must not
 * allocate device memory when they call it: runtimes that plan all device
 * memory at start-up and forbid later allocation, plug-ins whose host
 * framework owns the memory pool, and code that cannot afford the device-wide
 * synchronisation cudaMalloc may cause.  It runs the two-kernel path with its
 * scratch in a fixed GDN_NOALLOC_SCRATCH_BYTES array inside the library
 * (args->workspace is ignored) and makes no allocation itself.
 * - Limit: 256 + B*H*(98560 + V*K*4) bytes must fit in the array (a work
 *   counter, one chunk of operands and one fp32 state per (batch, head));
 *   larger requests return
 *   GDN_ERR_SCRATCH_LIMIT before any device work.  Longer sequences are run
 *   in as many segments of chunks as the array requires.
 * - Invalid or unsupported requests return the same codes as gdn_fwd_sm100,
 *   checked before the size limit.
 * - The array is reserved on a device from the library's first use there
 *   (lazy module loading; with CUDA_MODULE_LOADING=EAGER, from context
 *   creation) until the process exits.  The first call on a device looks up
 *   the array's device address, so make it before any stream capture; the
 *   address is cached, so the entry point must not be used after a
 *   cudaDeviceReset or other reset of the device's primary context.
 * - All calls share the array: calls that may overlap on the GPU (other
 *   streams, other host threads on the same device) race and must be
 *   serialised by the caller.
 * No counterpart in the reference, whose wrapper always allocates.
 */
#define GDN_NOALLOC_SCRATCH_BYTES (32ull << 20)
int gdn_fwd_sm100_noalloc(const gdn_fwd_args* args, void* stream);

/*
 * Chunk-parallel WY/UT preparation only (the per-chunk, state-independent
 * stage of gdn_ref.py:76-85): for every chunk writes
 *   W = (I+A)^-1 (beta exp(b) k)   [B, H, NT, C, K] float32
 *   U = (I+A)^-1 (beta v)          [B, H, NT, C, V] float32
 * with NT = ceil(T / C).  Used to test that stage in isolation.
 */
int gdn_wy_prep_sm100(const gdn_fwd_args* args, float* W, float* U, void* stream);

/*
 * Diagnostic of the device-side failure detection: launches one CTA that
 * waits on an mbarrier nothing ever arrives at, with the bounded wait every
 * kernel of this library uses, limited to `limit_cycles` SM clock cycles.
 * When the limit expires the kernel ORs (1 << GDN_ERR_TIMEOUT) into *status
 * (a device int) and exits, leaving the context usable.  No counterpart in
 * the reference, whose kernels have no device-side waits.
 */
int gdn_selftest_wait_timeout(int* status, long long limit_cycles, void* stream);

/* Human-readable text of a gdn_status code. */
const char* gdn_status_string(int code);

/* GDN_B200_ABI_VERSION of the loaded library. */
int gdn_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* GDN_B200_H_ */
