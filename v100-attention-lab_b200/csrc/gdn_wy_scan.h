// Parameters and launchers of the two-kernel path (gdn_wy_scan.cu).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "../../include/gdn_b200.h"

namespace gdn {

// Chunk-parallel prep: reads q, k, v (TMA, 64-column boxes, 128B swizzle),
// beta and g; writes one packet per (b, h, chunk).  Persistent: launched with
// at most two CTAs per SM, each taking every G-th item (chunk) of the segment.
struct WyParams {
  CUtensorMap tm_q, tm_k, tm_v;
  const float* beta;
  const float* g;
  uint8_t* packets;  // NS packets per (b, h)
  unsigned int* work;  // item counter, zero at launch
  int* status;
  long long* trace;  // GDN_TRACE builds: phase timestamps of CTAs 0-63
  long long sb_b, sb_t, sb_h;
  long long sg_b, sg_t, sg_h;
  int B, T, H, c0, NS;  // segment = chunks [c0, c0 + NS)
  float scale;          // multiplies Q' and o_intra (q scaled)
  int flags;            // GDN_FLAG_*
  int blk_len;          // chunks per block of the item order (NS: one block): see wy_item_blocked
};

// Serial scan over the packets of one segment.
struct ScanParams {
  const float* h0;   // state at the segment start [B, H, V, K] fp32, or NULL (zeros)
  float* ht;         // state at the segment end, same layout (may alias h0)
  void* o;
  const uint8_t* packets;
  int* status;
  long long* trace;  // GDN_TRACE builds: per-chunk role timestamps of CTA 0
  long long so_b, so_t, so_h;
  int B, T, H, c0, NS, nslice;
};

// Bytes of one packet: N and Q' images, e^{b_C}, c and o_intra slices (fp16).
constexpr uint64_t kPacketBytesPerChunk = 98560;
// Workspace header (the prep's item counter) before the state area and packets.
constexpr uint64_t kWorkspaceHeaderBytes = 256;

// Launch the prep over the segment's B * H * NS items with min(items, 2 * SMs) CTAs.
int run_wy(int in_bf16, const WyParams& p, int num_sms, cudaStream_t s);
// The argument checks of gdn_fwd_sm100 (a gdn_status code; GDN_OK if the
// request is valid and supported).  Defined in gdn_fwd.cu.
int validate_fwd_args(const ::gdn_fwd_args* a);
int run_scan(int out_dtype, const ScanParams& p, int grid, cudaStream_t s);

}  // namespace gdn
