// Parameters and launchers of the two-kernel path (gdn_wy_scan.cu).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace gdn {

struct WyParams {
  CUtensorMap tm_q, tm_k;
  const float* beta;
  const float* g;
  uint8_t* packets;  // NS packets of 40 KB per (b, h)
  int* status;
  long long sb_b, sb_t, sb_h;
  long long sg_b, sg_t, sg_h;
  int B, T, H, c0, NS;  // segment = chunks [c0, c0 + NS)
};

struct ScanParams {
  CUtensorMap tm_q, tm_k, tm_v;
  const float* beta;
  const float* g;
  const float* h0;
  float* ht;
  void* o;
  const uint8_t* packets;
  int* status;
  long long sb_b, sb_t, sb_h;
  long long sg_b, sg_t, sg_h;
  long long so_b, so_t, so_h;
  int B, T, H, c0, NS, nslice;
};

constexpr uint64_t kPacketBytesPerChunk = 40960;

int run_wy(int in_bf16, const WyParams& p, int grid, cudaStream_t s);
int run_scan(int in_bf16, int out_dtype, const ScanParams& p, int grid, cudaStream_t s);

}  // namespace gdn
