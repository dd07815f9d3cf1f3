// Internal host-side declarations shared by the kernel translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

namespace kvbp {

enum Status : int {
  kStatusOk = 0,
  kStatusArg = 1,          // invalid argument (null pointer, bad size, misalignment)
  kStatusUnsupported = 2,  // valid but unsupported shape
  kStatusCuda = 3,         // CUDA runtime / launch failure
};

// Records a message for kvbp_last_error() (thread-local) and returns ``status``.
int fail(int status, const char* fmt, ...);

// Launches ``kernel`` with programmatic stream serialization (the kernel calls
// pdl_wait() before reading what the previous kernel wrote) and, when cluster.x > 0,
// thread-block clusters of that shape.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       dim3 cluster, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
#ifndef KVBP_NO_PDL
  attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[n].val.programmaticStreamSerializationAllowed = 1;
  ++n;
#endif
  if (cluster.x > 0) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster.x;
    attr[n].val.clusterDim.y = cluster.y;
    attr[n].val.clusterDim.z = cluster.z;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Optional parts of the decode attention launch (all null: attention + per-slot score).
struct AttnExtra {
  const uint8_t* head_keep = nullptr;  // per-KV-head retention [B][Hkv][S]
  float* head_score = nullptr;         // per-head signal rows [B][Hkv][S]
  const void* knew = nullptr;          // fused scatter of this step's K/V row [B][Hkv][128]
  const void* vnew = nullptr;
  float* upd_attn = nullptr;           // fused score update: the kvbp_state arrays
  float* upd_maxa = nullptr;
  double* upd_cumul = nullptr;
  int* upd_last = nullptr;
  int* upd_cnt = nullptr;
  const int* seq_step = nullptr;
  int* seq_counter = nullptr;
};
int decode_attn_score(cudaStream_t stream, int B, int Hq, int Hkv, int D, int S, const void* q, const void* kcache,
                      const void* vcache, const int* slot_pos, const int* write_slot, void* out, float* step_score,
                      int* err, int cluster_override, const AttnExtra& extra, int persist_override = 0);

int demote_int8(cudaStream_t st, void* kc, void* vc, int layers, int B, int Hkv, int S, const int* slots, int stride,
                const int* counts, int* err);
int head_signal_update(cudaStream_t stream, int B, int Hkv, int S, const int* write_slot, float* head_score,
                       double* head_cumul, float* head_current, int* err);

// Policy identifiers understood by the eviction kernels.
enum PolicyId : int {
  kPolicyLRU = 0,
  kPolicyH2OFaithful = 1,  // "attention-mass"
  kPolicyH2O = 2,          // HeavyHitterH2OLikePolicy
  kPolicySnapKV = 3,
  kPolicySnapKVFaithful = 4,
  kPolicyAdaKV = 5,
  kPolicyQuest = 6,
  kPolicyStreamingLLM = 7,
  kPolicyRandom = 8,  // victims sampled on the host (kvbp_append_evict_listed)
  kPolicyCount = 9,
};

}  // namespace kvbp
