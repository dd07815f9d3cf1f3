// Internal host-side declarations shared by the kernel translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace kvbp {

enum Status : int {
  kStatusOk = 0,
  kStatusArg = 1,          // invalid argument (null pointer, bad size, misalignment)
  kStatusUnsupported = 2,  // valid but unsupported shape
  kStatusCuda = 3,         // CUDA runtime / launch failure
};

// Records a message for kvbp_last_error() (thread-local) and returns ``status``.
int fail(int status, const char* fmt, ...);

int decode_attn_score(cudaStream_t stream, int B, int Hq, int Hkv, int D, int S, const void* q, const void* kcache,
                      const void* vcache, const int* slot_pos, void* out, float* step_score, int* err,
                      int cluster_override);

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
  kPolicyCount = 8,
};

}  // namespace kvbp
