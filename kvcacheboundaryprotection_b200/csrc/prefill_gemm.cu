// Prefill projections on the 5th-generation tensor cores (tcgen05 + TMEM):
// Y[M][N] = X[M][K] . W[N][K]^T with bf16 operands and fp32 accumulation, for the prompt
// rows of every sequence at once (the q/k/v, o, gate/up and down products of
// _forward_jittable over the prompt, jax_inference.py:949-956,1081,1095-1107, as the
// prefill branch :1684-1790 runs them).
//
// W is the decode GEMM's packed layout (kvbp_pack_weight): each 128-row x 128-column
// block is two 128 x 64 halves, each half the 128-byte-swizzled K-major image the MMA
// reads -- so a B tile is a 1-D bulk copy per half, no repacking.  X is row-major; its
// 128 x 64 tiles arrive by 2-D TMA with the same 128-byte swizzle.
//
// Persistent, one CTA per SM over 128-row x BN-column output tiles (BN = 256: two packed
// blocks, or 128) in a grouped raster order, warp-specialised:
//   warp 0  TMA / bulk producer over a 4-stage ring (A 16 KiB + B BN/128 x 16 KiB) that
//           runs on across tile boundaries;
//   warp 1  allocates 2 x BN TMEM columns (two accumulators) and issues tcgen05.mma
//           (M = 128, N = BN, K = 16, four per 64-wide stage) from one thread, committing
//           each stage back to the producer and each finished tile to the epilogue;
//   warps 2-5  epilogue: TMEM -> registers (each warp its 32-lane quarter) -> bf16, then
//           the accumulator goes back to the MMA warp, which meanwhile fills the other.
// Epilogues: plain (out = bf16(acc)), fp32 (out = acc: the row-parallel partial sums of
// tensor parallelism, reduced over the ranks before rounding), and SwiGLU for the
// interleaved gate/up weights
// (rows 64t..64t+63 of block t are gate features, the next 64 the matching up ones):
// act = bf16(bf16(g * bf16(sigmoid(g))) * u) with g, u the bf16 GEMM outputs
// (jax_inference.py:702-704,1103-1107), so the 2F-wide gate/up product never reaches HBM.
#include "common.cuh"
#include "kvbp_internal.h"

namespace kvbp {
namespace pg {

constexpr int kBM = 128;
constexpr int kBK = 64;  // one swizzle atom of K per stage
constexpr int kStages = 4;
constexpr int kHalf = 128 * 128;  // bytes of one 128 x 64 bf16 tile (16 KiB)
constexpr int kThreads = 6 * 32;
constexpr int kGroupM = 8;  // row tiles per raster band

struct Args {
  const __nv_bfloat16* w;  // packed [N/128][K/128][2][128][64]
  void* out;               // plain: bf16 [M][ldo] (columns n); SwiGLU: bf16 [M][ldo] (features n / 2);
                           // fp32: float [M][ldo] (columns n)
  int ldo;
  int M, N, K;
  int epi;  // 0 plain bf16, 2 SwiGLU, 3 fp32 accumulators (row-parallel partial sums)
  int* err;
};

// Output tile t of the grouped raster: consecutive t walk the N tiles of a band of kGroupM
// row tiles, so the tiles in flight at one time share both their X rows and their weight
// blocks in L2 (row-major order would stream the whole weight matrix from HBM once per row
// tile when it exceeds L2, e.g. the 7B gate/up matrix of 271 MB).
__device__ __forceinline__ void tile_of(int t, int n_tn, int n_tm, int& tm, int& tn) {
  const int per_band = kGroupM * n_tn;
  const int band = t / per_band, in_band = t % per_band;
  const int band_rows = min(n_tm - band * kGroupM, kGroupM);
  tm = band * kGroupM + in_band % band_rows;
  tn = in_band / band_rows;
}

// Persistent: one CTA per SM walks the tiles t = blockIdx.x, + gridDim.x, ...  The ring of
// (X, W) stages runs across tile boundaries, and the accumulator is double-buffered in
// TMEM (2 x BN columns), so the MMAs of tile i + 1 run while the epilogue warps drain tile i.
template <int BN>
__global__ void __launch_bounds__(kThreads, 1) prefill_gemm_kernel(const __grid_constant__ CUtensorMap xmap,
                                                                  const Args a) {
  constexpr int kNB = BN / 128;               // packed blocks per tile
  constexpr int kStage = kHalf * (1 + kNB);   // A + B bytes per stage
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(base + kStages * kStage);
  uint64_t* empty = full + kStages;
  uint64_t* accfull = empty + kStages;  // [2] MMAs of the buffer's tile complete
  uint64_t* accempty = accfull + 2;     // [2] the epilogue warps have read the buffer
  uint32_t* tslot = reinterpret_cast<uint32_t*>(accempty + 2);
  int* bad = reinterpret_cast<int*>(tslot + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_tn = a.N / BN, n_tm = (a.M + kBM - 1) / kBM;
  const int n_tiles = n_tn * n_tm;
  const int kc = a.K / 128;      // packed k-blocks
  const int nk = a.K / kBK;      // 64-wide stages per tile

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accfull[b], 1);
      mbar_init(&accempty[b], 4);  // one arrival per epilogue warp
    }
    *bad = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(2 * BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  tc_before();
  __syncthreads();
  tc_after();
  const uint32_t tmem = *tslot;
  auto healthy = [&]() { return !*reinterpret_cast<volatile int*>(bad); };
  auto wait_or_fail = [&](uint64_t* bar, uint32_t ph) {
    if (!mbar_wait_bounded(bar, ph)) {
      set_err(a.err, kErrWaitTimeout);
      atomicExch(bad, 1);
      return false;
    }
    return true;
  };

  if (warp == 0) {
    // =========================== producer =============================================
    if (lane == 0) {
      prefetch_tmap(&xmap);
      long long g = 0;  // stages issued by this CTA (over all its tiles)
      for (int t = blockIdx.x; t < n_tiles && healthy(); t += gridDim.x) {
        int tm, tn;
        tile_of(t, n_tn, n_tm, tm, tn);
        for (int u = 0; u < nk; ++u, ++g) {
          const int st = static_cast<int>(g % kStages);
          if (g >= kStages && !wait_or_fail(&empty[st], static_cast<uint32_t>((g / kStages) - 1) & 1)) break;
          if (!healthy()) break;
          uint8_t* sA = base + st * kStage;
          mbar_expect_tx(&full[st], kStage);
          tma_load_2d(sA, &xmap, &full[st], u * kBK, tm * kBM);
          for (int b = 0; b < kNB; ++b) {
            const int blk = tn * kNB + b;
            const __nv_bfloat16* src =
                a.w + ((static_cast<size_t>(blk) * kc + (u >> 1)) * 2 + (u & 1)) * (128 * 64);
            bulk_load(sA + kHalf * (1 + b), src, kHalf, &full[st]);
          }
        }
      }
      if (!healthy()) {  // let the copies in flight land before the CTA can exit
        for (long long u = (g > kStages ? g - kStages : 0); u < g; ++u)
          mbar_wait_bounded(&full[u % kStages], static_cast<uint32_t>(u / kStages) & 1, 1u << 16);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // =========================== MMA issue ============================================
    if (lane == 0) {
      constexpr uint32_t id = tc_idesc(kBM, BN);
      long long g = 0;
      int i = 0;  // tiles of this CTA so far
      for (int t = blockIdx.x; t < n_tiles && healthy(); t += gridDim.x, ++i) {
        const int buf = i & 1;
        // the epilogue has drained this buffer's previous tile (tile i - 2)
        if (i >= 2 && !wait_or_fail(&accempty[buf], static_cast<uint32_t>((i >> 1) - 1) & 1)) break;
        tc_after();
        const uint32_t acc = tmem + static_cast<uint32_t>(buf * BN);
        bool ok = true;
        for (int u = 0; u < nk; ++u, ++g) {
          const int st = static_cast<int>(g % kStages);
          if (!wait_or_fail(&full[st], static_cast<uint32_t>(g / kStages) & 1)) {
            ok = false;
            break;
          }
          tc_after();
          const uint32_t sA = smem_u32(base + st * kStage);
          const uint32_t sB = sA + kHalf;
#pragma unroll
          for (int ks = 0; ks < kBK / 16; ++ks)
            tc_mma(acc, tc_sdesc(sA + ks * 32), tc_sdesc(sB + ks * 32), id, (u > 0 || ks > 0) ? 1u : 0u);
          tc_commit(&empty[st]);
        }
        if (!ok) break;
        tc_commit(&accfull[buf]);  // arrives when every MMA issued so far is complete
      }
    }
    __syncwarp();
  } else {
    // =========================== epilogue =============================================
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    int i = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++i) {
      const int buf = i & 1;
      int tm, tn;
      tile_of(t, n_tn, n_tm, tm, tn);
      const int row = tm * kBM + q * 32 + lane;
      const bool ok = wait_or_fail(&accfull[buf], static_cast<uint32_t>(i >> 1) & 1);
      tc_after();
      if (!__all_sync(0xffffffffu, ok && healthy())) break;
      const uint32_t acc = tmem + lane_base + static_cast<uint32_t>(buf * BN);
      if (a.epi == 3) {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          float v[32];
          tc_ld32(acc + c, v);
          const int n = tn * BN + c;
          if (row < a.M && n < a.N) {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) + static_cast<size_t>(row) * a.ldo + n);
#pragma unroll
            for (int k = 0; k < 8; ++k) dst[k] = make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
          }
        }
      } else if (a.epi == 0) {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          float v[32];
          tc_ld32(acc + c, v);
          const int n = tn * BN + c;
          if (row < a.M && n < a.N) {
            uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.out) + static_cast<size_t>(row) * a.ldo + n);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              dst[k] = make_uint4(pack_bf16(v[8 * k], v[8 * k + 1]), pack_bf16(v[8 * k + 2], v[8 * k + 3]),
                                  pack_bf16(v[8 * k + 4], v[8 * k + 5]), pack_bf16(v[8 * k + 6], v[8 * k + 7]));
          }
        }
      } else {
#pragma unroll 1
        for (int b = 0; b < kNB; ++b) {
#pragma unroll 1
          for (int j = 0; j < 64; j += 32) {  // 32 gate columns and the matching 32 up columns
            float gv[32], uv[32];
            tc_ld32(acc + b * 128 + j, gv);
            tc_ld32(acc + b * 128 + 64 + j, uv);
            const int f = (tn * kNB + b) * 64 + j;  // feature index
            if (row < a.M) {
              uint32_t pk[16];
#pragma unroll
              for (int k = 0; k < 32; k += 2) {
                float r2[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                  const float g = bf16r(gv[k + e]);
                  const float up = bf16r(uv[k + e]);
                  const float sig = bf16r(1.0f / (1.0f + expf(-g)));
                  r2[e] = bf16r(g * sig) * up;
                }
                pk[k / 2] = pack_bf16(r2[0], r2[1]);
              }
              uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.out) + static_cast<size_t>(row) * a.ldo + f);
#pragma unroll
              for (int k = 0; k < 4; ++k) dst[k] = make_uint4(pk[4 * k], pk[4 * k + 1], pk[4 * k + 2], pk[4 * k + 3]);
            }
          }
        }
      }
      // this warp's TMEM reads are complete: hand the buffer back to the MMA warp
      tc_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&accempty[buf]);
    }
  }
  tc_before();
  __syncthreads();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN));
}

}  // namespace pg

using EncodeTiledFnG = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFnG encode_fn_g() {
  static EncodeTiledFnG fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFnG>(ptr);
  }
  return fn;
}

template <int BN>
static cudaError_t launch_pg(cudaStream_t stream, const CUtensorMap& xm, const pg::Args& a, int grid_n) {
  constexpr int smem = pg::kStages * pg::kHalf * (1 + BN / 128) + 1024 + 256;  // ring + barriers
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(pg::prefill_gemm_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         smem);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  const long long tiles = static_cast<long long>(grid_n) * ((a.M + pg::kBM - 1) / pg::kBM);
  const int grid = static_cast<int>(tiles < sms ? tiles : sms);  // persistent: one CTA per SM
  pg::prefill_gemm_kernel<BN><<<grid, pg::kThreads, smem, stream>>>(xm, a);
  return cudaGetLastError();
}

int prefill_gemm(cudaStream_t stream, int epilogue, int M, int N, int K, const void* w, const void* x, int ldx,
                 void* out, int ldo, int* err) {
  if (!w || !x || !out) return fail(kStatusArg, "prefill_gemm: null pointer");
  if (epilogue != 0 && epilogue != 2 && epilogue != 3)
    return fail(kStatusUnsupported, "prefill_gemm: epilogue %d (plain 0, SwiGLU 2, fp32 3)", epilogue);
  if (M <= 0 || N <= 0 || K <= 0 || N % 128 || K % 128) return fail(kStatusArg, "prefill_gemm: bad size");
  if (static_cast<long long>((M + pg::kBM - 1) / pg::kBM) * (N / 128) >= (1ll << 31))
    return fail(kStatusArg, "prefill_gemm: too many tiles");
  if (ldx < K || ldx % 8 || ldo % 8) return fail(kStatusArg, "prefill_gemm: ldx / ldo must be >= K and multiples of 8");
  if (ldo < (epilogue == 2 ? N / 2 : N)) return fail(kStatusArg, "prefill_gemm: ldo too small");
  if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15)
    return fail(kStatusArg, "prefill_gemm: pointers must be 16-byte aligned");
  EncodeTiledFnG enc = encode_fn_g();
  if (!enc) return fail(kStatusCuda, "cuTensorMapEncodeTiled unavailable");
  CUtensorMap xm;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldx) * 2};
  cuuint32_t box[2] = {64, pg::kBM};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(&xm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(kStatusCuda, "prefill_gemm: tensor map failed (%d)", static_cast<int>(r));
  pg::Args a;
  a.w = static_cast<const __nv_bfloat16*>(w);
  a.out = out;
  a.ldo = ldo;
  a.M = M;
  a.N = N;
  a.K = K;
  a.epi = epilogue;
  a.err = err;
  const bool wide = (N / 128) % 2 == 0;
  cudaError_t e = wide ? launch_pg<256>(stream, xm, a, N / 256) : launch_pg<128>(stream, xm, a, N / 128);
  if (e != cudaSuccess) return fail(kStatusCuda, "prefill_gemm launch: %s", cudaGetErrorString(e));
  return kStatusOk;
}

}  // namespace kvbp

#include "../../include/kvbp.h"

extern "C" int kvbp_prefill_gemm(kvbp_stream_t stream, int32_t epilogue, int32_t M, int32_t N, int32_t K,
                                 const void* w_packed, const void* x, int32_t ldx, void* out, int32_t ldo,
                                 int32_t* dev_err) {
  return kvbp::prefill_gemm(reinterpret_cast<cudaStream_t>(stream), epilogue, M, N, K, w_packed, x, ldx, out, ldo,
                            dev_err);
}
