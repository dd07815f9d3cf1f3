// Weight-streaming GEMM for the decode step: Y[M, N] = X[M, K] . W[N, K]^T with M <= 32
// (the sequences of the batch), bf16 operands, fp32 accumulation, bf16 output -- the
// q/k/v, o, gate/up, down and lm_head products of _forward_jittable
// (src/counterfact_kv_eviction/jax_inference.py:949-956,1081,1095-1107,1330-1333), whose
// outputs the reference rounds to bf16.
//
// The weights dominate the traffic (M is tiny), so the kernel is an HBM stream: a
// producer warp feeds 128 x 128 weight tiles through a shared-memory ring with 2-D TMA
// loads (128-byte swizzle), and four consumer warps run mma.sync m16n8k16 with the
// activations as the M operand (16 rows per m-tile) and 32 output features per warp.
// Fusions that remove the per-token glue kernels of the step:
//   * NORM prologue: the producer warp builds each activation chunk as
//     bf16((h * inv_rms[m]) * w_norm[k]) from the residual stream h, with inv_rms formed
//     from per-tile sums of squares written by the previous GEMM's RESID epilogue
//     (RMSNorm, jax_inference.py:609-618, without a separate kernel).
//   * RESID epilogue: h = bf16(h + bf16(acc)) in place (the residual adds
//     jax_inference.py:1280,1325) plus this tile's sum of squares of the new h per row.
//   * SWIGLU epilogue: weight rows are stored gate/up interleaved in blocks of 64, so a
//     tile holds 64 gate and the matching 64 up features and writes
//     act = bf16(bf16(g * bf16(sigmoid(g))) * u) (jax_inference.py:702-704,1103-1107).
// Split-K (when N / 128 is small) writes fp32 partials; the last CTA of each column tile
// (atomic ticket) sums them in split order, so results are deterministic.
#include "common.cuh"
#include "kvbp_internal.h"

namespace kvbp {

namespace gemm {

constexpr int BN = 128;            // output features per CTA
constexpr int BK = 128;            // K per stage
constexpr int kStages = 3;
constexpr int kConsumerWarps = 4;  // 32 features each
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;
constexpr int kWBytes = BN * BK * 2;  // 32 KiB: two 128 x 64 boxes
constexpr int kWBox = kWBytes / 2;

enum Epi : int { kPlain = 0, kResid = 1, kSwiGLU = 2 };

struct Args {
  const __nv_bfloat16* x;  // [M][ldx] activations (plain) or residual stream h (norm)
  int ldx;
  const float* ss_parts;   // NORM: [n_parts][32] per-row partial sums of squares of h
  int n_parts;
  const __nv_bfloat16* norm_w;  // NORM: [K]
  float eps;
  __nv_bfloat16* out;  // PLAIN/SWIGLU: [M][ldo]; RESID: h [M][ldo], updated in place
  int ldo;
  float* ss_out;   // RESID: [N / BN][32] partial sums of squares of the new h
  float* partial;  // split-K: [splits][M][N] fp32
  int* tickets;    // split-K: [N / BN], zero between launches
  int M, N, K, splits;
  int* err;
};

template <int MT, int EPI, bool NORM>
__global__ void __launch_bounds__(kThreads) decode_gemm_kernel(const __grid_constant__ CUtensorMap wmap,
                                                               const __grid_constant__ CUtensorMap xmap, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int kABox = MT * 16 * 128;  // one 64-wide k box of the activation chunk
  constexpr int kStageBytes = kWBytes + 2 * kABox;
  uint8_t* ring = base;  // [stage][W 32 KiB | A box 0 | A box 1]
  __nv_bfloat16* wn_s = reinterpret_cast<__nv_bfloat16*>(base + kStages * kStageBytes);  // [stage][128] norm weights
  const int kc = a.K / BK;
  const int c0 = (blockIdx.y * kc) / a.splits, c1 = ((blockIdx.y + 1) * kc) / a.splits;
  const int nch = c1 - c0;
  float* inv_rms = reinterpret_cast<float*>(wn_s + kStages * BK);  // [32]
  float* red = inv_rms + 32;                         // [4 warps][32] epilogue sums
  int* flag = reinterpret_cast<int*>(red + 4 * 32);  // [0] bad, [1] last-CTA
  uint64_t* full = reinterpret_cast<uint64_t*>(flag + 4);
  uint64_t* empty = full + kStages;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int n0 = tile * BN;
  const int M = a.M;

  // one stage = two arrivals on full[st]: the constant part (weight tile, norm weights)
  // and the activation chunk, which the previous kernel produced
  auto issue_weights = [&](int u) {
    const int st = u % kStages;
    const int kb = (c0 + u) * BK;
    uint8_t* sb = ring + st * kStageBytes;
    mbar_expect_tx(&full[st], kWBytes + (NORM ? BK * 2 : 0));
    tma_load_2d(sb, &wmap, &full[st], kb, n0);
    tma_load_2d(sb + kWBox, &wmap, &full[st], kb + 64, n0);
    if (NORM) bulk_load(wn_s + st * BK, a.norm_w + kb, BK * 2, &full[st]);
  };
  auto issue_acts = [&](int u) {
    const int st = u % kStages;
    const int kb = (c0 + u) * BK;
    uint8_t* sb = ring + st * kStageBytes;
    mbar_expect_tx(&full[st], 2 * kABox);
    tma_load_2d(sb + kWBytes, &xmap, &full[st], kb, 0);
    tma_load_2d(sb + kWBytes + kABox, &xmap, &full[st], kb + 64, 0);
  };
  auto issue_stage = [&](int u) {
    issue_weights(u);
    issue_acts(u);
  };
  if (tid == kConsumers) {
    prefetch_tmap(&wmap);
    prefetch_tmap(&xmap);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 2);
      mbar_init(&empty[s], kConsumerWarps);
    }
    flag[0] = 0;
    fence_barrier_init();
    // weights are constant: stream the first stages before the previous kernel is done
    for (int u = 0; u < nch && u < kStages; ++u) issue_weights(u);
  }
  if (!KVBP_PDL_LATE) pdl_launch_dependents();
  pdl_wait();  // activations, norm statistics and workspace belong to earlier kernels
  if (tid == kConsumers)
    for (int u = 0; u < nch && u < kStages; ++u) issue_acts(u);
  if (NORM && tid < kConsumers) {
    if (tid < 32) {
      float ss = 0.f;
      if (tid < M)
        for (int t = 0; t < a.n_parts; ++t) ss += a.ss_parts[t * 32 + tid];
      inv_rms[tid] = 1.0f / sqrtf(ss / static_cast<float>(a.K) + a.eps);
    }
  }
  __syncthreads();

  // ================================ producer warp =================================
  if (warp == kConsumerWarps) {
    if (lane == 0) {
      int issued = nch < kStages ? nch : kStages;
      for (int u = kStages; u < nch; ++u) {
        const int st = u % kStages;
        if (*reinterpret_cast<volatile int*>(flag)) break;
        if (!mbar_wait_bounded(&empty[st], ((u / kStages) - 1) & 1)) {
          set_err(a.err, kErrWaitTimeout);
          atomicExch(flag, 1);
          break;
        }
        issue_stage(u);
        issued = u + 1;
      }
      if (*reinterpret_cast<volatile int*>(flag)) {
        // error path: let the loads still in flight land before the CTA can exit
        for (int u = (issued > kStages ? issued - kStages : 0); u < issued; ++u)
          mbar_wait_bounded(&full[u % kStages], (u / kStages) & 1, 1u << 16);
      }
    }
    if (KVBP_PDL_LATE) pdl_launch_dependents();
    return;
  }

  // ================================ consumer warps ================================
  const int g = lane >> 2, t = lane & 3;
  float acc[MT][4][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[mt][j][0] = acc[mt][j][1] = acc[mt][j][2] = acc[mt][j][3] = 0.f;
  float inv_lo[MT], inv_hi[MT];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    inv_lo[mt] = NORM ? inv_rms[mt * 16 + g] : 1.f;
    inv_hi[mt] = NORM ? inv_rms[mt * 16 + g + 8] : 1.f;
  }
  for (int u = 0; u < nch; ++u) {
    const int st = u % kStages;
    if (*reinterpret_cast<volatile int*>(flag)) break;
    if (!mbar_wait_bounded(&full[st], (u / kStages) & 1)) {
      set_err(a.err, kErrWaitTimeout);
      atomicExch(flag, 1);
      break;
    }
    const uint8_t* wb = ring + st * kStageBytes;
    const uint8_t* ab = wb + kWBytes;
#pragma unroll
    for (int kk = 0; kk < BK / 16; ++kk) {
      const int col = kk * 16;
      const int box = col >> 6, cb = (col & 63) >> 3;
      // A fragments (activations): rows 16*mt .. +15, k col .. col+15
      uint32_t af[MT][4];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int row = mt * 16 + (lane & 15);
        const int chunk = cb + (lane >> 4);
        ldmatrix_x4(smem_u32(ab + box * kABox + row * 128 + ((chunk ^ (row & 7)) << 4)), af[mt][0], af[mt][1],
                    af[mt][2], af[mt][3]);
        if (NORM) {
          // x = bf16((h * inv_rms[row]) * w_norm[k]) on the fragment (k = col + 2t, +1, +8, +9)
          const int kl = st * BK + col + 2 * t;
          const uint32_t w01 = *reinterpret_cast<const uint32_t*>(wn_s + kl);
          const uint32_t w89 = *reinterpret_cast<const uint32_t*>(wn_s + kl + 8);
          const float wa = bf16lo(w01), wb2 = bf16hi(w01), wc = bf16lo(w89), wd = bf16hi(w89);
          af[mt][0] = pack_bf16((bf16lo(af[mt][0]) * inv_lo[mt]) * wa, (bf16hi(af[mt][0]) * inv_lo[mt]) * wb2);
          af[mt][1] = pack_bf16((bf16lo(af[mt][1]) * inv_hi[mt]) * wa, (bf16hi(af[mt][1]) * inv_hi[mt]) * wb2);
          af[mt][2] = pack_bf16((bf16lo(af[mt][2]) * inv_lo[mt]) * wc, (bf16hi(af[mt][2]) * inv_lo[mt]) * wd);
          af[mt][3] = pack_bf16((bf16lo(af[mt][3]) * inv_hi[mt]) * wc, (bf16hi(af[mt][3]) * inv_hi[mt]) * wd);
        }
      }
      // B fragments (weights): features warp*32 .. +31, two x4 loads of 16 features each
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int j = lane >> 3;
        const int frow = warp * 32 + h * 16 + (lane & 7) + ((j >> 1) << 3);
        const int chunk = cb + (j & 1);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(smem_u32(wb + box * kWBox + frow * 128 + ((chunk ^ (frow & 7)) << 4)), b0, b1, b2, b3);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          mma_bf16_16816(acc[mt][2 * h], af[mt][0], af[mt][1], af[mt][2], af[mt][3], b0, b1);
          mma_bf16_16816(acc[mt][2 * h + 1], af[mt][0], af[mt][1], af[mt][2], af[mt][3], b2, b3);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }
  if (KVBP_PDL_LATE) pdl_launch_dependents();  // the next kernel may start its weight stream
  // acc[mt][j]: rows 16mt+g (c0,c1) and 16mt+g+8 (c2,c3); features n0 + warp*32 + 8j + 2t (+1)

  // ---- split-K: partials, then the last CTA of this column tile reduces ------------
  if (a.splits > 1) {
    float* pbase = a.partial + static_cast<size_t>(split) * M * a.N;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = n0 + warp * 32 + 8 * j + 2 * t;
        const int r0 = mt * 16 + g, r1 = r0 + 8;
        if (r0 < M) *reinterpret_cast<float2*>(&pbase[static_cast<size_t>(r0) * a.N + n]) = make_float2(acc[mt][j][0], acc[mt][j][1]);
        if (r1 < M) *reinterpret_cast<float2*>(&pbase[static_cast<size_t>(r1) * a.N + n]) = make_float2(acc[mt][j][2], acc[mt][j][3]);
      }
    __threadfence();
    named_bar(1, kConsumers);
    if (tid == 0) {
      const int prev = atomicAdd(&a.tickets[tile], 1);
      flag[1] = (prev == a.splits - 1);
    }
    named_bar(1, kConsumers);
    if (!flag[1]) return;
    __threadfence();
    // last CTA: sum every split in order
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = n0 + warp * 32 + 8 * j + 2 * t;
        const int r0 = mt * 16 + g, r1 = r0 + 8;
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
        for (int sp = 0; sp < a.splits; ++sp) {
          const float* pb = a.partial + static_cast<size_t>(sp) * M * a.N;
          if (r0 < M) {
            const float2 v = __ldcg(reinterpret_cast<const float2*>(&pb[static_cast<size_t>(r0) * a.N + n]));
            s0 += v.x;
            s1 += v.y;
          }
          if (r1 < M) {
            const float2 v = __ldcg(reinterpret_cast<const float2*>(&pb[static_cast<size_t>(r1) * a.N + n]));
            s2 += v.x;
            s3 += v.y;
          }
        }
        acc[mt][j][0] = s0;
        acc[mt][j][1] = s1;
        acc[mt][j][2] = s2;
        acc[mt][j][3] = s3;
      }
    if (tid == 0) a.tickets[tile] = 0;  // ready for the next launch
  }

  // ---- epilogues -------------------------------------------------------------------
  if (EPI == kPlain) {
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = n0 + warp * 32 + 8 * j + 2 * t;
        const int r0 = mt * 16 + g, r1 = r0 + 8;
        if (r0 < M) *reinterpret_cast<uint32_t*>(&a.out[static_cast<size_t>(r0) * a.ldo + n]) = pack_bf16(acc[mt][j][0], acc[mt][j][1]);
        if (r1 < M) *reinterpret_cast<uint32_t*>(&a.out[static_cast<size_t>(r1) * a.ldo + n]) = pack_bf16(acc[mt][j][2], acc[mt][j][3]);
      }
  } else if (EPI == kResid) {
    // h = bf16(h + bf16(acc)); per-row sum of squares of the new h over this tile
    float ssr[MT][2];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) ssr[mt][0] = ssr[mt][1] = 0.f;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = n0 + warp * 32 + 8 * j + 2 * t;
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          const int r = mt * 16 + g + 8 * hr;
          if (r < M) {
            uint32_t* hp = reinterpret_cast<uint32_t*>(&a.out[static_cast<size_t>(r) * a.ldo + n]);
            const uint32_t hv = *hp;
            const float x0 = bf16r(bf16lo(hv) + bf16r(acc[mt][j][2 * hr]));
            const float x1 = bf16r(bf16hi(hv) + bf16r(acc[mt][j][2 * hr + 1]));
            *hp = pack_bf16(x0, x1);
            ssr[mt][hr] += x0 * x0 + x1 * x1;
          }
        }
      }
    // reduce over the 4 lanes sharing a row (t), then over the 4 warps in order
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        float v = ssr[mt][hr];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        if (t == 0) red[warp * 32 + mt * 16 + g + 8 * hr] = v;
      }
    named_bar(1, kConsumers);
    if (tid < 32) {
      float s = 0.f;
      for (int w = 0; w < kConsumerWarps; ++w) s += red[w * 32 + tid];
      a.ss_out[tile * 32 + tid] = (tid < M) ? s : 0.f;
    }
  } else {  // SwiGLU: features 0..63 of the tile are gate, 64..127 the matching up
    __nv_bfloat16* stile = reinterpret_cast<__nv_bfloat16*>(ring);  // ring is free now
    named_bar(1, kConsumers);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = warp * 32 + 8 * j + 2 * t;
        const int r0 = mt * 16 + g, r1 = r0 + 8;
        *reinterpret_cast<uint32_t*>(&stile[r0 * BN + c]) = pack_bf16(acc[mt][j][0], acc[mt][j][1]);
        *reinterpret_cast<uint32_t*>(&stile[r1 * BN + c]) = pack_bf16(acc[mt][j][2], acc[mt][j][3]);
      }
    named_bar(1, kConsumers);
    const int f0 = tile * (BN / 2);
    for (int e = tid; e < M * (BN / 2); e += kConsumers) {
      const int r = e / (BN / 2), j = e % (BN / 2);
      const float gv = __bfloat162float(stile[r * BN + j]);
      const float uv = __bfloat162float(stile[r * BN + 64 + j]);
      const float sig = bf16r(1.0f / (1.0f + expf(-gv)));
      a.out[static_cast<size_t>(r) * a.ldo + f0 + j] = __float2bfloat16_rn(bf16r(gv * sig) * uv);
    }
  }
}

}  // namespace gemm

// ------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------
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

template <int MT, int EPI, bool NORM>
static cudaError_t launch_gemm(cudaStream_t stream, const CUtensorMap& map, const CUtensorMap& xmap,
                               const gemm::Args& a, int smem) {
  auto kern = gemm::decode_gemm_kernel<MT, EPI, NORM>;
  static int configured = 0;
  if (smem > configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured = smem;
  }
  dim3 grid(a.N / gemm::BN, a.splits);
  return launch_pdl(kern, grid, dim3(gemm::kThreads), smem, stream, 0, map, xmap, a);
}

int decode_gemm(cudaStream_t stream, int epi, int M, int N, int K, const void* w, const void* x, int ldx,
                const float* ss_parts, int n_parts, const void* norm_w, float eps, void* out, int ldo, float* ss_out,
                float* partial, int* tickets, int splits, int* err) {
  using namespace gemm;
  if (!w || !x || !out) return fail(kStatusArg, "decode_gemm: null pointer");
  if (M <= 0 || M > 32) return fail(kStatusUnsupported, "decode_gemm: M = %d outside 1..32", M);
  if (N <= 0 || K <= 0 || N % BN || K % BK)
    return fail(kStatusUnsupported, "decode_gemm: N (%d) and K (%d) must be positive multiples of 128", N, K);
  if (epi < kPlain || epi > kSwiGLU) return fail(kStatusArg, "decode_gemm: unknown epilogue %d", epi);
  const bool norm = norm_w != nullptr;
  if (norm && (!ss_parts || n_parts <= 0)) return fail(kStatusArg, "decode_gemm: norm needs ss_parts");
  if (epi == kResid && !ss_out) return fail(kStatusArg, "decode_gemm: residual epilogue needs ss_out");
  if (epi == kResid && N != ldo) return fail(kStatusArg, "decode_gemm: residual epilogue needs ldo == N");
  if (splits < 1 || splits > K / BK) return fail(kStatusArg, "decode_gemm: bad split count %d", splits);
  if (splits > 1 && (!partial || !tickets)) return fail(kStatusArg, "decode_gemm: split-K needs partial and tickets");
  if (N / BN > 65535 || splits > 65535) return fail(kStatusArg, "decode_gemm: grid too large");
  if ((reinterpret_cast<uintptr_t>(w) & 15) || (reinterpret_cast<uintptr_t>(x) & 15) || (ldx % 8) ||
      (reinterpret_cast<uintptr_t>(norm_w) & 15) || (reinterpret_cast<uintptr_t>(out) & 3) || (ldo % 2))
    return fail(kStatusArg, "decode_gemm: W, x, norm_w rows must be 16-byte aligned and out rows 4-byte aligned");
  EncodeTiledFnG enc = encode_fn_g();
  if (!enc) return fail(kStatusCuda, "cuTensorMapEncodeTiled unavailable");
  CUtensorMap map;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(N)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(BN)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(w), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(kStatusCuda, "decode_gemm: cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  const int MT = M > 16 ? 2 : 1;
  // activations [M][K] (row stride ldx): boxes of 64 k x 16*MT rows, rows >= M read as zero
  CUtensorMap xmap;
  cuuint64_t xdims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
  cuuint64_t xstrides[1] = {static_cast<cuuint64_t>(ldx) * 2};
  cuuint32_t xbox[2] = {64, static_cast<cuuint32_t>(16 * MT)};
  r = enc(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), xdims, xstrides, xbox, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(kStatusCuda, "decode_gemm: activation map failed (%d)", static_cast<int>(r));
  Args a;
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.ldx = ldx;
  a.ss_parts = ss_parts;
  a.n_parts = n_parts;
  a.norm_w = static_cast<const __nv_bfloat16*>(norm_w);
  a.eps = eps;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.ldo = ldo;
  a.ss_out = ss_out;
  a.partial = partial;
  a.tickets = tickets;
  a.M = M;
  a.N = N;
  a.K = K;
  a.splits = splits;
  a.err = err;
  const int smem = kStages * (kWBytes + MT * 16 * BK * 2) + kStages * BK * 2 + (32 + 4 * 32) * 4 + 16 +
                   2 * kStages * 8 + 1024;
  cudaError_t e = cudaSuccess;
#define KVBP_GEMM_CASE(mt, ep, nm) \
  if (MT == mt && epi == ep && norm == nm) e = launch_gemm<mt, ep, nm>(stream, map, xmap, a, smem); else
  KVBP_GEMM_CASE(1, kPlain, false)
  KVBP_GEMM_CASE(1, kPlain, true)
  KVBP_GEMM_CASE(1, kResid, false)
  KVBP_GEMM_CASE(1, kSwiGLU, true)
  KVBP_GEMM_CASE(1, kSwiGLU, false)
  KVBP_GEMM_CASE(2, kPlain, false)
  KVBP_GEMM_CASE(2, kPlain, true)
  KVBP_GEMM_CASE(2, kResid, false)
  KVBP_GEMM_CASE(2, kSwiGLU, true)
  KVBP_GEMM_CASE(2, kSwiGLU, false)
  return fail(kStatusUnsupported, "decode_gemm: epilogue %d with norm=%d not built", epi, static_cast<int>(norm));
#undef KVBP_GEMM_CASE
  if (e != cudaSuccess) return fail(kStatusCuda, "decode_gemm launch: %s", cudaGetErrorString(e));
  return kStatusOk;
}

}  // namespace kvbp

#include "../../include/kvbp.h"

extern "C" int kvbp_decode_gemm(kvbp_stream_t stream, int32_t epilogue, int32_t M, int32_t N, int32_t K,
                                const void* w, const void* x, int32_t ldx, const float* ss_parts, int32_t n_parts,
                                const void* norm_w, float eps, void* out, int32_t ldo, float* ss_out, float* partial,
                                int32_t* tickets, int32_t splits, int32_t* dev_err) {
  return kvbp::decode_gemm(reinterpret_cast<cudaStream_t>(stream), epilogue, M, N, K, w, x, ldx, ss_parts, n_parts,
                           norm_w, eps, out, ldo, ss_out, partial, tickets, splits, dev_err);
}
