// Weight-streaming GEMM for the decode step: Y[M, N] = X[M, K] . W[N, K]^T with M <= 32
// (the sequences of the batch), bf16 operands, fp32 accumulation, bf16 output -- the
// q/k/v, o, gate/up, down and lm_head products of _forward_jittable
// (src/counterfact_kv_eviction/jax_inference.py:949-956,1081,1095-1107,1330-1333), whose
// outputs the reference rounds to bf16.
//
// The weights dominate the traffic (M is tiny), so the kernel is an HBM stream.  Weights
// are stored pre-tiled ("packed"): every 128-feature x 128-k block is one contiguous
// 32 KiB run laid out exactly as a 128-byte-swizzled shared-memory tile (two 128 x 64
// halves), so a CTA streams one contiguous range of HBM with 1-D bulk copies -- full
// DRAM pages, no tensor map, no per-row 128-byte fragments.  A producer warp feeds a
// 3-stage ring; four consumer warps run mma.sync m16n8k16 with the activations as the
// M operand (16 rows per m-tile, loaded by 2-D TMA) and 32 output features per warp.
// For 17..32 rows, and whenever the RMSNorm prologue is fused, the main loop runs on the
// tcgen05 tensor cores instead, operands swapped: the packed weight block is the M = 128
// operand (already the 128-byte-swizzled K-major image the MMA reads), the activation
// chunk the N = 16 or 32 operand, and the fp32 accumulator lives in 32 TMEM columns; one
// thread issues the MMAs and commits each stage
// back to the producer, so the consumer warps only apply the RMSNorm prologue to the
// staged activations and read the accumulator out at the end.  Both main loops leave the
// same fp32 partial tile in shared memory, so the split-K reduction and every epilogue
// below are shared.
//
// Split-K: the `splits` CTAs of one column tile form a thread-block cluster.  Each CTA
// leaves its fp32 partial tile in its own shared memory; after a cluster barrier CTA r
// reduces rows [r*M/splits, (r+1)*M/splits) by reading every peer's tile over DSMEM in
// rank order (deterministic) and runs the epilogue on them.
//
// Fusions that remove the per-token glue kernels of the step:
//   * NORM prologue: activation fragments are formed as bf16((h * inv_rms[m]) * w_norm[k])
//     from the residual stream h, with inv_rms from per-tile sums of squares written by
//     the previous GEMM's RESID epilogue (RMSNorm, jax_inference.py:609-618).
//   * RESID epilogue: h = bf16(h + bf16(acc)) in place (the residual adds
//     jax_inference.py:1280,1325) plus this tile's sum of squares of the new h per row.
//   * SWIGLU epilogue: weight rows are stored gate/up interleaved in blocks of 64, so a
//     tile holds 64 gate and the matching 64 up features and writes
//     act = bf16(bf16(g * bf16(sigmoid(g))) * u) (jax_inference.py:702-704,1103-1107).
//   * RESID + ALLREDUCE epilogue (tensor parallelism, one rank per GPU): each CTA pushes
//     its rows of the rank's fp32 partial tile into every rank's symmetric receive buffer
//     over NVLink (peer stores), raises a per-(tile, row slice) flag on every rank
//     (release, system scope), waits for the flags of all ranks (acquire, bounded), and
//     then sums the ranks' rows in rank order before the residual add -- the o/down
//     allreduce-SUM fused into the GEMM, identical on every rank.
//   * QKV epilogue: a 128-feature tile of the stacked q/k/v projection is exactly one
//     head, so the tile finishes it in place: bias, q/k RMSNorm (Qwen3), RoPE, and the
//     store of q to its buffer or of k/v into the slot the sequence writes this step
//     (jax_inference.py:953-956,975-978,1000-1012) -- the same arithmetic as
//     kvbp_qkv_rope_scatter.
#include "common.cuh"
#include "kvbp_internal.h"

namespace kvbp {

namespace gemm {

constexpr int BN = 128;            // output features per CTA
constexpr int BK = 128;            // K per stage
#ifndef KVBP_GEMM_STAGES
#define KVBP_GEMM_STAGES 3
#endif
constexpr int kStagesM16 = KVBP_GEMM_STAGES;
// ring depth per activation height: with 32 rows (MT = 2) a third 40 KiB stage would leave
// room for one CTA per SM only; two stages keep two CTAs per SM
__host__ __device__ constexpr int stages_for(int MT) { return MT == 1 ? kStagesM16 : 2; }
#ifndef KVBP_GEMM_EARLY
#define KVBP_GEMM_EARLY 3  // weight stages issued before the wait on the previous kernel
#endif
// Consumer warps: four feature groups of 32 features, one warp per (group, 16-row m-tile)
// -- with 32 activation rows two warps share a feature group, so each warp's dependent
// ldmatrix / norm / mma chain covers one m-tile (with four warps doing both m-tiles the
// kernel was issue-latency bound: 24 % HMMA-pipe activity, 43 % issue slots busy)
__host__ __device__ constexpr int consumer_warps(int MT) { return 4 * MT; }
__host__ __device__ constexpr int gemm_threads(int MT) { return consumer_warps(MT) * 32 + 32; }
// Main loop per kernel instance: tcgen05 for 17..32 rows, and for any row count when the
// RMSNorm prologue is fused (the mma.sync loop re-forms the same normalised fragments in
// each of the four warps that share them; the tcgen05 loop rewrites each staged chunk
// once).  Without the prologue and with <= 16 rows the mma.sync loop is faster (shorter
// set-up and drain per CTA): measured on B200 for the 1-, 16- and 32-row decode shapes.
__host__ __device__ constexpr bool use_tc(int MT, bool norm) { return MT >= 2 || norm; }
constexpr int kTmemCols = 32;  // accumulator: 128 lanes (features) x 16*MT columns (rows)
constexpr int kWBytes = BN * BK * 2;  // 32 KiB: two 128 x 64 halves
constexpr int kWBox = kWBytes / 2;
constexpr int kBlockElems = BN * BK;  // one packed block
constexpr int kRedStride = BN + 8;    // fp32 partial tile row stride (fewer bank conflicts)
constexpr int kMaxSplits = 16;

enum Epi : int { kPlain = 0, kResid = 1, kSwiGLU = 2, kF32 = 3, kQKV = 4, kResidAR = 5 };

struct Args {
  const __nv_bfloat16* w;  // packed [N/128][K/128][2][128][64] (swizzled 16-byte chunks)
  const __nv_bfloat16* x;  // [M][ldx] activations (plain) or residual stream h (norm)
  int ldx;
  const float* ss_parts;   // NORM: [n_parts][32] per-row partial sums of squares of h
  int n_parts;
  const __nv_bfloat16* norm_w;  // NORM: [K]
  float eps;
  __nv_bfloat16* out;  // PLAIN/SWIGLU: [M][ldo]; RESID: h [M][ldo], updated in place; F32: float [M][ldo]
  int ldo;
  float* ss_out;  // RESID: [N / BN][32] partial sums of squares of the new h
  int M, N, K, splits;
  int* err;
  // QKV epilogue (head h = tile: q heads, then k heads, then v heads)
  const __nv_bfloat16* bias;  // [N] or null
  const __nv_bfloat16* qnw;   // [128] q RMSNorm weight or null
  const __nv_bfloat16* knw;   // [128] k RMSNorm weight or null
  const float* inv_freq;      // [64]
  const int* positions;       // [M]
  const int* write_slot;      // [M]
  int Hq, Hkv, S;
  __nv_bfloat16* q_out;   // [M][Hq][128]
  __nv_bfloat16* kcache;  // [M][Hkv][S][128]
  __nv_bfloat16* vcache;
  // RESID + ALLREDUCE epilogue: every rank's symmetric buffer holds the receive area
  //   [2 (call parity)][world (source rank)][M][N / 2] 16-byte slots {x, tag, y, tag}.
  //   Its layout depends on the world size, M and N only, never on the split count.
  const unsigned long long* peers;  // [world] base address of each rank's buffer (device array)
  int world, rank, call;            // call: index of this allreduce within the step (parity = call & 1)
  const int* epoch;                 // device counter that differs between steps
};

constexpr int kArMaxTiles = 64;  // N <= 8192
__host__ __device__ inline size_t ar_buffer_bytes(int world, int M, int N) {
  return static_cast<size_t>(2) * world * M * N * 8;
}

__device__ __forceinline__ void st_relaxed_sys_v4(uint4* p, uint4 v) {
  asm volatile("st.relaxed.sys.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 ld_relaxed_sys_v4(const uint4* p) {
  uint4 v;
  asm volatile("ld.relaxed.sys.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// named barrier that also ORs a predicate over the participating threads (the same
// result in every thread)
__device__ __forceinline__ int bar_any(int id, int nthreads, int pred) {
  int r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.s32 p, %1, 0;\n\tbar.red.or.pred q, %2, %3, p;\n\tselp.s32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(pred), "r"(id), "r"(nthreads)
      : "memory");
  return r;
}
// RMSNorm prologue on a packed bf16 pair: bf16((x * inv) * w), the mma.sync path's order
__device__ __forceinline__ uint32_t norm_pair(uint32_t x, uint32_t w, float inv) {
  return pack_bf16((bf16lo(x) * inv) * bf16lo(w), (bf16hi(x) * inv) * bf16hi(w));
}

template <int MT, int EPI, bool NORM, bool TC>
__global__ void __launch_bounds__(gemm_threads(MT)) decode_gemm_kernel(const __grid_constant__ CUtensorMap xmap,
                                                                       const Args a) {
  constexpr int kConsumerWarps = consumer_warps(MT);
  constexpr int kConsumers = kConsumerWarps * 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int kStages = stages_for(MT);
  constexpr int kABox = MT * 16 * 128;  // one 64-wide k box of the activation chunk
  constexpr int kStageBytes = kWBytes + 2 * kABox;
  static_assert(MT * 16 * kRedStride * 4 <= kStages * kStageBytes, "partial tile must fit in the ring");
  uint8_t* ring = base;  // [stage][W 32 KiB | A box 0 | A box 1]
  __nv_bfloat16* wn_s = reinterpret_cast<__nv_bfloat16*>(base + kStages * kStageBytes);  // [stage][128] norm weights
  const int kc = a.K / BK;
  const int cs = a.splits;
  const int c0 = (blockIdx.y * kc) / cs, c1 = ((blockIdx.y + 1) * kc) / cs;
  const int nch = c1 - c0;
  float* inv_rms = reinterpret_cast<float*>(wn_s + kStages * BK);  // [32]
  float* red = inv_rms + 32;                         // [32 rows][2 halves] epilogue sums
  int* flag = reinterpret_cast<int*>(red + 2 * 32);  // [0] bad, [1] its snapshot after the main loop
  uint64_t* full = reinterpret_cast<uint64_t*>(flag + 4);
  uint64_t* empty = full + kStages;
  uint64_t* accbar = empty + kStages;                         // TC: every MMA of the CTA complete
  uint32_t* tslot = reinterpret_cast<uint32_t*>(accbar + 1);  // TC: TMEM base address
  float* rtile = reinterpret_cast<float*>(ring);  // [16*MT][kRedStride] partial tile, after the main loop

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x;
  const int n0 = tile * BN;
  const int M = a.M;
  const __nv_bfloat16* wblk = a.w + (static_cast<size_t>(tile) * kc + c0) * kBlockElems;

  // one stage = two arrivals on full[st]: the constant part (weight block, norm weights)
  // and the activation chunk, which the previous kernel produced
  auto issue_weights = [&](int u) {
    const int st = u % kStages;
    mbar_expect_tx(&full[st], kWBytes + (NORM ? BK * 2 : 0));
    bulk_load(ring + st * kStageBytes, wblk + static_cast<size_t>(u) * kBlockElems, kWBytes, &full[st]);
    if (NORM) bulk_load(wn_s + st * BK, a.norm_w + (c0 + u) * BK, BK * 2, &full[st]);
  };
  auto issue_acts = [&](int u) {
    const int st = u % kStages;
    const int kb = (c0 + u) * BK;
    uint8_t* sb = ring + st * kStageBytes;
    mbar_expect_tx(&full[st], 2 * kABox);
    tma_load_2d(sb + kWBytes, &xmap, &full[st], kb, 0);
    tma_load_2d(sb + kWBytes + kABox, &xmap, &full[st], kb + 64, 0);
  };
  if (tid == kConsumers) {
    prefetch_tmap(&xmap);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 2);
      mbar_init(&empty[s], TC ? 1 : kConsumerWarps);  // TC: the MMA commit frees a stage
    }
    if (TC) mbar_init(accbar, 1);
    flag[0] = 0;
    fence_barrier_init();
  }
  if (TC && warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  if (TC) tc_before();
  __syncthreads();
  if (TC) tc_after();
  const uint32_t tmem = TC ? *tslot : 0u;
  if (!KVBP_PDL_LATE) pdl_launch_dependents();

  // ================================ producer warp =================================
  // (a TMA issue can stall its thread for microseconds, so no other thread waits for it)
  if (warp == kConsumerWarps) {
    if (lane == 0) {
      // weights are constant: stream the first stages before the previous kernel is done
      constexpr int kEarly = KVBP_GEMM_EARLY < kStages ? KVBP_GEMM_EARLY : kStages;
      for (int u = 0; u < nch && u < kEarly; ++u) issue_weights(u);
      pdl_wait();  // the activations belong to earlier kernels
      for (int u = 0; u < nch && u < kStages; ++u) {
        if (u >= kEarly) issue_weights(u);
        issue_acts(u);
      }
      int issued = nch < kStages ? nch : kStages;
      for (int u = kStages; u < nch; ++u) {
        const int st = u % kStages;
        if (*reinterpret_cast<volatile int*>(flag)) break;
        if (!mbar_wait_bounded(&empty[st], ((u / kStages) - 1) & 1)) {
          set_err(a.err, kErrWaitTimeout);
          atomicExch(flag, 1);
          break;
        }
        issue_weights(u);
        issue_acts(u);
        issued = u + 1;
      }
      if (*reinterpret_cast<volatile int*>(flag)) {
        // error path: let the loads still in flight land before the CTA can exit
        for (int u = (issued > kStages ? issued - kStages : 0); u < issued; ++u)
          mbar_wait_bounded(&full[u % kStages], (u / kStages) & 1, 1u << 16);
      }
    }
    __syncwarp();
    if (KVBP_PDL_LATE) pdl_launch_dependents();
    if (cs > 1) {  // the consumers' two cluster barriers
      cluster_sync_all();
      cluster_sync_all();
    }
    return;
  }

  // ================================ consumer warps ================================
  pdl_wait();  // activations, norm statistics and h belong to earlier kernels
  if (NORM && tid < 32) {
    float ss = 0.f;
    if (tid < M)
      for (int t = 0; t < a.n_parts; ++t) ss += a.ss_parts[t * 32 + tid];
    inv_rms[tid] = 1.0f / sqrtf(ss / static_cast<float>(a.K) + a.eps);
  }
  if (NORM) named_bar(1, kConsumers);
  const int rank = blockIdx.y;  // cluster shape (1, splits, 1): rank == split index
  const int r_lo = (rank * M) / cs, r_hi = ((rank + 1) * M) / cs;
  const int nrows = r_hi - r_lo;
  // Epilogue operands that do not depend on the accumulators, fetched for the first two
  // passes of the epilogue loops while the first stage is in flight (with 16 rows and
  // 7 splits every pass is covered); later passes load them in the loop.
  constexpr int kPre = 2;
  uint32_t pre_h[kPre] = {0u, 0u};                            // RESID: this thread's h pair
  int pre_pos[kPre] = {0, 0}, pre_slot[kPre] = {-1, -1};     // QKV: the row's position, write slot
  if (EPI == kResid) {
#pragma unroll
    for (int p = 0; p < kPre; ++p) {
      const int e = p * kConsumers + tid;
      if (e < nrows * (BN / 2)) {
        const int r = r_lo + e / (BN / 2), c = 2 * (e % (BN / 2));
        pre_h[p] = *reinterpret_cast<const uint32_t*>(&a.out[static_cast<size_t>(r) * a.ldo + n0 + c]);
      }
    }
  }
  if (EPI == kQKV) {
#pragma unroll
    for (int p = 0; p < kPre; ++p) {
      const int e = p * kConsumers + tid;
      if (e < nrows * 64) {
        const int r = r_lo + e / 64;
        if (tile < a.Hq + a.Hkv) pre_pos[p] = a.positions[r];  // q and k heads take RoPE
        if (tile >= a.Hq) pre_slot[p] = a.write_slot[r];       // k and v heads are stored
      }
    }
  }
  // one snapshot of the error flag for every consumer, taken after the main loop
  auto snapshot_flag = [&]() {
    named_bar(1, kConsumers);
    if (tid == 0) flag[1] = *reinterpret_cast<volatile int*>(flag);
    named_bar(1, kConsumers);
    return !flag[1];
  };
  bool ok;
  if constexpr (TC) {
    // ---- tcgen05 main loop: D[128 features][16*MT rows] += W[128][16] . X^T[16][16*MT],
    // eight MMAs per 128-wide stage issued by thread 0, the stage freed by their commit.
    // With the norm prologue every consumer first rewrites the staged activations in place
    // (x -> bf16((x * inv_rms[row]) * w_norm[k])) and the MMAs wait for all of them.
    constexpr uint32_t kId = tc_idesc(128, 16 * MT);
    constexpr int kChunks = 2 * MT * 16 * 8;  // 16-byte chunks of one stage's activation boxes
    if (NORM || tid == 0) {
      for (int u = 0; u < nch; ++u) {
        const int st = u % kStages;
        int bad = *reinterpret_cast<volatile int*>(flag) != 0;
        if (!bad && !mbar_wait_bounded(&full[st], (u / kStages) & 1)) {
          set_err(a.err, kErrWaitTimeout);
          atomicExch(flag, 1);
          bad = 1;
        }
        uint8_t* ab = ring + st * kStageBytes + kWBytes;
        if (NORM) {
          if (!bad) {
#pragma unroll
            for (int q = tid; q < kChunks; q += kConsumers) {
              const int box = q / (MT * 16 * 8);
              const int row = (q >> 3) % (MT * 16);
              const int pc = q & 7;            // stored chunk within the 128-byte row
              const int c = pc ^ (row & 7);    // logical chunk (128-byte swizzle)
              uint4* px = reinterpret_cast<uint4*>(ab + box * kABox + row * 128 + pc * 16);
              const uint4 wv = *reinterpret_cast<const uint4*>(wn_s + st * BK + box * 64 + c * 8);
              const float inv = inv_rms[row];
              uint4 xv = *px;
              xv.x = norm_pair(xv.x, wv.x, inv);
              xv.y = norm_pair(xv.y, wv.y, inv);
              xv.z = norm_pair(xv.z, wv.z, inv);
              xv.w = norm_pair(xv.w, wv.w, inv);
              *px = xv;
            }
            fence_proxy_async_smem();  // the tensor cores read the rewritten tile next
          }
          if (bar_any(1, kConsumers, bad)) break;  // every consumer leaves together
        } else if (bad) {
          break;
        }
        if (tid == 0) {
          tc_after();
          const uint32_t wa = smem_u32(ring + st * kStageBytes), xa = smem_u32(ab);
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              tc_mma(tmem, tc_sdesc(wa + h * kWBox + ks * 32), tc_sdesc(xa + h * kABox + ks * 32), kId,
                     (u > 0 || h > 0 || ks > 0) ? 1u : 0u);
          tc_commit(&empty[st]);
        }
      }
      if (tid == 0) tc_commit(accbar);  // also when the loop ended early: nothing stays in flight
    }
    __syncwarp();
    if (!mbar_wait_bounded(accbar, 0)) {
      set_err(a.err, kErrWaitTimeout);
      atomicExch(flag, 1);
    }
    tc_after();
    if (KVBP_PDL_LATE) pdl_launch_dependents();  // the next kernel may start its weight stream
    ok = snapshot_flag();
    // ---- accumulator -> partial tile: warp w reads features 32(w%4) .. +31 (its TMEM lane
    // quarter), rows 16(w/4) .. +15 (columns)
    if (ok) {
      const int quarter = warp & 3, half = warp >> 2;
      float v[16];
      tc_ld16(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(half * 16), v);
#pragma unroll
      for (int j = 0; j < 16; ++j) rtile[(half * 16 + j) * kRedStride + quarter * 32 + lane] = v[j];
    }
    tc_before();
  } else {
    const int g = lane >> 2, t = lane & 3;
    const int fgrp = warp & 3;  // features fgrp * 32 .. + 31 of the tile
    const int mtw = warp >> 2;  // this warp's 16-row m-tile
    float acc[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    const float inv_lo = NORM ? inv_rms[mtw * 16 + g] : 1.f;
    const float inv_hi = NORM ? inv_rms[mtw * 16 + g + 8] : 1.f;
    for (int u = 0; u < nch; ++u) {
      const int st = u % kStages;
      bool go = !*reinterpret_cast<volatile int*>(flag);
      if (go && !mbar_wait_bounded(&full[st], (u / kStages) & 1)) {
        set_err(a.err, kErrWaitTimeout);
        atomicExch(flag, 1);
        go = false;
      }
      if (!__all_sync(0xffffffffu, go)) break;  // the warp leaves together (ldmatrix/mma are warp-wide)
      const uint8_t* wb = ring + st * kStageBytes;
      const uint8_t* ab = wb + kWBytes;
#pragma unroll
      for (int kk = 0; kk < BK / 16; ++kk) {
        const int col = kk * 16;
        const int box = col >> 6, cb = (col & 63) >> 3;
        // A fragments (activations): rows 16*mtw .. +15, k col .. col+15
        uint32_t af[4];
        {
          const int row = mtw * 16 + (lane & 15);
          const int chunk = cb + (lane >> 4);
          ldmatrix_x4(smem_u32(ab + box * kABox + row * 128 + ((chunk ^ (row & 7)) << 4)), af[0], af[1], af[2], af[3]);
          if (NORM) {
            // x = bf16((h * inv_rms[row]) * w_norm[k]) on the fragment (k = col + 2t, +1, +8, +9)
            const int kl = st * BK + col + 2 * t;
            const uint32_t w01 = *reinterpret_cast<const uint32_t*>(wn_s + kl);
            const uint32_t w89 = *reinterpret_cast<const uint32_t*>(wn_s + kl + 8);
            const float wa = bf16lo(w01), wb2 = bf16hi(w01), wc = bf16lo(w89), wd = bf16hi(w89);
            af[0] = pack_bf16((bf16lo(af[0]) * inv_lo) * wa, (bf16hi(af[0]) * inv_lo) * wb2);
            af[1] = pack_bf16((bf16lo(af[1]) * inv_hi) * wa, (bf16hi(af[1]) * inv_hi) * wb2);
            af[2] = pack_bf16((bf16lo(af[2]) * inv_lo) * wc, (bf16hi(af[2]) * inv_lo) * wd);
            af[3] = pack_bf16((bf16lo(af[3]) * inv_hi) * wc, (bf16hi(af[3]) * inv_hi) * wd);
          }
        }
        // B fragments (weights): features fgrp*32 .. +31, two x4 loads of 16 features each
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int j = lane >> 3;
          const int frow = fgrp * 32 + h * 16 + (lane & 7) + ((j >> 1) << 3);
          const int chunk = cb + (j & 1);
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(smem_u32(wb + box * kWBox + frow * 128 + ((chunk ^ (frow & 7)) << 4)), b0, b1, b2, b3);
          mma_bf16_16816(acc[2 * h], af[0], af[1], af[2], af[3], b0, b1);
          mma_bf16_16816(acc[2 * h + 1], af[0], af[1], af[2], af[3], b2, b3);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
    if (KVBP_PDL_LATE) pdl_launch_dependents();  // the next kernel may start its weight stream

    // ---- partial tile -> this CTA's shared memory (the ring is idle once every warp is done)
    // acc[j]: rows 16mtw+g (c0,c1) and 16mtw+g+8 (c2,c3); columns fgrp*32 + 8j + 2t (+1)
    ok = snapshot_flag();
    if (ok) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = fgrp * 32 + 8 * j + 2 * t;
        const int r0 = mtw * 16 + g;
        *reinterpret_cast<float2*>(&rtile[r0 * kRedStride + c]) = make_float2(acc[j][0], acc[j][1]);
        *reinterpret_cast<float2*>(&rtile[(r0 + 8) * kRedStride + c]) = make_float2(acc[j][2], acc[j][3]);
      }
    }
  }
  if (cs > 1) cluster_sync_all();  // every partial tile of the cluster is complete
  else named_bar(1, kConsumers);
  if (TC && warp == 0)  // every TMEM read and MMA of the CTA is complete
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));

  // ---- reduce this CTA's row slice over the cluster (rank order) and run the epilogue
  const uint32_t rt_local = smem_u32(rtile);
  // The peers' values are all loaded before the first add (one DSMEM round trip instead of
  // one per peer), then summed in rank order.
  auto sum_pair = [&](int r, int c) -> float2 {  // columns c, c+1 of row r, summed over splits
    if (cs == 1) return *reinterpret_cast<const float2*>(&rtile[r * kRedStride + c]);
    const uint32_t off = static_cast<uint32_t>((r * kRedStride + c) * 4);
    float2 v[kMaxSplits];
#pragma unroll
    for (int q = 0; q < kMaxSplits; ++q)
      if (q < cs) v[q] = ld_dsmem_f2(mapa_u32(rt_local + off, q));
    float2 s = v[0];
#pragma unroll
    for (int q = 1; q < kMaxSplits; ++q)
      if (q < cs) {
        s.x += v[q].x;
        s.y += v[q].y;
      }
    return s;
  };
  auto sum_one = [&](int r, int c) -> float {
    if (cs == 1) return rtile[r * kRedStride + c];
    const uint32_t off = static_cast<uint32_t>((r * kRedStride + c) * 4);
    float v[kMaxSplits];
#pragma unroll
    for (int q = 0; q < kMaxSplits; ++q)
      if (q < cs) v[q] = ld_dsmem_f32(mapa_u32(rt_local + off, q));
    float s = v[0];
#pragma unroll
    for (int q = 1; q < kMaxSplits; ++q)
      if (q < cs) s += v[q];
    return s;
  };
  if (ok) {
    if (EPI == kPlain) {
      // every pass's sums first, then the stores (the lm_head's 1188 tiles run in waves, so
      // the epilogue is on the critical path)
      constexpr int kMaxPass = 8 * MT;  // nrows * 64 <= kMaxPass * kConsumers
      const int nel = nrows * (BN / 2);
      float2 v[kMaxPass];
#pragma unroll
      for (int p = 0; p < kMaxPass; ++p) {
        const int e = p * kConsumers + tid;
        if (e < nel) v[p] = sum_pair(r_lo + e / (BN / 2), 2 * (e % (BN / 2)));
      }
#pragma unroll
      for (int p = 0; p < kMaxPass; ++p) {
        const int e = p * kConsumers + tid;
        if (e < nel) {
          const int r = r_lo + e / (BN / 2), c = 2 * (e % (BN / 2));
          *reinterpret_cast<uint32_t*>(&a.out[static_cast<size_t>(r) * a.ldo + n0 + c]) = pack_bf16(v[p].x, v[p].y);
        }
      }
    } else if (EPI == kF32) {  // unrounded partial sums (a tensor-parallel shard's share)
      float* of = reinterpret_cast<float*>(a.out);
      for (int e = tid; e < nrows * (BN / 2); e += kConsumers) {
        const int r = r_lo + e / (BN / 2), c = 2 * (e % (BN / 2));
        *reinterpret_cast<float2*>(&of[static_cast<size_t>(r) * a.ldo + n0 + c]) = sum_pair(r, c);
      }
    } else if (EPI == kResid) {
      // h = bf16(h + bf16(acc)); 64 threads (two warps) per row, so each warp holds half a row
      for (int e0 = 0; e0 < nrows * (BN / 2); e0 += kConsumers) {
        const int e = e0 + tid;
        float ss = 0.f;
        if (e < nrows * (BN / 2)) {
          const int r = r_lo + e / (BN / 2), c = 2 * (e % (BN / 2));
          const int pass = e0 / kConsumers;
          uint32_t* hp = reinterpret_cast<uint32_t*>(&a.out[static_cast<size_t>(r) * a.ldo + n0 + c]);
          const uint32_t hv = pass == 0 ? pre_h[0] : (pass == 1 ? pre_h[1] : *hp);  // before the DSMEM loads
          const float2 v = sum_pair(r, c);
          const float x0 = bf16r(bf16lo(hv) + bf16r(v.x));
          const float x1 = bf16r(bf16hi(hv) + bf16r(v.y));
          *hp = pack_bf16(x0, x1);
          ss = x0 * x0 + x1 * x1;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        // e / 64 is the slice row of this warp's half row, (e / 32) & 1 the half
        if (lane == 0 && e < nrows * (BN / 2)) red[2 * (e / (BN / 2)) + ((e >> 5) & 1)] = ss;
      }
      named_bar(1, kConsumers);
      if (tid < 32) {
        const int r = tid;
        if (r >= r_lo && r < r_hi) a.ss_out[tile * 32 + r] = red[2 * (r - r_lo)] + red[2 * (r - r_lo) + 1];
        if (rank == 0 && r >= M) a.ss_out[tile * 32 + r] = 0.f;
      }
    } else if (EPI == kResidAR) {
      // Low-latency allreduce: every fp32 partial travels with its tag in the same 8 bytes
      // ({x, tag, y, tag} per column pair, one 16-byte store per peer), so a receiver
      // spins on the data itself -- no fences, no separate flags.  Each rank sums the
      // ranks' values in rank order, so every rank holds the same bits.
      const int W = a.world;
      const int par = a.call & 1;
      const uint32_t tag = static_cast<uint32_t>(*a.epoch) * 256u + static_cast<uint32_t>(a.call) + 1u;
      const int np = a.N / 2;  // column pairs per row
      auto slot = [&](int q, int src, int r, int c) {  // rank q's 16-byte slot for (src, r, pair c/2)
        return reinterpret_cast<uint4*>(a.peers[q]) + ((static_cast<size_t>(par) * W + src) * M + r) * np + (n0 + c) / 2;
      };
      // 1. this rank's rows of the tile into every peer's receive area
      for (int e = tid; e < nrows * (BN / 2); e += kConsumers) {
        const int r = r_lo + e / (BN / 2), c = 2 * (e % (BN / 2));
        const float2 val = sum_pair(r, c);
        const uint4 pk = make_uint4(__float_as_uint(val.x), tag, __float_as_uint(val.y), tag);
        for (int q = 0; q < W; ++q)
          if (q != a.rank) st_relaxed_sys_v4(slot(q, a.rank, r, c), pk);
      }
      // 2. every rank's value, summed in rank order; residual add, sums of squares
      for (int e0 = 0; e0 < nrows * (BN / 2); e0 += kConsumers) {
        const int e = e0 + tid;
        float ss = 0.f;
        if (e < nrows * (BN / 2)) {
          const int r = r_lo + e / (BN / 2), c = 2 * (e % (BN / 2));
          const float2 own = sum_pair(r, c);
          float2 sum = make_float2(0.f, 0.f);
          for (int q = 0; q < W; ++q) {
            float2 v = own;
            if (q != a.rank) {
              const uint4* src = slot(a.rank, q, r, c);
              uint4 got = ld_relaxed_sys_v4(src);
              uint32_t spins = 0;
              while (got.y != tag || got.w != tag) {
                if (++spins > (1u << 22)) {
                  set_err(a.err, kErrPeerTimeout);
                  break;
                }
                if (spins > 32) __nanosleep(64);
                got = ld_relaxed_sys_v4(src);
              }
              v = make_float2(__uint_as_float(got.x), __uint_as_float(got.z));
            }
            if (q == 0) {
              sum = v;
            } else {
              sum.x += v.x;
              sum.y += v.y;
            }
          }
          uint32_t* hp = reinterpret_cast<uint32_t*>(&a.out[static_cast<size_t>(r) * a.ldo + n0 + c]);
          const uint32_t hv = *hp;
          const float x0 = bf16r(bf16lo(hv) + bf16r(sum.x));
          const float x1 = bf16r(bf16hi(hv) + bf16r(sum.y));
          *hp = pack_bf16(x0, x1);
          ss = x0 * x0 + x1 * x1;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0 && e < nrows * (BN / 2)) red[2 * (e / (BN / 2)) + ((e >> 5) & 1)] = ss;
      }
      named_bar(1, kConsumers);
      if (tid < 32) {
        const int r = tid;
        if (r >= r_lo && r < r_hi) a.ss_out[tile * 32 + r] = red[2 * (r - r_lo)] + red[2 * (r - r_lo) + 1];
        if (rank == 0 && r >= M) a.ss_out[tile * 32 + r] = 0.f;
      }
    } else if (EPI == kSwiGLU) {  // features 0..63 of the tile are gate, 64..127 the matching up
      const int f0 = tile * (BN / 2);
      for (int e = tid; e < nrows * (BN / 2); e += kConsumers) {
        const int r = r_lo + e / (BN / 2), j = e % (BN / 2);
        const float gv = bf16r(sum_one(r, j));
        const float uv = bf16r(sum_one(r, 64 + j));
        const float sig = bf16r(1.0f / (1.0f + expf(-gv)));
        a.out[static_cast<size_t>(r) * a.ldo + f0 + j] = __float2bfloat16_rn(bf16r(gv * sig) * uv);
      }
    } else {  // QKV: one head per tile; 64 threads per row, thread i holds features i, i + 64
      const int hh = tile, i = tid & 63;
      const bool is_q = hh < a.Hq, is_k = !is_q && hh < a.Hq + a.Hkv;
      const __nv_bfloat16* nw = is_q ? a.qnw : (is_k ? a.knw : nullptr);
      // global operands first: the DSMEM loads of the reduction are ordered after them
      const float fq = (is_q || is_k) ? a.inv_freq[i] : 0.f;
      const float b0 = a.bias ? __bfloat162float(a.bias[hh * 128 + i]) : 0.f;
      const float b1 = a.bias ? __bfloat162float(a.bias[hh * 128 + i + 64]) : 0.f;
      const float nw0 = nw ? __bfloat162float(nw[i]) : 0.f;
      const float nw1 = nw ? __bfloat162float(nw[i + 64]) : 0.f;
      for (int e0 = 0; e0 < nrows * 64; e0 += kConsumers) {  // two rows per pass
        const int e = e0 + tid;
        const int pass = e0 / kConsumers;
        const bool live = e < nrows * 64;
        const int r = r_lo + e / 64;
        int pos = pass == 0 ? pre_pos[0] : pre_pos[1];
        int slot = pass == 0 ? pre_slot[0] : pre_slot[1];
        if (live && pass >= kPre) {
          if (is_q || is_k) pos = a.positions[r];
          if (!is_q) slot = a.write_slot[r];
        }
        float x0 = 0.f, x1 = 0.f;
        if (live) {
          x0 = bf16r(sum_one(r, i));  // the GEMM's bf16 output
          x1 = bf16r(sum_one(r, i + 64));
          if (a.bias) {
            x0 = bf16r(x0 + b0);
            x1 = bf16r(x1 + b1);
          }
        }
        if (nw) {  // CTA-uniform: RMSNorm over the head's 128 features
          float ss = x0 * x0 + x1 * x1;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
          if (lane == 0) red[warp] = ss;
          named_bar(1, kConsumers);
          const float tot = red[(warp >> 1) * 2] + red[(warp >> 1) * 2 + 1];
          named_bar(1, kConsumers);  // red is reused by the next pass
          const float inv = 1.0f / sqrtf(tot / 128.0f + a.eps);
          x0 = bf16r((x0 * inv) * nw0);
          x1 = bf16r((x1 * inv) * nw1);
        }
        if (!live) continue;
        if (is_q || is_k) {
          const float ang = static_cast<float>(pos) * fq;
          const float c = bf16r(cosf(ang)), sn = bf16r(sinf(ang));
          const float y0 = bf16r(bf16r(x0 * c) - bf16r(x1 * sn));
          const float y1 = bf16r(bf16r(x1 * c) + bf16r(x0 * sn));
          x0 = y0;
          x1 = y1;
        }
        __nv_bfloat16* dst;
        if (is_q) {
          dst = a.q_out + (static_cast<size_t>(r) * a.Hq + hh) * 128;
        } else {
          if (slot < 0) continue;  // position evicted before its forward: nothing to store
          if (slot >= a.S) {
            set_err(a.err, kErrIndex);
            continue;
          }
          const int kvh = is_k ? hh - a.Hq : hh - a.Hq - a.Hkv;
          dst = (is_k ? a.kcache : a.vcache) + ((static_cast<size_t>(r) * a.Hkv + kvh) * a.S + slot) * 128;
        }
        dst[i] = __float2bfloat16_rn(x0);
        dst[i + 64] = __float2bfloat16_rn(x1);
      }
    }
  }
  if (cs > 1) cluster_sync_all();  // no CTA leaves while a peer may still read its tile
}

// Packed weight layout: element (n, k) of a row-major [N][K] matrix lives in block
// (n / 128, k / 128), half (k % 128) / 64, row n % 128, 16-byte chunk
// ((k % 64) / 8) ^ (n % 8), element k % 8.  One thread moves one 16-byte chunk.
__device__ __forceinline__ size_t packed_chunk(int n, int kch, int kc_total) {
  const int tile = n >> 7, r = n & 127;
  const int kb = kch >> 4, half = (kch >> 3) & 1, c = kch & 7;
  return ((static_cast<size_t>(tile) * kc_total + kb) * 2 + half) * (128 * 8) + r * 8 + (c ^ (r & 7));
}

__global__ void pack_weight_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, int N, int K, int unpack) {
  const int kch_row = K / 8;  // 16-byte chunks per row
  const size_t total = static_cast<size_t>(N) * kch_row;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int n = static_cast<int>(i / kch_row), kch = static_cast<int>(i % kch_row);
    const size_t p = packed_chunk(n, kch, K / 128);
    if (unpack) dst[i] = src[p];
    else dst[p] = src[i];
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

static int gemm_smem_bytes(int MT) {
  using namespace gemm;
  const int kStages = stages_for(MT);
  return kStages * (kWBytes + MT * 16 * BK * 2) + kStages * BK * 2 + (32 + 2 * 32) * 4 + 16 + 2 * kStages * 8 + 16 +
         1024;
}

template <int MT, int EPI, bool NORM>
static cudaError_t launch_gemm(cudaStream_t stream, const CUtensorMap& xmap, const gemm::Args& a) {
  auto kern = gemm::decode_gemm_kernel<MT, EPI, NORM, gemm::use_tc(MT, NORM)>;
  const int smem = gemm_smem_bytes(MT);
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  dim3 grid(a.N / gemm::BN, a.splits);
  return launch_pdl(kern, grid, dim3(gemm::gemm_threads(MT)), smem, stream, a.splits > 1 ? dim3(1, a.splits, 1) : dim3(0),
                    xmap, a);
}

static int decode_gemm_launch(cudaStream_t stream, int epi, gemm::Args& a);

int decode_gemm(cudaStream_t stream, int epi, int M, int N, int K, const void* w, const void* x, int ldx,
                const float* ss_parts, int n_parts, const void* norm_w, float eps, void* out, int ldo, float* ss_out,
                int splits, int* err) {
  using namespace gemm;
  if (epi < kPlain || epi > kF32) return fail(kStatusArg, "decode_gemm: unknown epilogue %d", epi);
  if (!out) return fail(kStatusArg, "decode_gemm: null pointer");
  if (epi == kF32 && ((reinterpret_cast<uintptr_t>(out) & 7) || (ldo % 2)))
    return fail(kStatusArg, "decode_gemm: fp32 output rows must be 8-byte aligned");
  if (epi == kResid && !ss_out) return fail(kStatusArg, "decode_gemm: residual epilogue needs ss_out");
  if (epi == kResid && N != ldo) return fail(kStatusArg, "decode_gemm: residual epilogue needs ldo == N");
  if ((reinterpret_cast<uintptr_t>(out) & 3) || (ldo % 2))
    return fail(kStatusArg, "decode_gemm: out rows must be 4-byte aligned");
  Args a = {};
  a.w = static_cast<const __nv_bfloat16*>(w);
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.ldx = ldx;
  a.ss_parts = ss_parts;
  a.n_parts = n_parts;
  a.norm_w = static_cast<const __nv_bfloat16*>(norm_w);
  a.eps = eps;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.ldo = ldo;
  a.ss_out = ss_out;
  a.M = M;
  a.N = N;
  a.K = K;
  a.splits = splits;
  a.err = err;
  return decode_gemm_launch(stream, epi, a);
}

int decode_qkv_gemm(cudaStream_t stream, int M, int Hq, int Hkv, int K, const void* w, const void* x, int ldx,
                    const float* ss_parts, int n_parts, const void* norm_w, float eps, const void* bias,
                    const void* q_norm, const void* k_norm, const float* inv_freq, const int* positions,
                    const int* write_slot, int S, void* q_out, void* kcache, void* vcache, int splits, int* err) {
  using namespace gemm;
  if (!inv_freq || !positions || !write_slot || !q_out || !kcache || !vcache)
    return fail(kStatusArg, "decode_qkv_gemm: null pointer");
  if (Hq <= 0 || Hkv <= 0 || Hq % Hkv || S <= 0) return fail(kStatusArg, "decode_qkv_gemm: bad head counts or S");
  Args a = {};
  a.w = static_cast<const __nv_bfloat16*>(w);
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.ldx = ldx;
  a.ss_parts = ss_parts;
  a.n_parts = n_parts;
  a.norm_w = static_cast<const __nv_bfloat16*>(norm_w);
  a.eps = eps;
  a.M = M;
  a.N = (Hq + 2 * Hkv) * 128;
  a.K = K;
  a.splits = splits;
  a.err = err;
  a.bias = static_cast<const __nv_bfloat16*>(bias);
  a.qnw = static_cast<const __nv_bfloat16*>(q_norm);
  a.knw = static_cast<const __nv_bfloat16*>(k_norm);
  a.inv_freq = inv_freq;
  a.positions = positions;
  a.write_slot = write_slot;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.S = S;
  a.q_out = static_cast<__nv_bfloat16*>(q_out);
  a.kcache = static_cast<__nv_bfloat16*>(kcache);
  a.vcache = static_cast<__nv_bfloat16*>(vcache);
  return decode_gemm_launch(stream, kQKV, a);
}

int decode_gemm_allreduce(cudaStream_t stream, int M, int N, int K, const void* w, const void* x, int ldx, void* h,
                          float* ss_out, int splits, const unsigned long long* peers, int world, int rank, int call,
                          const int* epoch, long long buffer_bytes, int* err) {
  using namespace gemm;
  if (!h || !ss_out || !peers || !epoch) return fail(kStatusArg, "decode_gemm_allreduce: null pointer");
  if (world < 1 || world > 64 || rank < 0 || rank >= world || call < 0 || call > 254)
    return fail(kStatusArg, "decode_gemm_allreduce: bad world %d / rank %d / call %d", world, rank, call);
  if (N <= 0 || N % BN || N / BN > kArMaxTiles || splits < 1 || splits > kMaxSplits)
    return fail(kStatusArg, "decode_gemm_allreduce: bad size (N %d, splits %d)", N, splits);
  {
    // the ranks' CTAs wait on each other: every CTA of the grid must be resident at once
    const int MT = M > 16 ? 2 : 1;
    const int smem = gemm_smem_bytes(MT);
    auto kern = MT == 2 ? decode_gemm_kernel<2, kResidAR, false, use_tc(2, false)>
                        : decode_gemm_kernel<1, kResidAR, false, use_tc(1, false)>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return fail(kStatusCuda, "decode_gemm_allreduce: %s", cudaGetErrorString(e));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(N / BN, splits);
    cfg.blockDim = dim3(gemm_threads(MT));
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 1;
    attr.val.clusterDim.y = splits;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
    if (e != cudaSuccess) return fail(kStatusCuda, "decode_gemm_allreduce: occupancy query: %s", cudaGetErrorString(e));
    if (clusters < N / BN)
      return fail(kStatusUnsupported, "decode_gemm_allreduce: %d column tiles but only %d clusters of %d resident",
                  N / BN, clusters, splits);
  }
  const size_t need = ar_buffer_bytes(world, M, N);
  if (buffer_bytes < 0 || static_cast<size_t>(buffer_bytes) < need)
    return fail(kStatusArg, "decode_gemm_allreduce: symmetric buffer of %lld bytes < %zu needed", buffer_bytes, need);
  if (reinterpret_cast<uintptr_t>(h) & 3) return fail(kStatusArg, "decode_gemm_allreduce: h rows must be 4-byte aligned");
  Args a = {};
  a.w = static_cast<const __nv_bfloat16*>(w);
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.ldx = ldx;
  a.out = static_cast<__nv_bfloat16*>(h);
  a.ldo = N;
  a.ss_out = ss_out;
  a.M = M;
  a.N = N;
  a.K = K;
  a.splits = splits;
  a.err = err;
  a.peers = peers;
  a.world = world;
  a.rank = rank;
  a.call = call;
  a.epoch = epoch;
  return decode_gemm_launch(stream, kResidAR, a);
}

static int decode_gemm_launch(cudaStream_t stream, int epi, gemm::Args& a) {
  using namespace gemm;
  const int M = a.M, N = a.N, K = a.K, splits = a.splits, ldx = a.ldx, n_parts = a.n_parts;
  const void* w = a.w;
  const void* x = a.x;
  const void* norm_w = a.norm_w;
  const float* ss_parts = a.ss_parts;
  if (!w || !x) return fail(kStatusArg, "decode_gemm: null pointer");
  if (M <= 0 || M > 32) return fail(kStatusUnsupported, "decode_gemm: M = %d outside 1..32", M);
  if (N <= 0 || K <= 0 || N % BN || K % BK)
    return fail(kStatusUnsupported, "decode_gemm: N (%d) and K (%d) must be positive multiples of 128", N, K);
  const bool norm = norm_w != nullptr;
  if (norm && (!ss_parts || n_parts <= 0)) return fail(kStatusArg, "decode_gemm: norm needs ss_parts");
  if (splits < 1 || splits > kMaxSplits || splits > K / BK)
    return fail(kStatusArg, "decode_gemm: split count %d outside 1..min(16, K/128)", splits);
  if (N / BN > 65535) return fail(kStatusArg, "decode_gemm: grid too large");
  if ((reinterpret_cast<uintptr_t>(w) & 15) || (reinterpret_cast<uintptr_t>(x) & 15) || (ldx % 8) ||
      (reinterpret_cast<uintptr_t>(norm_w) & 15))
    return fail(kStatusArg, "decode_gemm: W, x and norm_w rows must be 16-byte aligned");
  EncodeTiledFnG enc = encode_fn_g();
  if (!enc) return fail(kStatusCuda, "cuTensorMapEncodeTiled unavailable");
  const int MT = M > 16 ? 2 : 1;
  // activations [M][K] (row stride ldx): boxes of 64 k x 16*MT rows, rows >= M read as zero
  CUtensorMap xmap;
  cuuint64_t xdims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
  cuuint64_t xstrides[1] = {static_cast<cuuint64_t>(ldx) * 2};
  cuuint32_t xbox[2] = {64, static_cast<cuuint32_t>(16 * MT)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), xdims, xstrides, xbox, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(kStatusCuda, "decode_gemm: activation map failed (%d)", static_cast<int>(r));
  cudaError_t e = cudaSuccess;
#define KVBP_GEMM_CASE(mt, ep, nm) \
  if (MT == mt && epi == ep && norm == nm) e = launch_gemm<mt, ep, nm>(stream, xmap, a); else
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
  KVBP_GEMM_CASE(1, kF32, false)
  KVBP_GEMM_CASE(1, kF32, true)
  KVBP_GEMM_CASE(2, kF32, false)
  KVBP_GEMM_CASE(2, kF32, true)
  KVBP_GEMM_CASE(1, kResidAR, false)
  KVBP_GEMM_CASE(2, kResidAR, false)
  KVBP_GEMM_CASE(1, kQKV, true)
  KVBP_GEMM_CASE(1, kQKV, false)
  KVBP_GEMM_CASE(2, kQKV, true)
  KVBP_GEMM_CASE(2, kQKV, false)
  return fail(kStatusUnsupported, "decode_gemm: epilogue %d with norm=%d not built", epi, static_cast<int>(norm));
#undef KVBP_GEMM_CASE
  if (e != cudaSuccess) return fail(kStatusCuda, "decode_gemm launch: %s", cudaGetErrorString(e));
  return kStatusOk;
}

int pack_weight(cudaStream_t stream, int N, int K, const void* src, void* dst, int unpack) {
  if (!src || !dst) return fail(kStatusArg, "pack_weight: null pointer");
  if (N <= 0 || K <= 0 || N % 128 || K % 128)
    return fail(kStatusUnsupported, "pack_weight: N (%d) and K (%d) must be positive multiples of 128", N, K);
  if ((reinterpret_cast<uintptr_t>(src) & 15) || (reinterpret_cast<uintptr_t>(dst) & 15))
    return fail(kStatusArg, "pack_weight: src and dst must be 16-byte aligned");
  const size_t bytes = static_cast<size_t>(N) * K * 2;
  const uintptr_t s0 = reinterpret_cast<uintptr_t>(src), d0 = reinterpret_cast<uintptr_t>(dst);
  if (s0 < d0 + bytes && d0 < s0 + bytes) return fail(kStatusArg, "pack_weight: src and dst overlap");
  const size_t chunks = static_cast<size_t>(N) * (K / 8);
  size_t blocks = (chunks + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  gemm::pack_weight_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(static_cast<const uint4*>(src),
                                                                          static_cast<uint4*>(dst), N, K, unpack);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(kStatusCuda, "pack_weight launch: %s", cudaGetErrorString(e));
  return kStatusOk;
}

}  // namespace kvbp

#include "../../include/kvbp.h"

extern "C" int kvbp_decode_gemm(kvbp_stream_t stream, int32_t epilogue, int32_t M, int32_t N, int32_t K,
                                const void* w_packed, const void* x, int32_t ldx, const float* ss_parts,
                                int32_t n_parts, const void* norm_w, float eps, void* out, int32_t ldo, float* ss_out,
                                int32_t splits, int32_t* dev_err) {
  return kvbp::decode_gemm(reinterpret_cast<cudaStream_t>(stream), epilogue, M, N, K, w_packed, x, ldx, ss_parts,
                           n_parts, norm_w, eps, out, ldo, ss_out, splits, dev_err);
}

extern "C" int kvbp_decode_qkv_gemm(kvbp_stream_t stream, int32_t M, int32_t n_heads, int32_t n_kv_heads, int32_t K,
                                    const void* w_packed, const void* x, int32_t ldx, const float* ss_parts,
                                    int32_t n_parts, const void* norm_w, float eps, const void* bias,
                                    const void* q_norm, const void* k_norm, const float* inv_freq,
                                    const int32_t* positions, const int32_t* write_slot, int32_t S, void* q_out,
                                    void* kcache, void* vcache, int32_t splits, int32_t* dev_err) {
  return kvbp::decode_qkv_gemm(reinterpret_cast<cudaStream_t>(stream), M, n_heads, n_kv_heads, K, w_packed, x, ldx,
                               ss_parts, n_parts, norm_w, eps, bias, q_norm, k_norm, inv_freq, positions, write_slot,
                               S, q_out, kcache, vcache, splits, dev_err);
}

extern "C" int kvbp_decode_gemm_allreduce(kvbp_stream_t stream, int32_t M, int32_t N, int32_t K,
                                          const void* w_packed, const void* x, int32_t ldx, void* h, float* ss_out,
                                          int32_t splits, const uint64_t* peer_bases, int32_t world, int32_t rank,
                                          int32_t call_index, const int32_t* epoch, int64_t buffer_bytes,
                                          int32_t* dev_err) {
  return kvbp::decode_gemm_allreduce(reinterpret_cast<cudaStream_t>(stream), M, N, K, w_packed, x, ldx, h, ss_out,
                                     splits, reinterpret_cast<const unsigned long long*>(peer_bases), world, rank,
                                     call_index, epoch, buffer_bytes, dev_err);
}

extern "C" int kvbp_pack_weight(kvbp_stream_t stream, int32_t N, int32_t K, const void* src, void* dst) {
  return kvbp::pack_weight(reinterpret_cast<cudaStream_t>(stream), N, K, src, dst, 0);
}

extern "C" int kvbp_unpack_weight(kvbp_stream_t stream, int32_t N, int32_t K, const void* src, void* dst) {
  return kvbp::pack_weight(reinterpret_cast<cudaStream_t>(stream), N, K, src, dst, 1);
}
