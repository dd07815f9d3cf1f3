// Fused decode attention over the capped KV slot cache + per-slot eviction score.
//
// One decode step of GQA attention for one layer (the reference computes it in
// src/counterfact_kv_eviction/jax_inference.py:1018-1050 over every cache column with
// an additive mask, and reduces the probabilities by max over heads at :1345 and over
// layers at :1670-1673).  Here attention runs over the S slots of a compact cache;
// free slots (slot_pos < 0) are excluded, which gives the same probabilities as the
// reference's -1e9 mask (those columns underflow to exactly 0 there).
//
// Numerics follow the reference's rounding points:
//   s_j   = bf16( bf16(q . k_j) * bf16(1/sqrt(128)) )      q.k accumulated in fp32
//   p_j   = exp(s_j - M) / sum_i exp(s_i - M)              fp32
//   out   = bf16( sum_j p_j * fp32(v_j) )                   fp32 accumulation
//   score[slot] = max over the layer's query heads of p   -> atomicMax into step_score
//
// Work decomposition (B200): grid = (CS, Hkv, B) with a thread-block cluster of CS CTAs
// per (sequence, kv head); each CTA owns a contiguous range of 64-slot tiles.  The last
// warp is a TMA producer that streams (K tile, V tile) pairs through a shared-memory ring
// (tensor-map loads, 128-byte swizzle, no multicast; full/empty mbarriers).  The consumer
// warps form two groups of four that take alternate tiles (two tiles in flight through
// the compute, so one group's dependent mma/softmax chain overlaps the other's); within a
// group each warp owns 16 slots of the tile.  Every warp runs one continuous
// flash-decoding pass with no CTA-wide synchronisation per tile:
//   Q.K^T   tensor cores (mma.sync m16n8k16: slots on M, the <= 8 query heads of the
//           group on N); the rounded logits are kept in shared memory,
//   softmax online per warp (running max / sum per head, rescaled partial output),
//   P.V     tensor cores: V^T from the swizzled tile via ldmatrix.trans, the weights
//           split into bf16 hi + lo parts (two mma, ~16-bit mantissa), fp32 accumulate.
// At the end the warps' (max, sum, O) are merged in shared memory and one st.async
// round pushes every CTA's (max, sum) and its O slice r to cluster CTA r (transaction-
// counted mbarrier).  Each CTA then forms the final max M and sum L, writes its slice
// of bf16 output, and turns its stored logits into the exact probabilities
// p = exp(s - M) * (1 / L) for the per-slot score (max over heads -> atomicMax).  The K/V
// cache is read exactly once, in a single stream.
//
// Early streaming: the kernel is launched with programmatic dependent launch, so its
// CTAs can be resident while the q/k/v kernel before it finishes.  When the caller
// passes write_slot (the one slot per sequence that the preceding kernels store this
// step's K/V into), the producer issues the first stages before waiting on that kernel
// -- every other cache row is unchanged since the previous step -- and the warp that
// owns the written row re-reads it from global memory into the staged tile after the
// wait.
#include "common.cuh"
#include "kvbp_internal.h"

namespace kvbp {

constexpr int kD = 128;
constexpr int kTile = 64;
#ifndef KVBP_ATTN_STAGES
#define KVBP_ATTN_STAGES 2
#endif
constexpr int kStages = KVBP_ATTN_STAGES;
// Consumer warps come in groups of four; group g takes tiles g, g + GR, ... (GR = 1 or
// 2, a template parameter).  Threads per CTA: 4 * GR warps + one TMA producer warp.
__host__ __device__ constexpr int attn_threads(int groups) { return 4 * groups * 32 + 32; }
constexpr int kMinBlocks = 2;  // two CTAs per SM: registers are capped to fit
constexpr int kHalfBytes = kTile * kD * 2;  // 16 KiB: K (or V) of one tile, two 64x64 boxes
constexpr int kBoxBytes = kHalfBytes / 2;
constexpr int kStageBytes = 2 * kHalfBytes;  // K tile + V tile
constexpr int kMaxCluster = 8;

struct AttnSmem {
  // byte offsets from the 1024-aligned base
  int logits, escr, spos, orecv, srecv, wstat, fin, bars, total;
};

__host__ __device__ inline int align_up(int x, int a) { return (x + a - 1) / a * a; }

__host__ __device__ inline AttnSmem attn_smem_layout(int nloc_tiles, int consumer_warps) {
  AttnSmem L;
  const int nloc = nloc_tiles * kTile;
  L.logits = kStages * kStageBytes;  // [nloc][8] rounded logits (bf16: they are bf16 values)
  L.escr = L.logits + nloc * 8 * 2;  // [warp][16 rows][8] softmax weights of the current tile
  L.spos = L.escr + consumer_warps * 16 * 8 * 4;
  L.orecv = align_up(L.spos + nloc * 4, 16);  // [CS][per] received O slices
  L.srecv = L.orecv + (8 * kD + kMaxCluster) * 4;  // [CS][16] received (max, sum)
  L.wstat = L.srecv + kMaxCluster * 16 * 4;  // [warp][16] per-warp (max, sum) + CTA (max, sum) + flags
  L.fin = align_up(L.wstat + (consumer_warps + 2) * 16 * 4, 16);  // final M[8], L[8], scale[cluster][8]
  L.bars = align_up(L.fin + (16 + kMaxCluster * 8) * 4, 8);
  L.total = L.bars + (2 * kStages + 1) * 8;
  // the [warp][8][128] partial outputs alias the ring at the end
  return L;
}

struct AttnArgs {
  const __nv_bfloat16* q;  // [B, Hq, D]
  const __nv_bfloat16* kc;  // [B, Hkv, S, D] (row re-reads after the wait)
  const __nv_bfloat16* vc;
  const int* slot_pos;     // [B, S]; < 0 = free slot
  const int* write_slot;   // [B] or null: see "Early streaming"
  __nv_bfloat16* out;      // [B, Hq, D]
  float* step_score;       // [B, S], non-negative; atomicMax target
  // per-KV-head retention (Ada-KV / QUEST faithful): slot s is visible to kv head h only
  // when head_keep[b][h][s] != 0 (null: every valid slot); head_score[b][r][s] receives the
  // max over calls of query head r's probability for r < Hkv (null: not kept)
  const uint8_t* head_keep;
  float* head_score;
  // fused scatter: this step's K/V row [B][Hkv][128] (null: already in the cache)
  const __nv_bfloat16* knew;
  const __nv_bfloat16* vnew;
  // fused score update (null upd_last: none): the last CTA to finish a sequence runs K2
  float* upd_attn;
  float* upd_maxa;
  double* upd_cumul;
  int* upd_last;
  int* upd_cnt;
  const int* seq_step;
  int* seq_counter;  // [B], zero between launches
  int* err;
  int B, Hq, Hkv, S;
  int tiles;       // ceil(S / 64)
  int cluster;     // CTAs per (sequence, kv head)
  int nloc_tiles;  // max tiles per CTA
  int ipc;         // kv heads per CTA (multi-item kernel; 1 otherwise)
  float scale;     // bfloat16(1/sqrt(D)) as float
};

// X: the heavier optional parts (per-head keep masks and scores, fused score update) are
// compiled in; the plain kernel (X = false) carries none of their code.  The fused scatter
// (knew / vnew) is a runtime branch of both.
template <int G, int GR, bool X>
__global__ void __launch_bounds__(attn_threads(GR), kMinBlocks) decode_attn_score_kernel(const __grid_constant__ CUtensorMap kmap,
                                                                     const __grid_constant__ CUtensorMap vmap,
                                                                     const AttnArgs p) {
  constexpr int kConsumerWarps = 4 * GR;
  constexpr int kConsumers = kConsumerWarps * 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const AttnSmem L = attn_smem_layout(p.nloc_tiles, kConsumerWarps);
  uint8_t* ring = base;
  __nv_bfloat16* logits = reinterpret_cast<__nv_bfloat16*>(base + L.logits);
  float* escr = reinterpret_cast<float*>(base + L.escr);
  int* spos_s = reinterpret_cast<int*>(base + L.spos);
  float* orecv = reinterpret_cast<float*>(base + L.orecv);
  float* srecv = reinterpret_cast<float*>(base + L.srecv);
  float* wstat = reinterpret_cast<float*>(base + L.wstat);  // [warp][m 8 | l 8]
  float* cstat = wstat + kConsumerWarps * 16;                // CTA m[8], l[8]
  int* flags = reinterpret_cast<int*>(cstat + 16);           // [0] bad, [1] issued
  int* bad_flag = flags;
  int* n_issued = flags + 1;
  float* opart = reinterpret_cast<float*>(base);  // [warp][8][128], aliases the ring
  uint64_t* full = reinterpret_cast<uint64_t*>(base + L.bars);
  uint64_t* empty = full + kStages;
  uint64_t* xbar = empty + kStages;

  const int CS = p.cluster;
  uint32_t rank_u;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank_u));
  const int rank = static_cast<int>(rank_u);
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = (rank * p.tiles) / CS, t1 = ((rank + 1) * p.tiles) / CS;
  const int nt = t1 - t0, nloc = nt * kTile;
  const int S = p.S;
  const int per = (G * kD + CS - 1) / CS;  // output slice per CTA
  const int n_mine = (rank * per < G * kD) ? ((rank * per + per < G * kD) ? per : G * kD - rank * per) : 0;
  const float NEG_INF = -__int_as_float(0x7f800000);

  // [pair][slot][128] view: rows past S are out of bounds and arrive as zeros without
  // touching memory, so the last tile of a pair costs no extra HBM traffic
  const int pair = b * p.Hkv + kvh;
  auto issue = [&](int u) {
    const int st = u % kStages;
    uint8_t* dst = ring + st * kStageBytes;
    const int y = (t0 + u) * kTile;
    mbar_expect_tx(&full[st], kStageBytes);
    tma_load_3d(dst, &kmap, &full[st], 0, y, pair);
    tma_load_3d(dst + kBoxBytes, &kmap, &full[st], 64, y, pair);
    tma_load_3d(dst + kHalfBytes, &vmap, &full[st], 0, y, pair);
    tma_load_3d(dst + kHalfBytes + kBoxBytes, &vmap, &full[st], 64, y, pair);
  };
  const int n_first = nt < kStages ? nt : kStages;
  const bool early = p.write_slot != nullptr;
  if (tid == kConsumers) {
    prefetch_tmap(&kmap);
    prefetch_tmap(&vmap);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);  // the four warps of the group that consumes the tile
    }
    mbar_init(xbar, 1);
    *bad_flag = 0;
    *n_issued = 0;
    fence_barrier_init();
  }
  __syncthreads();
  // every peer's barriers must be initialised before any st.async: arrive now, wait just
  // before the exchange, so the tile loop does not wait for the slowest CTA's setup
  cluster_arrive_release();
  if (!KVBP_PDL_LATE) pdl_launch_dependents();

  // ================================ producer warp =================================
  // (the first TMA issue of a launch can stall its thread for microseconds, so no other
  // thread waits for it)
  if (warp == kConsumerWarps) {
    if (lane == 0) {
      if (early) {  // all rows but write_slot's are final: stream before the wait
        for (int u = 0; u < n_first; ++u) issue(u);
        *n_issued = n_first;
      }
      pdl_wait();  // the slot positions and this step's K/V row come from earlier kernels
      if (!early) {
        for (int u = 0; u < n_first; ++u) issue(u);
        *n_issued = n_first;
      }
      for (int u = n_first; u < nt; ++u) {
        const int st = u % kStages;
        if (*reinterpret_cast<volatile int*>(bad_flag)) break;
        if (!mbar_wait_bounded(&empty[st], ((u / kStages) - 1) & 1)) {
          set_err(p.err, kErrWaitTimeout);
          atomicExch(bad_flag, 1);
          break;
        }
        if (*reinterpret_cast<volatile int*>(bad_flag)) break;
        issue(u);
        *reinterpret_cast<volatile int*>(n_issued) = u + 1;
      }
      if (*reinterpret_cast<volatile int*>(bad_flag)) {
        // error path: let the loads still in flight (the last one of each stage) land
        // before this CTA can exit
        const int ni = *reinterpret_cast<volatile int*>(n_issued);
        for (int u = (ni > kStages ? ni - kStages : 0); u < ni; ++u)
          mbar_wait_bounded(&full[u % kStages], (u / kStages) & 1, 1u << 16);
      }
    }
    __syncwarp();
    if (KVBP_PDL_LATE) pdl_launch_dependents();
    cluster_wait_acquire();  // the setup phase (the consumers wait before their exchange)
    cluster_sync_all();      // matches the consumers' final cluster barrier
    if (X && p.upd_last) cluster_sync_all();  // and the fused score update's flag exchange
    return;
  }

  // ================================ consumer warps ================================
  pdl_wait();  // q, the slot positions and this step's K/V row come from earlier kernels
  if (tid == 0) mbar_expect_tx(xbar, CS * (16 + n_mine) * 4);  // local arrival; completes on the bytes
  const int g = lane >> 2, t = lane & 3;
  uint32_t qb[8][2];
  {
    const uint32_t* qrow = reinterpret_cast<const uint32_t*>(
        p.q + (static_cast<size_t>(b) * p.Hq + kvh * G + (g < G ? g : 0)) * kD);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      qb[kk][0] = g < G ? qrow[(kk * 16 + 2 * t) >> 1] : 0u;
      qb[kk][1] = g < G ? qrow[(kk * 16 + 8 + 2 * t) >> 1] : 0u;
    }
  }
  const bool h0_ok = 2 * t < G, h1_ok = 2 * t + 1 < G;
  float m0 = NEG_INF, m1 = NEG_INF;  // running max of heads 2t, 2t+1 over this warp's rows
  float l0 = 0.f, l1 = 0.f;          // this lane's share of the running sums
  float oacc[8][4];
#pragma unroll
  for (int m = 0; m < 8; ++m) oacc[m][0] = oacc[m][1] = oacc[m][2] = oacc[m][3] = 0.f;
  float* ew = escr + warp * 16 * 8;
  const int r0 = (warp & 3) * 16;  // the warp's 16 slots of each tile its group takes
  const int grp = warp >> 2;
  const int wslot = early ? p.write_slot[b] : -1;  // row of this step's K/V (read after the wait)

  const int* spos_g = p.slot_pos + static_cast<size_t>(b) * S;
  // slot positions of the warp's rows g and g + 8 of a tile (< 0: free slot), read one
  // tile of the group ahead so that their latency overlaps the previous tile's math;
  // lanes t == 0 keep them for the score pass
  auto slot_of = [&](int uu, int r) { return t0 * kTile + uu * kTile + r0 + g + r < S ? spos_g[t0 * kTile + uu * kTile + r0 + g + r] : -1; };
  int pa_next = grp < nt ? slot_of(grp, 0) : -1, pb_next = grp < nt ? slot_of(grp, 8) : -1;
  for (int u = grp; u < nt; u += GR) {
    const int st = u % kStages;
    const int lta = u * kTile + r0 + g, ltb = lta + 8;
    int pa = pa_next, pb = pb_next;
    if (u + GR < nt) {
      pa_next = slot_of(u + GR, 0);
      pb_next = slot_of(u + GR, 8);
    }
    if (X && p.head_keep) {  // a slot this kv head does not retain counts as free for it
      const uint8_t* hk = p.head_keep + static_cast<size_t>(pair) * S + t0 * kTile;
      if (pa >= 0 && !hk[lta]) pa = -1;
      if (pb >= 0 && !hk[ltb]) pb = -1;
    }
    bool ok_tile = !(*reinterpret_cast<volatile int*>(bad_flag));
    if (ok_tile && !mbar_wait_bounded(&full[st], (u / kStages) & 1)) {
      set_err(p.err, kErrWaitTimeout);
      atomicExch(bad_flag, 1);
      ok_tile = false;
    }
    ok_tile = __all_sync(0xffffffffu, ok_tile);  // warp-uniform: the tile's mma/ldmatrix are warp-wide
    if (ok_tile && (u < n_first || p.knew) && wslot >= 0 && wslot < S) {
      // a tile staged before the wait may hold a stale copy of this step's row (and with a
      // fused scatter every tile may): the warp that owns the row (rows r0..r0+15 of the
      // tile) writes it into the staged tile, K by lanes 0-15 and V by lanes 16-31, one
      // 16-byte chunk each, at the 128-byte-swizzled position -- from the cache, or from
      // knew/vnew, which it also stores into the cache for the next steps
      const int lr = wslot - (t0 + u) * kTile;
      if (lr >= r0 && lr < r0 + 16) {
        const int half = lane >> 4, ch = lane & 15, box = ch >> 3, c = ch & 7;
        __nv_bfloat16* crow = const_cast<__nv_bfloat16*>(half ? p.vc : p.kc) + (static_cast<size_t>(pair) * S + wslot) * kD + ch * 8;
        uint4 v;
        if (p.knew) {
          v = __ldg(reinterpret_cast<const uint4*>((half ? p.vnew : p.knew) + static_cast<size_t>(pair) * kD + ch * 8));
          *reinterpret_cast<uint4*>(crow) = v;
        } else {
          v = __ldcg(reinterpret_cast<const uint4*>(crow));
        }
        uint8_t* dst = ring + st * kStageBytes + half * kHalfBytes + box * kBoxBytes + lr * 128 + ((c ^ (lr & 7)) << 4);
        *reinterpret_cast<uint4*>(dst) = v;
        fence_proxy_async_smem();  // the stage is refilled by TMA later
        __syncwarp();
      }
    }
    if (ok_tile) {
      const uint8_t* kt = ring + st * kStageBytes;
      const uint8_t* vt = kt + kHalfBytes;
      // ---- Q.K^T for rows r0..r0+15 (two independent mma chains) -------------------
      float a0c[4] = {0.f, 0.f, 0.f, 0.f}, a1c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int col = kk * 16;
        const int box = col >> 6, cb = (col & 63) >> 3;
        const int j = lane >> 3;
        const int row = r0 + (lane & 7) + ((j & 1) << 3);
        const int chunk = cb + (j >> 1);
        uint32_t x0, x1, x2, x3;
        ldmatrix_x4(smem_u32(kt + box * kBoxBytes + row * 128 + ((chunk ^ (row & 7)) << 4)), x0, x1, x2, x3);
        if (kk & 1)
          mma_bf16_16816(a1c, x0, x1, x2, x3, qb[kk][0], qb[kk][1]);
        else
          mma_bf16_16816(a0c, x0, x1, x2, x3, qb[kk][0], qb[kk][1]);
      }
      // ---- rounded logits (reference rounding points) -> shared memory ---------------
      const bool va = pa >= 0, vb = pb >= 0;
      if (t == 0) {
        spos_s[lta] = pa;
        spos_s[ltb] = pb;
      }
      float sa0 = va ? bf16r(bf16r(a0c[0] + a1c[0]) * p.scale) : NEG_INF;
      float sa1 = va ? bf16r(bf16r(a0c[1] + a1c[1]) * p.scale) : NEG_INF;
      float sb0 = vb ? bf16r(bf16r(a0c[2] + a1c[2]) * p.scale) : NEG_INF;
      float sb1 = vb ? bf16r(bf16r(a0c[3] + a1c[3]) * p.scale) : NEG_INF;
      *reinterpret_cast<uint32_t*>(&logits[lta * 8 + 2 * t]) = pack_bf16(sa0, sa1);  // exact: bf16 values
      *reinterpret_cast<uint32_t*>(&logits[ltb * 8 + 2 * t]) = pack_bf16(sb0, sb1);
      // ---- online softmax over the warp's 16 rows -----------------------------------
      float tm0 = fmaxf(sa0, sb0), tm1 = fmaxf(sa1, sb1);
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        tm0 = fmaxf(tm0, __shfl_xor_sync(0xffffffffu, tm0, o));
        tm1 = fmaxf(tm1, __shfl_xor_sync(0xffffffffu, tm1, o));
      }
      const float n0 = fmaxf(m0, tm0), n1 = fmaxf(m1, tm1);
      const float al0 = (m0 == NEG_INF) ? 1.f : expf(m0 - n0);
      const float al1 = (m1 == NEG_INF) ? 1.f : expf(m1 - n1);
      m0 = n0;
      m1 = n1;
      const float ea0 = (va && h0_ok) ? expf(sa0 - n0) : 0.f;
      const float ea1 = (va && h1_ok) ? expf(sa1 - n1) : 0.f;
      const float eb0 = (vb && h0_ok) ? expf(sb0 - n0) : 0.f;
      const float eb1 = (vb && h1_ok) ? expf(sb1 - n1) : 0.f;
      l0 = l0 * al0 + ea0 + eb0;
      l1 = l1 * al1 + ea1 + eb1;
      if (__any_sync(0xffffffffu, al0 != 1.f || al1 != 1.f)) {
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          oacc[m][0] *= al0;
          oacc[m][1] *= al1;
          oacc[m][2] *= al0;
          oacc[m][3] *= al1;
        }
      }
      *reinterpret_cast<float2*>(&ew[g * 8 + 2 * t]) = make_float2(ea0, ea1);
      *reinterpret_cast<float2*>(&ew[(g + 8) * 8 + 2 * t]) = make_float2(eb0, eb1);
      __syncwarp();
      if (__any_sync(0xffffffffu, va || vb)) {
        // ---- P.V: O^T (dims x heads) += V^T (dims x slots) * P^T (slots x heads) --------
        const float p0 = ew[(2 * t) * 8 + g], p1 = ew[(2 * t + 1) * 8 + g];
        const float p2 = ew[(2 * t + 8) * 8 + g], p3 = ew[(2 * t + 9) * 8 + g];
        const float h0 = bf16r(p0), h1 = bf16r(p1), h2 = bf16r(p2), h3 = bf16r(p3);
        const uint32_t bh0 = pack_bf16(h0, h1), bh1 = pack_bf16(h2, h3);
        const uint32_t bl0 = pack_bf16(p0 - h0, p1 - h1), bl1 = pack_bf16(p2 - h2, p3 - h3);
        const int slot = r0 + (lane & 7) + ((lane >> 4) << 3);
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          const int dchunk = m * 16 + (((lane >> 3) & 1) << 3);
          const int box = dchunk >> 6, c = (dchunk & 63) >> 3;
          uint32_t x0, x1, x2, x3;
          ldmatrix_x4_trans(smem_u32(vt + box * kBoxBytes + slot * 128 + ((c ^ (slot & 7)) << 4)), x0, x1, x2, x3);
          mma_bf16_16816(oacc[m], x0, x1, x2, x3, bh0, bh1);
          mma_bf16_16816(oacc[m], x0, x1, x2, x3, bl0, bl1);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }
  if (KVBP_PDL_LATE) pdl_launch_dependents();

  // ---- merge the warps: per-head (max, sum), then the partial outputs ---------------
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, o);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o);
  }
  if (lane < 4) {
    wstat[warp * 16 + 2 * lane] = m0;
    wstat[warp * 16 + 2 * lane + 1] = m1;
    wstat[warp * 16 + 8 + 2 * lane] = l0;
    wstat[warp * 16 + 8 + 2 * lane + 1] = l1;
  }
  named_bar(1, kConsumers);  // also: every tile consumed, the ring is free for the partials
  if (tid < 8) {
    float mc = NEG_INF;
    for (int w = 0; w < kConsumerWarps; ++w) mc = fmaxf(mc, wstat[w * 16 + tid]);
    float lc = 0.f;
    for (int w = 0; w < kConsumerWarps; ++w) {
      const float mw = wstat[w * 16 + tid];
      if (mw != NEG_INF) lc += wstat[w * 16 + 8 + tid] * expf(mw - mc);
    }
    cstat[tid] = mc;
    cstat[8 + tid] = lc;
  }
  {
    // scale this warp's partial to the CTA max; heads >= G never leave the warp
    const float mw0 = __shfl_sync(0xffffffffu, m0, t), mw1 = __shfl_sync(0xffffffffu, m1, t);
    float mc0 = NEG_INF, mc1 = NEG_INF;
    for (int w = 0; w < kConsumerWarps; ++w) {
      mc0 = fmaxf(mc0, wstat[w * 16 + 2 * t]);
      mc1 = fmaxf(mc1, wstat[w * 16 + 2 * t + 1]);
    }
    const float s0 = (mw0 == NEG_INF) ? 0.f : expf(mw0 - mc0);
    const float s1 = (mw1 == NEG_INF) ? 0.f : expf(mw1 - mc1);
    float* ow = opart + warp * 8 * kD;
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      if (h0_ok) {
        ow[(2 * t) * kD + 16 * m + g] = oacc[m][0] * s0;
        ow[(2 * t) * kD + 16 * m + g + 8] = oacc[m][2] * s0;
      }
      if (h1_ok) {
        ow[(2 * t + 1) * kD + 16 * m + g] = oacc[m][1] * s1;
        ow[(2 * t + 1) * kD + 16 * m + g + 8] = oacc[m][3] * s1;
      }
    }
  }
  named_bar(1, kConsumers);
  cluster_wait_acquire();  // every peer is past its setup (barriers initialised)
  // ---- one st.async round: (max, sum) to every peer, O element e to CTA e / per ------
  if (warp == 0 && lane < CS) {
    const uint32_t rbar = mapa_u32(smem_u32(xbar), lane);
    const uint32_t rdst = mapa_u32(smem_u32(srecv + rank * 16), lane);
    for (int h = 0; h < 16; ++h) st_async_f32(rdst + 4 * h, cstat[h], rbar);
  }
  if (per % 4 == 0) {  // 16-byte pieces never straddle two CTAs' slices
    for (int e = 4 * tid; e < G * kD; e += 4 * kConsumers) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        const float4 v = *reinterpret_cast<const float4*>(&opart[w * 8 * kD + e]);
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      const int r = e / per;
      st_async_v4(mapa_u32(smem_u32(orecv + rank * per + (e - r * per)), r), acc, mapa_u32(smem_u32(xbar), r));
    }
  } else {
    for (int e = tid; e < G * kD; e += kConsumers) {
      float acc = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) acc += opart[w * 8 * kD + e];
      const int r = e / per;
      st_async_f32(mapa_u32(smem_u32(orecv + rank * per + (e - r * per)), r), acc, mapa_u32(smem_u32(xbar), r));
    }
  }
  if (!mbar_wait_cluster_bounded(xbar, 0)) {
    set_err(p.err, kErrWaitTimeout);
    atomicExch(bad_flag, 1);
  }
  // ---- final max M and sum L per head (identical in every CTA of the cluster) ------
  // thread h of the first warp forms head h's M, L and each CTA's rescale exp(m_c - M)
  float* finM = reinterpret_cast<float*>(base + L.fin);
  float* finL = finM + 8;
  float* fscale = finL + 8;  // [c][8]
  if (tid < G) {
    const int h = tid;
    float M = NEG_INF;
    for (int c = 0; c < CS; ++c) M = fmaxf(M, srecv[c * 16 + h]);
    float Ls = 0.f;
    for (int c = 0; c < CS; ++c) {
      const float mc = srecv[c * 16 + h];
      const float f = (mc != NEG_INF) ? expf(mc - M) : 0.f;
      fscale[c * 8 + h] = f;
      if (mc != NEG_INF) Ls += srecv[c * 16 + 8 + h] * f;
    }
    finM[h] = M;
    finL[h] = Ls;
    if (rank == 0 && !(Ls > 0.f)) set_err(p.err, kErrNoValidSlot);
  }
  named_bar(1, kConsumers);
  // output slice
  {
    const int e0 = rank * per;
    __nv_bfloat16* orow = p.out + (static_cast<size_t>(b) * p.Hq + kvh * G) * kD;
    for (int j = tid; j < n_mine; j += kConsumers) {
      const int h = (e0 + j) / kD;
      float acc = 0.f;
      for (int c = 0; c < CS; ++c) {
        if (srecv[c * 16 + h] != NEG_INF) acc += orecv[c * per + j] * fscale[c * 8 + h];
      }
      const float Lh = finL[h];
      orow[e0 + j] = __float2bfloat16_rn(Lh > 0.f ? acc / Lh : 0.f);
    }
  }
  // per-slot eviction score: max over the group's heads of p = exp(s - M) * (1 / L)
  if (!(*reinterpret_cast<volatile int*>(bad_flag))) {
    float Mh[G], iLh[G];  // max and 1 / sum per head (0 for a head without valid slots)
#pragma unroll
    for (int h = 0; h < G; ++h) {
      Mh[h] = finM[h];
      iLh[h] = finL[h] > 0.f ? 1.0f / finL[h] : 0.f;
    }
    float* sscore = p.step_score + static_cast<size_t>(b) * S;
    if (!X || !p.head_score) {
      for (int i = tid; i < nloc; i += kConsumers) {
        if (spos_s[i] < 0) continue;
        float mx = 0.f;
#pragma unroll
        for (int h = 0; h < G; ++h) {
          const float pr = iLh[h] > 0.f ? expf(__bfloat162float(logits[i * 8 + h]) - Mh[h]) * iLh[h] : 0.f;
          mx = fmaxf(mx, pr);
        }
        if (mx != mx) set_err(p.err, kErrNanScore);
        atomicMax(reinterpret_cast<int*>(&sscore[t0 * kTile + i]), __float_as_int(mx));
      }
    } else {
      // query heads kvh * G + h below Hkv also feed the per-head signal rows
      float* hrow = p.head_score + (static_cast<size_t>(b) * p.Hkv + kvh * G) * S;
      for (int i = tid; i < nloc; i += kConsumers) {
        if (spos_s[i] < 0) continue;
        float mx = 0.f;
#pragma unroll
        for (int h = 0; h < G; ++h) {
          const float pr = iLh[h] > 0.f ? expf(__bfloat162float(logits[i * 8 + h]) - Mh[h]) * iLh[h] : 0.f;
          mx = fmaxf(mx, pr);
          if (kvh * G + h < p.Hkv)
            atomicMax(reinterpret_cast<int*>(&hrow[static_cast<size_t>(h) * S + t0 * kTile + i]), __float_as_int(pr));
        }
        if (mx != mx) set_err(p.err, kErrNanScore);
        atomicMax(reinterpret_cast<int*>(&sscore[t0 * kTile + i]), __float_as_int(mx));
      }
    }
  }
  int* last_flag = flags + 2;
  if (X && p.upd_last) {
    // fused score update (kv_coupled_generator.py:504-516): the sequence's CTAs (every kv
    // head, every cluster rank) count themselves in; the cluster holding the last arrival
    // updates every slot of the sequence, split over its CTAs
    __threadfence();  // this CTA's score maxima are visible before it counts itself
    named_bar(1, kConsumers);
    if (tid == 0) *last_flag = atomicAdd(&p.seq_counter[b], 1) == static_cast<int>(gridDim.x * gridDim.y) - 1;
  }
  __syncwarp();
  cluster_sync_all();  // no CTA leaves while a peer may still target its shared memory
  if (X && p.upd_last) {
    int* any_last = flags + 3;
    if (tid == 0) {
      int a = 0;
      for (int q = 0; q < CS; ++q) a |= __float_as_int(ld_dsmem_f32(mapa_u32(smem_u32(last_flag), q)));
      *any_last = a;
    }
    named_bar(1, kConsumers);
    const bool mine = *any_last != 0;
    cluster_sync_all();  // every peer has read this CTA's flag
    if (mine) {
      __threadfence();
      constexpr int kU = 4;  // slots per thread with their loads in flight together
      const size_t o0 = static_cast<size_t>(b) * S;
      const float* scr = p.step_score + o0;
      float mx = 0.f;
      for (int i0 = tid; i0 < S; i0 += kU * kConsumers) {
        float v[kU];
        int ps[kU];
#pragma unroll
        for (int k = 0; k < kU; ++k) {
          const int i = i0 + k * kConsumers;
          v[k] = i < S ? __ldcg(&scr[i]) : 0.f;
          ps[k] = i < S ? spos_g[i] : -1;
        }
#pragma unroll
        for (int k = 0; k < kU; ++k)
          if (ps[k] >= 0) mx = fmaxf(mx, v[k]);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      if (lane == 0) escr[warp] = mx;
      named_bar(1, kConsumers);
      float gmx = 0.f;
      for (int w = 0; w < kConsumerWarps; ++w) gmx = fmaxf(gmx, escr[w]);
      const float thr = static_cast<float>(0.05 * static_cast<double>(gmx));
      const int step = p.seq_step[b];
      const int lo = (rank * S) / CS, hi = ((rank + 1) * S) / CS;
      float* scw = p.step_score + o0;
      for (int i0 = lo + tid; i0 < hi; i0 += kU * kConsumers) {
        float ks[kU], ma[kU];
        double cu[kU];
        int ps[kU], cn[kU];
#pragma unroll
        for (int k = 0; k < kU; ++k) {
          const int i = i0 + k * kConsumers;
          const bool in = i < hi;
          ps[k] = in ? spos_g[i] : -1;
          ks[k] = in ? __ldcg(&scw[i]) : 0.f;
          ma[k] = in ? p.upd_maxa[o0 + i] : 0.f;
          cu[k] = in ? p.upd_cumul[o0 + i] : 0.0;
          cn[k] = in ? p.upd_cnt[o0 + i] : 0;
        }
#pragma unroll
        for (int k = 0; k < kU; ++k) {
          const int i = i0 + k * kConsumers;
          if (i >= hi) continue;
          if (ps[k] >= 0) {
            if (ks[k] != ks[k]) set_err(p.err, kErrNanScore);
            p.upd_attn[o0 + i] = ks[k];
            p.upd_maxa[o0 + i] = fmaxf(ma[k], ks[k]);
            p.upd_cumul[o0 + i] = __dadd_rn(cu[k], static_cast<double>(ks[k]));
            if (ks[k] > thr) {
              p.upd_last[o0 + i] = step;
              p.upd_cnt[o0 + i] = cn[k] + 1;
            }
          }
          scw[i] = 0.f;
        }
      }
      if (tid == 0 && *last_flag) p.seq_counter[b] = 0;
    }
  }
}

// ------------------------------------------------------------------------------------
// Persistent variant for launches with more (sequence, kv head) pairs than one wave of two
// CTAs per SM holds.  One CTA per pair would run in waves, and every CTA's set-up,
// exchange and epilogue would stall its share of the stream at the same moment; here a
// single wave of clusters (CS CTAs each, CS * clusters <= 2 per SM) walks the pairs
// round-robin -- cluster c takes pairs c, c + clusters, ... -- and each CTA's producer
// streams its tiles of the next pair through the same ring while the consumer warps
// finish the previous pair's merge, exchange, output and per-slot score.  Per pair the
// arithmetic is the cluster kernel's (same tile split, merge order and exchange), so the
// results are bit-identical to it.  Partial outputs get their own shared memory (the ring
// is busy with the next pair), logits and partials are HP = 4 heads wide for groups of at
// most 4 query heads.  Cluster barriers: every thread arrives once after set-up and once
// after reading each pair's exchange, and waits once before each pair's exchange and once
// at exit, so a peer's next pushes never overwrite data still being read.
// ------------------------------------------------------------------------------------
struct PersistSmem {
  int opart, logits, escr, spos, orecv, srecv, wstat, fin, bars, total;
};

__host__ __device__ inline PersistSmem persist_smem_layout(int nloc_tiles, int consumer_warps, int hp) {
  PersistSmem L;
  const int nloc = nloc_tiles * kTile;
  L.opart = kStages * kStageBytes;                    // [warp][hp][128] partial outputs
  L.logits = L.opart + consumer_warps * hp * kD * 4;  // [nloc][hp] rounded logits (bf16 values)
  L.escr = L.logits + nloc * hp * 2;                  // [warp][16][8] softmax weights of a tile
  L.spos = L.escr + consumer_warps * 16 * 8 * 4;      // [nloc] slot positions
  L.orecv = align_up(L.spos + nloc * 4, 16);          // received O slices
  L.srecv = L.orecv + (8 * kD + kMaxCluster) * 4;     // [CS][16] received (max, sum)
  L.wstat = L.srecv + kMaxCluster * 16 * 4;           // [warp][16] + CTA (max, sum) + flags
  L.fin = align_up(L.wstat + (consumer_warps + 2) * 16 * 4, 16);  // M[8], L[8], scale[cluster][8]
  L.bars = align_up(L.fin + (16 + kMaxCluster * 8) * 4, 8);
  L.total = L.bars + (2 * kStages + 1) * 8;
  return L;
}

template <int G, int GR>
__global__ void __launch_bounds__(attn_threads(GR), kMinBlocks) decode_attn_persist_kernel(
    const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, const AttnArgs p) {
  constexpr int kConsumerWarps = 4 * GR;
  constexpr int kConsumers = kConsumerWarps * 32;
  constexpr int HP = G <= 4 ? 4 : 8;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const PersistSmem L = persist_smem_layout(p.nloc_tiles, kConsumerWarps, HP);
  uint8_t* ring = base;
  float* opart = reinterpret_cast<float*>(base + L.opart);
  __nv_bfloat16* logits = reinterpret_cast<__nv_bfloat16*>(base + L.logits);
  float* escr = reinterpret_cast<float*>(base + L.escr);
  int* spos_s = reinterpret_cast<int*>(base + L.spos);
  float* orecv = reinterpret_cast<float*>(base + L.orecv);
  float* srecv = reinterpret_cast<float*>(base + L.srecv);
  float* wstat = reinterpret_cast<float*>(base + L.wstat);
  float* cstat = wstat + kConsumerWarps * 16;
  int* flags = reinterpret_cast<int*>(cstat + 16);
  int* bad_flag = flags;
  int* n_issued = flags + 1;
  float* finM = reinterpret_cast<float*>(base + L.fin);
  float* finL = finM + 8;
  float* fscale = finL + 8;  // [c][8]
  uint64_t* full = reinterpret_cast<uint64_t*>(base + L.bars);
  uint64_t* empty = full + kStages;
  uint64_t* xbar = empty + kStages;

  const int CS = p.cluster;
  uint32_t rank_u = 0;
  if (CS > 1) asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank_u));
  const int rank = static_cast<int>(rank_u);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = (rank * p.tiles) / CS, t1 = ((rank + 1) * p.tiles) / CS;
  const int nt = t1 - t0, nloc = nt * kTile;
  const int S = p.S;
  const int n_pairs_all = p.B * p.Hkv, n_cl = gridDim.y, c0 = blockIdx.y;
  const int npairs = c0 < n_pairs_all ? (n_pairs_all - c0 + n_cl - 1) / n_cl : 0;
  const int total = npairs * nt;  // tiles this CTA streams, pair after pair
  const int n_first = total < kStages ? total : kStages;
  const int per = (G * kD + CS - 1) / CS;
  const int n_mine = (rank * per < G * kD) ? ((rank * per + per < G * kD) ? per : G * kD - rank * per) : 0;
  const float NEG_INF = -__int_as_float(0x7f800000);
  const bool early = p.write_slot != nullptr;

  auto issue = [&](int gi) {
    const int j = gi / nt, u = gi - j * nt;
    const int st = gi % kStages;
    uint8_t* dst = ring + st * kStageBytes;
    const int y = (t0 + u) * kTile, pair = c0 + j * n_cl;
    mbar_expect_tx(&full[st], kStageBytes);
    tma_load_3d(dst, &kmap, &full[st], 0, y, pair);
    tma_load_3d(dst + kBoxBytes, &kmap, &full[st], 64, y, pair);
    tma_load_3d(dst + kHalfBytes, &vmap, &full[st], 0, y, pair);
    tma_load_3d(dst + kHalfBytes + kBoxBytes, &vmap, &full[st], 64, y, pair);
  };
  if (tid == kConsumers) {
    prefetch_tmap(&kmap);
    prefetch_tmap(&vmap);
    for (int s2 = 0; s2 < kStages; ++s2) {
      mbar_init(&full[s2], 1);
      mbar_init(&empty[s2], 4);  // the four warps of the group that consumes the tile
    }
    mbar_init(xbar, 1);
    *bad_flag = 0;
    *n_issued = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (CS > 1) cluster_arrive_release();  // every peer's barriers are initialised before any push
  if (!KVBP_PDL_LATE) pdl_launch_dependents();

  // ================================ producer warp =================================
  if (warp == kConsumerWarps) {
    if (lane == 0) {
      if (early) {  // all rows but write_slot's are final: stream before the wait
        for (int gi = 0; gi < n_first; ++gi) issue(gi);
        *n_issued = n_first;
      }
      pdl_wait();
      if (!early) {
        for (int gi = 0; gi < n_first; ++gi) issue(gi);
        *n_issued = n_first;
      }
    }
    for (int j = 0; j < npairs; ++j) {
      if (lane == 0) {
        const int g_end = (j + 1) * nt;
        for (int gi = (j * nt > n_first ? j * nt : n_first); gi < g_end; ++gi) {
          const int st = gi % kStages;
          if (*reinterpret_cast<volatile int*>(bad_flag)) break;
          if (!mbar_wait_bounded(&empty[st], ((gi / kStages) - 1) & 1)) {
            set_err(p.err, kErrWaitTimeout);
            atomicExch(bad_flag, 1);
            break;
          }
          if (*reinterpret_cast<volatile int*>(bad_flag)) break;
          issue(gi);
          *reinterpret_cast<volatile int*>(n_issued) = gi + 1;
        }
      }
      __syncwarp();
      if (CS > 1) {  // the consumers' wait before this pair's exchange and arrival after it
        cluster_wait_acquire();
        cluster_arrive_release();
      }
    }
    if (lane == 0 && *reinterpret_cast<volatile int*>(bad_flag)) {
      const int ni = *reinterpret_cast<volatile int*>(n_issued);
      for (int u = (ni > kStages ? ni - kStages : 0); u < ni; ++u)
        mbar_wait_bounded(&full[u % kStages], (u / kStages) & 1, 1u << 16);
    }
    __syncwarp();
    if (KVBP_PDL_LATE) pdl_launch_dependents();
    if (CS > 1) cluster_wait_acquire();  // matches the consumers' exit wait
    return;
  }

  // ================================ consumer warps ================================
  pdl_wait();  // q, the slot positions and this step's K/V row come from earlier kernels
  const int g = lane >> 2, t = lane & 3;
  const bool h0_ok = 2 * t < G, h1_ok = 2 * t + 1 < G;
  float* ew = escr + warp * 16 * 8;
  const int r0 = (warp & 3) * 16;
  const int grp = warp >> 2;

  for (int j = 0; j < npairs; ++j) {
    const int pair = c0 + j * n_cl;
    const int b = pair / p.Hkv, kvh = pair - b * p.Hkv;
    const int wslot = early ? p.write_slot[b] : -1;
    const int* spos_g = p.slot_pos + static_cast<size_t>(b) * S;
    if (CS > 1 && tid == 0) mbar_expect_tx(xbar, CS * (16 + n_mine) * 4);  // this pair's exchange
    uint32_t qb[8][2];
    {
      const uint32_t* qrow = reinterpret_cast<const uint32_t*>(
          p.q + (static_cast<size_t>(b) * p.Hq + kvh * G + (g < G ? g : 0)) * kD);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        qb[kk][0] = g < G ? qrow[(kk * 16 + 2 * t) >> 1] : 0u;
        qb[kk][1] = g < G ? qrow[(kk * 16 + 8 + 2 * t) >> 1] : 0u;
      }
    }
    float m0 = NEG_INF, m1 = NEG_INF;
    float l0 = 0.f, l1 = 0.f;
    float oacc[8][4];
#pragma unroll
    for (int m = 0; m < 8; ++m) oacc[m][0] = oacc[m][1] = oacc[m][2] = oacc[m][3] = 0.f;

    // slot positions read one tile of the group ahead (their latency overlaps the math)
    auto slot_of = [&](int uu, int r) { return t0 * kTile + uu * kTile + r0 + g + r < S ? spos_g[t0 * kTile + uu * kTile + r0 + g + r] : -1; };
    int pa_next = grp < nt ? slot_of(grp, 0) : -1, pb_next = grp < nt ? slot_of(grp, 8) : -1;
    for (int u = grp; u < nt; u += GR) {
      const int gi = j * nt + u;
      const int st = gi % kStages;
      const int lta = u * kTile + r0 + g, ltb = lta + 8;  // local slot index within this CTA's range
      const int pa = pa_next, pb = pb_next;
      if (u + GR < nt) {
        pa_next = slot_of(u + GR, 0);
        pb_next = slot_of(u + GR, 8);
      }
      bool ok_tile = !(*reinterpret_cast<volatile int*>(bad_flag));
      if (ok_tile && !mbar_wait_bounded(&full[st], (gi / kStages) & 1)) {
        set_err(p.err, kErrWaitTimeout);
        atomicExch(bad_flag, 1);
        ok_tile = false;
      }
      ok_tile = __all_sync(0xffffffffu, ok_tile);
      if (ok_tile && (gi < n_first || p.knew) && wslot >= 0 && wslot < S) {
        // this step's row: re-read for tiles staged before the wait, or taken from
        // knew / vnew (and stored into the cache) -- as in the cluster kernel
        const int lr = wslot - (t0 + u) * kTile;
        if (lr >= r0 && lr < r0 + 16) {
          const int half = lane >> 4, ch = lane & 15, box = ch >> 3, c = ch & 7;
          __nv_bfloat16* crow =
              const_cast<__nv_bfloat16*>(half ? p.vc : p.kc) + (static_cast<size_t>(pair) * S + wslot) * kD + ch * 8;
          uint4 v;
          if (p.knew) {
            v = __ldg(reinterpret_cast<const uint4*>((half ? p.vnew : p.knew) + static_cast<size_t>(pair) * kD + ch * 8));
            *reinterpret_cast<uint4*>(crow) = v;
          } else {
            v = __ldcg(reinterpret_cast<const uint4*>(crow));
          }
          uint8_t* dst = ring + st * kStageBytes + half * kHalfBytes + box * kBoxBytes + lr * 128 + ((c ^ (lr & 7)) << 4);
          *reinterpret_cast<uint4*>(dst) = v;
          fence_proxy_async_smem();
          __syncwarp();
        }
      }
      if (ok_tile) {
        const uint8_t* kt = ring + st * kStageBytes;
        const uint8_t* vt = kt + kHalfBytes;
        float a0c[4] = {0.f, 0.f, 0.f, 0.f}, a1c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const int col = kk * 16;
          const int box = col >> 6, cb = (col & 63) >> 3;
          const int jj = lane >> 3;
          const int row = r0 + (lane & 7) + ((jj & 1) << 3);
          const int chunk = cb + (jj >> 1);
          uint32_t x0, x1, x2, x3;
          ldmatrix_x4(smem_u32(kt + box * kBoxBytes + row * 128 + ((chunk ^ (row & 7)) << 4)), x0, x1, x2, x3);
          if (kk & 1)
            mma_bf16_16816(a1c, x0, x1, x2, x3, qb[kk][0], qb[kk][1]);
          else
            mma_bf16_16816(a0c, x0, x1, x2, x3, qb[kk][0], qb[kk][1]);
        }
        const bool va = pa >= 0, vb = pb >= 0;
        if (t == 0) {
          spos_s[lta] = pa;
          spos_s[ltb] = pb;
        }
        float sa0 = va ? bf16r(bf16r(a0c[0] + a1c[0]) * p.scale) : NEG_INF;
        float sa1 = va ? bf16r(bf16r(a0c[1] + a1c[1]) * p.scale) : NEG_INF;
        float sb0 = vb ? bf16r(bf16r(a0c[2] + a1c[2]) * p.scale) : NEG_INF;
        float sb1 = vb ? bf16r(bf16r(a0c[3] + a1c[3]) * p.scale) : NEG_INF;
        if (2 * t < HP) {
          *reinterpret_cast<uint32_t*>(&logits[lta * HP + 2 * t]) = pack_bf16(sa0, sa1);  // exact: bf16 values
          *reinterpret_cast<uint32_t*>(&logits[ltb * HP + 2 * t]) = pack_bf16(sb0, sb1);
        }
        float tm0 = fmaxf(sa0, sb0), tm1 = fmaxf(sa1, sb1);
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          tm0 = fmaxf(tm0, __shfl_xor_sync(0xffffffffu, tm0, o));
          tm1 = fmaxf(tm1, __shfl_xor_sync(0xffffffffu, tm1, o));
        }
        const float n0 = fmaxf(m0, tm0), n1 = fmaxf(m1, tm1);
        const float al0 = (m0 == NEG_INF) ? 1.f : expf(m0 - n0);
        const float al1 = (m1 == NEG_INF) ? 1.f : expf(m1 - n1);
        m0 = n0;
        m1 = n1;
        const float ea0 = (va && h0_ok) ? expf(sa0 - n0) : 0.f;
        const float ea1 = (va && h1_ok) ? expf(sa1 - n1) : 0.f;
        const float eb0 = (vb && h0_ok) ? expf(sb0 - n0) : 0.f;
        const float eb1 = (vb && h1_ok) ? expf(sb1 - n1) : 0.f;
        l0 = l0 * al0 + ea0 + eb0;
        l1 = l1 * al1 + ea1 + eb1;
        if (__any_sync(0xffffffffu, al0 != 1.f || al1 != 1.f)) {
#pragma unroll
          for (int m = 0; m < 8; ++m) {
            oacc[m][0] *= al0;
            oacc[m][1] *= al1;
            oacc[m][2] *= al0;
            oacc[m][3] *= al1;
          }
        }
        *reinterpret_cast<float2*>(&ew[g * 8 + 2 * t]) = make_float2(ea0, ea1);
        *reinterpret_cast<float2*>(&ew[(g + 8) * 8 + 2 * t]) = make_float2(eb0, eb1);
        __syncwarp();
        if (__any_sync(0xffffffffu, va || vb)) {
          const float p0 = ew[(2 * t) * 8 + g], p1 = ew[(2 * t + 1) * 8 + g];
          const float p2 = ew[(2 * t + 8) * 8 + g], p3 = ew[(2 * t + 9) * 8 + g];
          const float h0 = bf16r(p0), h1 = bf16r(p1), h2 = bf16r(p2), h3 = bf16r(p3);
          const uint32_t bh0 = pack_bf16(h0, h1), bh1 = pack_bf16(h2, h3);
          const uint32_t bl0 = pack_bf16(p0 - h0, p1 - h1), bl1 = pack_bf16(p2 - h2, p3 - h3);
          const int slot = r0 + (lane & 7) + ((lane >> 4) << 3);
#pragma unroll
          for (int m = 0; m < 8; ++m) {
            const int dchunk = m * 16 + (((lane >> 3) & 1) << 3);
            const int box = dchunk >> 6, c = (dchunk & 63) >> 3;
            uint32_t x0, x1, x2, x3;
            ldmatrix_x4_trans(smem_u32(vt + box * kBoxBytes + slot * 128 + ((c ^ (slot & 7)) << 4)), x0, x1, x2, x3);
            mma_bf16_16816(oacc[m], x0, x1, x2, x3, bh0, bh1);
            mma_bf16_16816(oacc[m], x0, x1, x2, x3, bl0, bl1);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }

    // ---- merge the warps (the cluster kernel's order) ----------------------------
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, o);
      l1 += __shfl_xor_sync(0xffffffffu, l1, o);
    }
    if (lane < 4) {
      wstat[warp * 16 + 2 * lane] = m0;
      wstat[warp * 16 + 2 * lane + 1] = m1;
      wstat[warp * 16 + 8 + 2 * lane] = l0;
      wstat[warp * 16 + 8 + 2 * lane + 1] = l1;
    }
    named_bar(1, kConsumers);
    if (tid < 8) {
      float mc = NEG_INF;
      for (int w = 0; w < kConsumerWarps; ++w) mc = fmaxf(mc, wstat[w * 16 + tid]);
      float lc = 0.f;
      for (int w = 0; w < kConsumerWarps; ++w) {
        const float mw = wstat[w * 16 + tid];
        if (mw != NEG_INF) lc += wstat[w * 16 + 8 + tid] * expf(mw - mc);
      }
      cstat[tid] = mc;
      cstat[8 + tid] = lc;
    }
    {
      const float mw0 = __shfl_sync(0xffffffffu, m0, t), mw1 = __shfl_sync(0xffffffffu, m1, t);
      float mc0 = NEG_INF, mc1 = NEG_INF;
      for (int w = 0; w < kConsumerWarps; ++w) {
        mc0 = fmaxf(mc0, wstat[w * 16 + 2 * t]);
        mc1 = fmaxf(mc1, wstat[w * 16 + 2 * t + 1]);
      }
      const float s0 = (mw0 == NEG_INF) ? 0.f : expf(mw0 - mc0);
      const float s1 = (mw1 == NEG_INF) ? 0.f : expf(mw1 - mc1);
      float* ow = opart + warp * HP * kD;
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        if (h0_ok) {
          ow[(2 * t) * kD + 16 * m + g] = oacc[m][0] * s0;
          ow[(2 * t) * kD + 16 * m + g + 8] = oacc[m][2] * s0;
        }
        if (h1_ok) {
          ow[(2 * t + 1) * kD + 16 * m + g] = oacc[m][1] * s1;
          ow[(2 * t + 1) * kD + 16 * m + g + 8] = oacc[m][3] * s1;
        }
      }
    }
    named_bar(1, kConsumers);
    __nv_bfloat16* orow = p.out + (static_cast<size_t>(b) * p.Hq + kvh * G) * kD;
    if (CS == 1) {
      // ---- one CTA per pair: the final statistics are this CTA's --------------------
      if (tid < G) {
        finM[tid] = cstat[tid];
        finL[tid] = cstat[8 + tid];
        if (!(cstat[8 + tid] > 0.f)) set_err(p.err, kErrNoValidSlot);
      }
      for (int e = tid; e < G * kD; e += kConsumers) {
        const int h = e / kD;
        float acc = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) acc += opart[w * HP * kD + e];
        const float Lh = cstat[8 + h];
        orow[e] = __float2bfloat16_rn(Lh > 0.f ? acc / Lh : 0.f);
      }
      named_bar(1, kConsumers);
    } else {
      // ---- one st.async round over the cluster, as in the cluster kernel ------------
      cluster_wait_acquire();  // every peer has read the previous pair's exchange
      if (warp == 0 && lane < CS) {
        const uint32_t rbar = mapa_u32(smem_u32(xbar), lane);
        const uint32_t rdst = mapa_u32(smem_u32(srecv + rank * 16), lane);
        for (int h = 0; h < 16; ++h) st_async_f32(rdst + 4 * h, cstat[h], rbar);
      }
      if (per % 4 == 0) {
        for (int e = 4 * tid; e < G * kD; e += 4 * kConsumers) {
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int w = 0; w < kConsumerWarps; ++w) {
            const float4 v = *reinterpret_cast<const float4*>(&opart[w * HP * kD + e]);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
          }
          const int r = e / per;
          st_async_v4(mapa_u32(smem_u32(orecv + rank * per + (e - r * per)), r), acc, mapa_u32(smem_u32(xbar), r));
        }
      } else {
        for (int e = tid; e < G * kD; e += kConsumers) {
          float acc = 0.f;
#pragma unroll
          for (int w = 0; w < kConsumerWarps; ++w) acc += opart[w * HP * kD + e];
          const int r = e / per;
          st_async_f32(mapa_u32(smem_u32(orecv + rank * per + (e - r * per)), r), acc, mapa_u32(smem_u32(xbar), r));
        }
      }
      if (!mbar_wait_cluster_bounded(xbar, static_cast<uint32_t>(j) & 1)) {
        set_err(p.err, kErrWaitTimeout);
        atomicExch(bad_flag, 1);
      }
      if (tid < G) {
        const int h = tid;
        float M = NEG_INF;
        for (int c = 0; c < CS; ++c) M = fmaxf(M, srecv[c * 16 + h]);
        float Ls = 0.f;
        for (int c = 0; c < CS; ++c) {
          const float mc = srecv[c * 16 + h];
          const float f = (mc != NEG_INF) ? expf(mc - M) : 0.f;
          fscale[c * 8 + h] = f;
          if (mc != NEG_INF) Ls += srecv[c * 16 + 8 + h] * f;
        }
        finM[h] = M;
        finL[h] = Ls;
        if (rank == 0 && !(Ls > 0.f)) set_err(p.err, kErrNoValidSlot);
      }
      named_bar(1, kConsumers);
      const int e0 = rank * per;
      for (int jj = tid; jj < n_mine; jj += kConsumers) {
        const int h = (e0 + jj) / kD;
        float acc = 0.f;
        for (int c = 0; c < CS; ++c) {
          if (srecv[c * 16 + h] != NEG_INF) acc += orecv[c * per + jj] * fscale[c * 8 + h];
        }
        const float Lh = finL[h];
        orow[e0 + jj] = __float2bfloat16_rn(Lh > 0.f ? acc / Lh : 0.f);
      }
      __syncwarp();
      cluster_arrive_release();  // this thread is done with the received data of this pair
    }
    // ---- per-slot eviction score: max over the group's heads of exp(s - M) / L ------
    if (!(*reinterpret_cast<volatile int*>(bad_flag))) {
      float Mh[G], iLh[G];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        Mh[h] = finM[h];
        iLh[h] = finL[h] > 0.f ? 1.0f / finL[h] : 0.f;
      }
      float* sscore = p.step_score + static_cast<size_t>(b) * S + t0 * kTile;
      for (int i = tid; i < nloc; i += kConsumers) {
        if (spos_s[i] < 0) continue;
        float mx = 0.f;
#pragma unroll
        for (int h = 0; h < G; ++h) {
          const float pr = iLh[h] > 0.f ? expf(__bfloat162float(logits[i * HP + h]) - Mh[h]) * iLh[h] : 0.f;
          mx = fmaxf(mx, pr);
        }
        if (mx != mx) set_err(p.err, kErrNanScore);
        atomicMax(reinterpret_cast<int*>(&sscore[i]), __float_as_int(mx));
      }
    }
    named_bar(1, kConsumers);  // logits, slot positions, partials and statistics are reused next
  }
  if (CS > 1) cluster_wait_acquire();  // exit only after every peer's last push has landed
}

// ------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// [pairs][S][128] bf16 view of a [B, Hkv, S, 128] cache; 64 x 64 x 1 boxes, 128-byte swizzle.
static int make_cache_map(CUtensorMap* map, const void* ptr, long long pairs, int S) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return fail(kStatusCuda, "cuTensorMapEncodeTiled unavailable (driver too old or no GPU)");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(S), static_cast<cuuint64_t>(pairs)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(kD * 2), static_cast<cuuint64_t>(S) * kD * 2};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(kTile), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(kStatusCuda, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return kStatusOk;
}

// CTAs per (sequence, kv head).  A CTA's fixed cost (launch, barrier setup, the final
// exchange) is several microseconds, so clusters are kept as small as possible: the
// smallest size that (a) keeps two CTAs per SM within shared memory and (b) launches
// at least ~1.6 CTAs per SM in total.  Measured on B200 (decode microbench shapes).
static int choose_cluster(int pairs, int tiles, int sms, int max_nloc_tiles) {
  int per_max = 1;
  for (int per = 1; per <= max_nloc_tiles; ++per)
    if (2 * (attn_smem_layout(per, 8).total + 2048) <= 228 * 1024) per_max = per;
  int cs = (tiles + per_max - 1) / per_max;
  const int want = (16 * sms / 10 + pairs - 1) / pairs;
  if (cs < want) cs = want;
  if (cs > tiles) cs = tiles;
  if (cs < 1) cs = 1;
  if (cs > kMaxCluster) cs = kMaxCluster;
  return cs;
}

template <int G, int GR>
static cudaError_t launch_persist(cudaStream_t stream, const CUtensorMap& km, const CUtensorMap& vm, const AttnArgs& a,
                                  int smem, int n_clusters) {
  auto kern = decode_attn_persist_kernel<G, GR>;
  static int configured_smem = 0;
  if (smem > configured_smem) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    configured_smem = smem;
  }
  if (a.cluster > 1) {
    // a cluster needs all its CTAs placed inside one GPC: fewer clusters than SM slots / CS
    // may be resident at once, and a cluster that does not fit would run its whole share of
    // the pairs after the others -- keep the count to what is resident together
    static int cached[kMaxCluster + 1][2] = {};  // [cluster size] -> (smem, max active clusters)
    if (cached[a.cluster][0] != smem) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(a.cluster, n_clusters);
      cfg.blockDim = dim3(attn_threads(GR));
      cfg.dynamicSmemBytes = smem;
      cudaLaunchAttribute attr;
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = a.cluster;
      attr.val.clusterDim.y = 1;
      attr.val.clusterDim.z = 1;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = 0;
      }
      cached[a.cluster][0] = smem;
      cached[a.cluster][1] = n;
    }
    // and leave an eighth of them free: the kernel is launched while the step's previous
    // kernel still holds SMs (programmatic dependent launch), and clusters placed around it
    // can leave too few slots in a GPC for the last ones (measured at 64 sequences x 8 kv
    // heads, clusters of 4: 74 clusters, all resident when launched alone, made the step
    // 1.5x slower than 64); then spread the pairs evenly over as few clusters as that allows
    const int pairs = a.B * a.Hkv;
    const int cap = cached[a.cluster][1] * 7 / 8;
    if (cap >= 1 && n_clusters > cap) n_clusters = cap;
    const int per_cluster = (pairs + n_clusters - 1) / n_clusters;
    n_clusters = (pairs + per_cluster - 1) / per_cluster;
  } else {
    // the fewest CTAs that keep the same largest number of pairs per CTA: with equal shares
    // each CTA's stream gets a larger part of the bandwidth (64 x 8 pairs at C = 1024: 256
    // CTAs of 2 pairs 57.3 us, 296 CTAs of 1 or 2 pairs 59.4 us)
    const int pairs = a.B * a.Hkv;
    const int per_cta = (pairs + n_clusters - 1) / n_clusters;
    n_clusters = (pairs + per_cta - 1) / per_cta;
  }
  return launch_pdl(kern, dim3(a.cluster, n_clusters), dim3(attn_threads(GR)), smem, stream,
                    a.cluster > 1 ? dim3(a.cluster, 1, 1) : dim3(0), km, vm, a);
}

// Clusters of the persistent kernel (0: use one cluster per pair).  Only when one cluster
// per (sequence, kv head) pair would not fit in one wave of two CTAs per SM, the group has
// at most 4 query heads, no per-head retention or fused score update is asked for, and two
// CTAs of its layout fit in one SM's shared memory: then as many clusters as one wave holds.
static int choose_persist(int B, int Hkv, int G, int cs, int nloc_tiles, int groups, int sms, const AttnExtra& x) {
  // one-CTA pairs only by default: with clusters the count that stays resident depends on
  // the chip's GPC layout and on what the previous kernel still holds (measured on two
  // B200s at 64 x 8 pairs, clusters of 4: 213 and 231 us persistent vs 217 us one cluster
  // per pair), while one CTA fits any free slot
  if (cs != 1) return 0;
  if (G > 4 || x.head_keep || x.head_score || x.upd_last) return 0;
  const int slots = 2 * sms;
  if (B * Hkv * cs <= slots) return 0;
  if (2 * (persist_smem_layout(nloc_tiles, 4 * groups, 4).total + 1024 + 1024) > 228 * 1024) return 0;
  return slots / cs;
}

template <int G, int GR>
static cudaError_t launch_g(cudaStream_t stream, const CUtensorMap& km, const CUtensorMap& vm, const AttnArgs& a,
                            int smem) {
  // the fused scatter (knew / vnew) is a small runtime branch in both kernels; the heavier
  // options (per-head retention, in-kernel score update) select the second kernel
  const bool x = a.head_keep || a.head_score || a.upd_last;
  auto kern = x ? decode_attn_score_kernel<G, GR, true> : decode_attn_score_kernel<G, GR, false>;
  static int configured_smem[2] = {0, 0};  // per kernel (plain, with the optional parts)
  if (smem > configured_smem[x]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured_smem[x] = smem;
  }
  return launch_pdl(kern, dim3(a.cluster, a.Hkv, a.B), dim3(attn_threads(GR)), smem, stream, dim3(a.cluster, 1, 1), km,
                    vm, a);
}

int decode_attn_score(cudaStream_t stream, int B, int Hq, int Hkv, int D, int S, const void* q, const void* kcache,
                      const void* vcache, const int* slot_pos, const int* write_slot, void* out, float* step_score,
                      int* err, int cluster_override, const AttnExtra& x, int persist_override) {
  if (!q || !kcache || !vcache || !slot_pos || !out || !step_score)
    return fail(kStatusArg, "decode_attn_score: null pointer");
  if (D != kD) return fail(kStatusUnsupported, "decode_attn_score: head_dim %d unsupported (only 128)", D);
  if (B <= 0 || Hkv <= 0 || Hq <= 0 || S <= 0) return fail(kStatusArg, "decode_attn_score: non-positive size");
  if (Hq % Hkv) return fail(kStatusArg, "decode_attn_score: Hq %% Hkv != 0");
  const int G = Hq / Hkv;
  if (G > 8) return fail(kStatusUnsupported, "decode_attn_score: group size %d > 8 unsupported", G);
  if (B > 65535 || Hkv > 65535) return fail(kStatusArg, "decode_attn_score: grid too large");
  const long long rows = static_cast<long long>(B) * Hkv * S;
  if (rows + kTile >= (1ll << 31)) return fail(kStatusArg, "decode_attn_score: cache too large for 32-bit TMA rows");
  if ((reinterpret_cast<uintptr_t>(kcache) | reinterpret_cast<uintptr_t>(vcache)) & 15)
    return fail(kStatusArg, "decode_attn_score: cache base must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(q) & 3) return fail(kStatusArg, "decode_attn_score: q must be 4-byte aligned");

  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  const int tiles = (S + kTile - 1) / kTile;
  constexpr int kMaxNlocTiles = 48;  // 3072 slots of logits per CTA
  int cs = cluster_override > 0 ? cluster_override : choose_cluster(B * Hkv, tiles, sms, kMaxNlocTiles);
  if (cs > 8) cs = 8;
  const int nloc_tiles = (tiles + cs - 1) / cs;
  if (nloc_tiles > kMaxNlocTiles)
    return fail(kStatusUnsupported, "decode_attn_score: %d slots exceed the per-cluster limit", S);

  CUtensorMap km, vm;
  int st = make_cache_map(&km, kcache, static_cast<long long>(B) * Hkv, S);
  if (st) return st;
  st = make_cache_map(&vm, vcache, static_cast<long long>(B) * Hkv, S);
  if (st) return st;

  AttnArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.kc = static_cast<const __nv_bfloat16*>(kcache);
  a.vc = static_cast<const __nv_bfloat16*>(vcache);
  a.slot_pos = slot_pos;
  a.write_slot = write_slot;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.step_score = step_score;
  a.head_keep = x.head_keep;
  a.head_score = x.head_score;
  a.knew = static_cast<const __nv_bfloat16*>(x.knew);
  a.vnew = static_cast<const __nv_bfloat16*>(x.vnew);
  a.upd_attn = x.upd_attn;
  a.upd_maxa = x.upd_maxa;
  a.upd_cumul = x.upd_cumul;
  a.upd_last = x.upd_last;
  a.upd_cnt = x.upd_cnt;
  a.seq_step = x.seq_step;
  a.seq_counter = x.seq_counter;
  if ((a.knew || a.vnew) && !(a.knew && a.vnew && write_slot))
    return fail(kStatusArg, "decode_attn_score: k_new and v_new need each other and write_slot");
  if (a.knew && ((reinterpret_cast<uintptr_t>(a.knew) | reinterpret_cast<uintptr_t>(a.vnew)) & 15))
    return fail(kStatusArg, "decode_attn_score: k_new / v_new must be 16-byte aligned");
  if (a.upd_last && !(a.upd_attn && a.upd_maxa && a.upd_cumul && a.upd_cnt && a.seq_step && a.seq_counter))
    return fail(kStatusArg, "decode_attn_score: the fused score update needs every state array");
  a.err = err;
  a.B = B;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.S = S;
  a.tiles = tiles;
  a.cluster = cs;
  a.nloc_tiles = nloc_tiles;
  a.ipc = 1;
  a.scale = __bfloat162float(__float2bfloat16_rn(1.0f / sqrtf(static_cast<float>(kD))));
  // two consumer groups pay off once a CTA streams enough tiles to keep both busy
  const int groups = nloc_tiles >= 8 ? 2 : 1;
  const int smem = attn_smem_layout(nloc_tiles, 4 * groups).total + 1024;
  if (smem > 227 * 1024)
    return fail(kStatusUnsupported, "decode_attn_score: %d slots per CTA need %d B of shared memory", nloc_tiles * kTile,
                smem);

  cudaError_t e;
  const int n_cl = persist_override < 0 ? 0
                   : persist_override > 0 ? persist_override
                                          : choose_persist(B, Hkv, G, cs, nloc_tiles, groups, sms, x);
  if (n_cl > 0) {
    if (G > 4 || x.head_keep || x.head_score || x.upd_last)
      return fail(kStatusUnsupported, "decode_attn_score: the persistent kernel takes groups <= 4 without options");
    const int psmem = persist_smem_layout(nloc_tiles, 4 * groups, 4).total + 1024;
    if (psmem > 227 * 1024) return fail(kStatusUnsupported, "decode_attn_score: persistent layout too large");
    switch (G) {
      case 1:
        e = groups == 2 ? launch_persist<1, 2>(stream, km, vm, a, psmem, n_cl)
                        : launch_persist<1, 1>(stream, km, vm, a, psmem, n_cl);
        break;
      case 2:
        e = groups == 2 ? launch_persist<2, 2>(stream, km, vm, a, psmem, n_cl)
                        : launch_persist<2, 1>(stream, km, vm, a, psmem, n_cl);
        break;
      case 3:
        e = groups == 2 ? launch_persist<3, 2>(stream, km, vm, a, psmem, n_cl)
                        : launch_persist<3, 1>(stream, km, vm, a, psmem, n_cl);
        break;
      default:
        e = groups == 2 ? launch_persist<4, 2>(stream, km, vm, a, psmem, n_cl)
                        : launch_persist<4, 1>(stream, km, vm, a, psmem, n_cl);
        break;
    }
    if (e != cudaSuccess) return fail(kStatusCuda, "decode_attn_score launch: %s", cudaGetErrorString(e));
    return kStatusOk;
  }
#define KVBP_ATTN_CASE(g)                                                                        \
  case g:                                                                                        \
    e = groups == 2 ? launch_g<g, 2>(stream, km, vm, a, smem) : launch_g<g, 1>(stream, km, vm, a, smem); \
    break;
  switch (G) {
    KVBP_ATTN_CASE(1)
    KVBP_ATTN_CASE(2)
    KVBP_ATTN_CASE(3)
    KVBP_ATTN_CASE(4)
    KVBP_ATTN_CASE(5)
    KVBP_ATTN_CASE(6)
    KVBP_ATTN_CASE(7)
    default:
      e = groups == 2 ? launch_g<8, 2>(stream, km, vm, a, smem) : launch_g<8, 1>(stream, km, vm, a, smem);
      break;
  }
#undef KVBP_ATTN_CASE
  if (e != cudaSuccess) return fail(kStatusCuda, "decode_attn_score launch: %s", cudaGetErrorString(e));
  return kStatusOk;
}

}  // namespace kvbp

#include "../../include/kvbp.h"

extern "C" int kvbp_decode_attn_score(kvbp_stream_t stream, int32_t B, int32_t Hq, int32_t Hkv, int32_t head_dim,
                                      int32_t S, const void* q, const void* kcache, const void* vcache,
                                      const int32_t* slot_pos, const int32_t* write_slot, void* out,
                                      float* step_score, int32_t* dev_err) {
  return kvbp::decode_attn_score(reinterpret_cast<cudaStream_t>(stream), B, Hq, Hkv, head_dim, S, q, kcache, vcache,
                                 slot_pos, write_slot, out, step_score, dev_err, 0, kvbp::AttnExtra{});
}

extern "C" int kvbp_decode_attn_score_update(kvbp_stream_t stream, int32_t B, int32_t Hq, int32_t Hkv,
                                             int32_t head_dim, int32_t S, const void* q, const void* k_new,
                                             const void* v_new, void* kcache, void* vcache,
                                             const int32_t* slot_pos, const int32_t* write_slot, void* out,
                                             float* step_score, const kvbp_state* st, const int32_t* seq_step,
                                             int32_t* seq_counter, int32_t* dev_err) {
  kvbp::AttnExtra x;
  x.knew = k_new;
  x.vnew = v_new;
  if (!st) {  // scatter only: the score update runs elsewhere (kvbp_update_append_evict)
    if (!k_new) return kvbp::fail(kvbp::kStatusArg, "decode_attn_score_update: nothing to fuse (no state, no k_new)");
    return kvbp::decode_attn_score(reinterpret_cast<cudaStream_t>(stream), B, Hq, Hkv, head_dim, S, q, kcache, vcache,
                                   slot_pos, write_slot, out, step_score, dev_err, 0, x);
  }
  if (!seq_step || !seq_counter)
    return kvbp::fail(kvbp::kStatusArg, "decode_attn_score_update: seq_step and seq_counter are required with st");
  if (st->B != B || st->S != S || st->slot_pos != slot_pos)
    return kvbp::fail(kvbp::kStatusArg, "decode_attn_score_update: state does not match B / S / slot_pos");
  x.upd_attn = st->attn;
  x.upd_maxa = st->max_attn;
  x.upd_cumul = st->cumul;
  x.upd_last = st->last_access;
  x.upd_cnt = st->access_count;
  x.seq_step = seq_step;
  x.seq_counter = seq_counter;
  return kvbp::decode_attn_score(reinterpret_cast<cudaStream_t>(stream), B, Hq, Hkv, head_dim, S, q, kcache, vcache,
                                 slot_pos, write_slot, out, step_score, dev_err, 0, x);
}

extern "C" int kvbp_decode_attn_score_heads(kvbp_stream_t stream, int32_t B, int32_t Hq, int32_t Hkv,
                                            int32_t head_dim, int32_t S, const void* q, const void* kcache,
                                            const void* vcache, const int32_t* slot_pos, const int32_t* write_slot,
                                            const uint8_t* head_keep, void* out, float* step_score,
                                            float* head_score, int32_t* dev_err) {
  if (!head_keep || !head_score)
    return kvbp::fail(kvbp::kStatusArg, "decode_attn_score_heads: head_keep and head_score are required");
  kvbp::AttnExtra x;
  x.head_keep = head_keep;
  x.head_score = head_score;
  return kvbp::decode_attn_score(reinterpret_cast<cudaStream_t>(stream), B, Hq, Hkv, head_dim, S, q, kcache, vcache,
                                 slot_pos, write_slot, out, step_score, dev_err, 0, x);
}

// Same as kvbp_decode_attn_score with the launch shape chosen by the caller (tests, sweeps):
// cluster = CTAs per (sequence, kv head) (0: automatic); persist_clusters = clusters of the
// persistent kernel (-1: never persistent, 0: automatic).
extern "C" int kvbp_decode_attn_score_cfg(kvbp_stream_t stream, int32_t B, int32_t Hq, int32_t Hkv, int32_t head_dim,
                                          int32_t S, const void* q, const void* kcache, const void* vcache,
                                          const int32_t* slot_pos, const int32_t* write_slot, void* out,
                                          float* step_score, int32_t* dev_err, int32_t cluster,
                                          int32_t persist_clusters) {
  return kvbp::decode_attn_score(reinterpret_cast<cudaStream_t>(stream), B, Hq, Hkv, head_dim, S, q, kcache, vcache,
                                 slot_pos, write_slot, out, step_score, dev_err, cluster, kvbp::AttnExtra{},
                                 persist_clusters);
}

// Same as kvbp_decode_attn_score with an explicit cluster size (CTAs per sequence and
// kv head, 1..8); 0 selects automatically.  Used by tests and tuning sweeps.
extern "C" int kvbp_decode_attn_score_cs(kvbp_stream_t stream, int32_t B, int32_t Hq, int32_t Hkv, int32_t head_dim,
                                         int32_t S, const void* q, const void* kcache, const void* vcache,
                                         const int32_t* slot_pos, const int32_t* write_slot, void* out,
                                         float* step_score, int32_t* dev_err, int32_t cluster) {
  return kvbp::decode_attn_score(reinterpret_cast<cudaStream_t>(stream), B, Hq, Hkv, head_dim, S, q, kcache, vcache,
                                 slot_pos, write_slot, out, step_score, dev_err, cluster, kvbp::AttnExtra{});
}
