// Causal prefill attention with the per-key score on the 5th-generation tensor cores
// (tcgen05 + TMEM), one sequence, one layer.
//
// Reference: the prefill branch of JAXModelAdapter (jax_inference.py:1684-1790) runs
// _attention_layer (:1018-1050) over the prompt with the causal mask (:1169-1179); the
// generator reduces the probabilities to one score per key position, max over layers,
// heads and query rows (jax_inference.py:1754-1760, kv_coupled_generator.py:636-658).
// Rounding points as in the decode kernel: s = bf16(bf16(q.k) * bf16(1/sqrt(128))),
// fp32 softmax, out = bf16(sum_j p_j * fp32(v_j)), score[j] = max p[., j].
//
// One CTA per (128-query tile, query head), warp-specialised:
//   * one control warp issues the TMA loads (Q once, K tiles double-buffered, V) and the
//     tcgen05.mma instructions, and commits them to mbarriers;
//   * 16 softmax warps: warp w reads TMEM lanes 32*(w % 4) .. +31 (its 32 query rows) and
//     columns 32*(w / 4) .. +31 of every score tile, so four warps share each row.
//   pass 1: S = Q.K^T tile by tile (M = 128 queries, N = 128 keys, K = 128 dims, bf16 in,
//           fp32 accumulator in TMEM, two S buffers so the next tile's MMA overlaps this
//           tile's softmax work); each thread keeps the running max and sum of exp(s - M)
//           of its row share; the four shares are merged at the end of the pass.
//   pass 2: S again; p = exp(s - M) / L (the final statistics are known; exp is the
//           hardware 2^x of s * log2(e) - M * log2(e), one FFMA and one MUFU op, relative
//           error ~1e-6 for |s| < 30, and 1/L is formed once); the
//           per-key maximum over the tile's rows (a warp max reduction per key across
//           the warp's 32 rows, then one atomicMax per key and warp) goes to the score; P is written
//           in bf16 hi + lo parts (two MMAs, ~16-bit mantissa; V is exact in bf16) and
//           O += P.V accumulates in TMEM.
// The softmax warps' element work is kept to few instructions per score: a pair of
// scores takes one packed conversion (cvt.rn.bf16x2.f32) and one packed bf16 multiply by
// the scale (the exact product rounded once, = bf16(bf16(q.k) * bf16(1/sqrt(128)))), exp
// is one FFMA + ex2, P's hi part is a mask, packing is a byte permute, and the causal /
// tail masks are applied only to the blocks that straddle them.
// Q, K and V tiles arrive by 3-D TMA (128-byte swizzle) in the K-major layout the MMA
// descriptors describe; P is written by the threads in the same swizzled layout.  V is
// the MN-major B operand of P.V.  K tiles are double-buffered (the next tile's load
// overlaps the current tile's softmax work).
#include "common.cuh"
#include "kvbp_internal.h"

namespace kvbp {
namespace pf {

constexpr int kRows = 128;        // queries per CTA (= TMEM lanes)
constexpr int kKeys = 128;        // keys per tile
constexpr int kD = 128;
constexpr int kCWarps = 16;       // softmax warps
constexpr int kConsumers = kCWarps * 32;
constexpr int kThreads = kConsumers + 32;  // + the control warp
constexpr int kHalf = kRows * 128;  // one 64-column half of a [128][128] bf16 tile: 16 KiB
constexpr int kTile = 2 * kHalf;    // 32 KiB
constexpr int kTmemCols = 512;      // S0: 0..127, S1: 128..255, O: 256..383

// smem layout (from a 1024-aligned base)
constexpr int kOffQ = 0;
constexpr int kOffK0 = kOffQ + kTile;
constexpr int kOffK1 = kOffK0 + kTile;
constexpr int kOffV = kOffK1 + kTile;
constexpr int kOffPh = kOffV + kTile;
constexpr int kOffPl = kOffPh + kTile;
constexpr int kOffStat = kOffPl + kTile;              // float2 [4 column groups][128 rows]
constexpr int kOffBars = kOffStat + 4 * kRows * 8;    // 12 mbarriers
constexpr int kOffMisc = kOffBars + 128;              // tmem address, flags
constexpr int kSmem = kOffMisc + 64 + 1024;

// 2^x (the hardware approximation; -inf gives +0)
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// the upper halves of two fp32 words packed as bf16x2 (a in the low half)
__device__ __forceinline__ uint32_t hi_halves(float a, float b) {
  return __byte_perm(__float_as_uint(a), __float_as_uint(b), 0x7632);
}

// bf16(bf16(a) * scale), bf16(bf16(b) * scale) for fp32 a, b: one packed conversion and
// one packed bf16 multiply (the exact product of two bf16 values is rounded once to
// nearest-even), returned as fp32
__device__ __forceinline__ void rnd_scaled_pair(float& a, float& b, uint32_t scale2) {
  uint32_t w;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(w) : "f"(b), "f"(a));  // b -> upper half, a -> lower
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(w) : "r"(w), "r"(scale2));
  a = __uint_as_float(w << 16);
  b = __uint_as_float(w & 0xFFFF0000u);
}


struct Args {
  int P, Hq, Hkv, G;
  float scale;         // bf16(1/sqrt(128)) as float
  __nv_bfloat16* out;  // [P][Hq][128]
  float* colmax;       // [P] or null: max-accumulated per-key score
  int* err;
};

__global__ void __launch_bounds__(kThreads, 1) prefill_attn_kernel(const __grid_constant__ CUtensorMap qmap,
                                                                  const __grid_constant__ CUtensorMap kmap,
                                                                  const __grid_constant__ CUtensorMap vmap,
                                                                  const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + kOffBars);
  uint64_t* qfull = bars + 0;
  uint64_t* kfull = bars + 1;   // [2] K tile landed
  uint64_t* kfree = bars + 3;   // [2] the Q.K^T that read the K buffer is done
  uint64_t* vfull = bars + 5;
  uint64_t* sfull = bars + 6;   // [2] S buffer written
  uint64_t* sfree = bars + 8;   // [2] every softmax warp has read the S buffer
  uint64_t* pfull = bars + 10;  // every softmax warp has written its share of P
  uint64_t* pvdone = bars + 11; // O += P.V done (P and V may be overwritten)
  float2* stat = reinterpret_cast<float2*>(base + kOffStat);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(base + kOffMisc);
  int* bad = reinterpret_cast<int*>(base + kOffMisc + 4);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // largest query tiles first: they carry the most keys under the causal mask
  const int ntq = (a.P + kRows - 1) / kRows;
  const int qt = ntq - 1 - static_cast<int>(blockIdx.x);
  const int h = blockIdx.y, g = h / a.G;
  const int q0 = qt * kRows;
  const int nkt = qt + 1;  // key tiles 0 .. the diagonal one
  const int T = 2 * nkt;   // S tiles over both passes
  const float NEG_INF = -__int_as_float(0x7f800000);

  if (tid == 0) {
    for (int i = 0; i < 12; ++i) mbar_init(bars + i, (i == 8 || i == 9 || i == 10) ? kCWarps : 1);
    *bad = 0;
    fence_barrier_init();
  }
  if (warp == kCWarps) {
    if (lane == 0) {
      prefetch_tmap(&qmap);
      prefetch_tmap(&kmap);
      prefetch_tmap(&vmap);
    }
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  tc_before();
  __syncthreads();
  tc_after();
  const uint32_t tmem = *tslot;
  const uint32_t tO = tmem + 256;
  uint8_t* sQ = base + kOffQ;
  uint8_t* sV = base + kOffV;
  uint8_t* sPh = base + kOffPh;
  uint8_t* sPl = base + kOffPl;
  auto kbuf = [&](int b) { return base + (b ? kOffK1 : kOffK0); };
  auto healthy = [&]() { return !*reinterpret_cast<volatile int*>(bad); };
  auto wait_or_fail = [&](uint64_t* bar, uint32_t ph) {
    if (!mbar_wait_bounded(bar, ph)) {
      set_err(a.err, kErrWaitTimeout);
      atomicExch(bad, 1);
    }
  };

  // =============================== control warp =====================================
  if (warp == kCWarps) {
    if (lane == 0) {
      const uint32_t idS = tc_idesc(128, 128, 0), idO = tc_idesc(128, 128, 1);
      auto key_tile = [&](int j) { return j < nkt ? j : j - nkt; };
      auto issue_k = [&](int j) {  // K tile of S-tile j into buffer j & 1
        const int b = j & 1;
        if (j >= 2) wait_or_fail(&kfree[b], ((j >> 1) - 1) & 1);
        mbar_expect_tx(&kfull[b], kTile);
        tma_load_3d(kbuf(b), &kmap, &kfull[b], 0, key_tile(j) * kKeys, g);
        tma_load_3d(kbuf(b) + kHalf, &kmap, &kfull[b], 64, key_tile(j) * kKeys, g);
      };
      auto issue_s = [&](int j) {  // S-tile j = Q . K^T into S buffer j & 1
        const int b = j & 1;
        wait_or_fail(&kfull[b], (j >> 1) & 1);
        if (j >= 2) wait_or_fail(&sfree[b], ((j >> 1) - 1) & 1);
        tc_after();
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t off = (ks >> 2) * kHalf + (ks & 3) * 32;
          tc_mma(tmem + b * 128, tc_sdesc(smem_u32(sQ) + off, 16, 1024), tc_sdesc(smem_u32(kbuf(b)) + off, 16, 1024),
                   idS, ks > 0);
        }
        tc_commit(&sfull[b]);
        tc_commit(&kfree[b]);
      };
      mbar_expect_tx(qfull, kTile);
      tma_load_3d(sQ, &qmap, qfull, 0, h, q0);
      tma_load_3d(sQ + kHalf, &qmap, qfull, 64, h, q0);
      issue_k(0);
      if (T > 1) issue_k(1);
      wait_or_fail(qfull, 0);
      if (healthy()) issue_s(0);
      for (int j = 0; j < T && healthy(); ++j) {
        if (j + 1 < T) issue_s(j + 1);
        if (j + 2 < T) issue_k(j + 2);
        if (j >= nkt) {  // pass 2: O += P.V for key tile kt
          const int kt = j - nkt;
          if (kt > 0) wait_or_fail(pvdone, (kt - 1) & 1);  // the V buffer is free
          mbar_expect_tx(vfull, kTile);
          tma_load_3d(sV, &vmap, vfull, 0, kt * kKeys, g);
          tma_load_3d(sV + kHalf, &vmap, vfull, 64, kt * kKeys, g);
          wait_or_fail(pfull, kt & 1);
          wait_or_fail(vfull, kt & 1);
          tc_after();
          for (int ks = 0; ks < 8; ++ks) {  // K = 128 keys in steps of 16
            const uint32_t aoff = (ks >> 2) * kHalf + (ks & 3) * 32;
            const uint64_t dv = tc_sdesc(smem_u32(sV) + ks * 16 * 128, kHalf, 1024);  // MN-major V
            tc_mma(tO, tc_sdesc(smem_u32(sPh) + aoff, 16, 1024), dv, idO, (kt > 0 || ks > 0));
            tc_mma(tO, tc_sdesc(smem_u32(sPl) + aoff, 16, 1024), dv, idO, 1);
          }
          tc_commit(pvdone);
        }
      }
    }
    __syncwarp();
  } else {
    // =============================== softmax warps ====================================
    const int lg = warp & 3, cg = warp >> 2;
    const int rloc = lg * 32 + lane;  // TMEM lane = query row within the tile
    const int row = q0 + rloc;
    const uint32_t lane_base = static_cast<uint32_t>(lg * 32) << 16;
    const int rmin = q0 + lg * 32;             // this warp's rows: rmin .. rmin + 31
    const bool rows_in = rmin + 31 < a.P;
    constexpr float kLog2e = 1.4426950408889634f;
    const uint32_t scale2 = (__float_as_uint(a.scale) >> 16) * 0x10001u;  // bf16(scale) in both halves
    float m = NEG_INF, l = 0.f;
    // ---- pass 1: row statistics over this warp's columns
    for (int j = 0; j < nkt; ++j) {
      const int b = j & 1;
      wait_or_fail(&sfull[b], (j >> 1) & 1);
      tc_after();
      float s[32];
      const bool ok = __all_sync(0xffffffffu, healthy());
      if (ok) tc_ld32(tmem + b * 128 + lane_base + cg * 32, s);
      tc_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sfree[b]);
      if (ok) {
        const int kb = j * kKeys + cg * 32;
        float mt = NEG_INF;
#pragma unroll
        for (int i = 0; i < 32; i += 2) rnd_scaled_pair(s[i], s[i + 1], scale2);  // bf16(bf16(q.k) * scale)
        if (kb + 31 <= rmin && rows_in) {  // warp-uniform: no key of the block is masked
#pragma unroll
          for (int i = 0; i < 32; ++i) mt = fmaxf(mt, s[i]);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int key = kb + i;
            s[i] = (key <= row && key < a.P) ? s[i] : NEG_INF;
            mt = fmaxf(mt, s[i]);
          }
        }
        if (mt != NEG_INF) {
          const float mn = fmaxf(m, mt);
          const float mL = mn * kLog2e;
          float add[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int i = 0; i < 32; ++i) add[i & 3] += ex2(fmaf(s[i], kLog2e, -mL));  // masked: 2^-inf = 0
          l = l * ex2((m - mn) * kLog2e) + ((add[0] + add[1]) + (add[2] + add[3]));
          m = mn;
        }
      }
    }
    // ---- merge the four column groups' statistics of each row
    stat[cg * kRows + rloc] = make_float2(m, l);
    named_bar(1, kConsumers);
    {
      float M = NEG_INF;
#pragma unroll
      for (int c = 0; c < 4; ++c) M = fmaxf(M, stat[c * kRows + rloc].x);
      float Ls = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float2 st = stat[c * kRows + rloc];
        if (st.x != NEG_INF) Ls += st.y * ex2((st.x - M) * kLog2e);
      }
      m = M;
      l = 1.0f / Ls;  // from here on: the reciprocal of the row sum
    }
    const float mL = m * kLog2e;
    // ---- pass 2: exact probabilities, per-key score, P for the tensor cores
    for (int kt = 0; kt < nkt; ++kt) {
      const int j = nkt + kt, b = j & 1;
      wait_or_fail(&sfull[b], (j >> 1) & 1);
      tc_after();
      float s[32];
      const bool ok = __all_sync(0xffffffffu, healthy());
      if (ok) tc_ld32(tmem + b * 128 + lane_base + cg * 32, s);
      tc_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sfree[b]);
#pragma unroll
      for (int i = 0; i < 32; i += 2) rnd_scaled_pair(s[i], s[i + 1], scale2);  // bf16(bf16(q.k) * scale)
      float p[32];
      const int kb = kt * kKeys + cg * 32;
      if (ok && kb + 31 <= rmin && rows_in) {  // warp-uniform: no key of the block is masked
#pragma unroll
        for (int i = 0; i < 32; ++i) p[i] = __fmul_rn(ex2(fmaf(s[i], kLog2e, -mL)), l);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int key = kb + i;
          p[i] = (ok && key <= row && key < a.P && row < a.P)
                     ? __fmul_rn(ex2(fmaf(s[i], kLog2e, -mL)), l)
                     : 0.f;
        }
      }
      if (a.colmax) {
        // per-key maximum over the warp's 32 rows: p >= 0, so its bit pattern orders like
        // an unsigned integer; lane i keeps key (tile column cg * 32 + i)
        float v[1];
        {
          uint32_t mine = 0;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            uint32_t r;
            asm volatile("redux.sync.max.u32 %0, %1, 0xffffffff;" : "=r"(r) : "r"(__float_as_uint(p[i])));
            mine = (lane == i) ? r : mine;
          }
          v[0] = __uint_as_float(mine);
        }
        const int key = kt * kKeys + cg * 32 + lane;
        if (ok && key < a.P && v[0] > 0.f) atomicMax(reinterpret_cast<int*>(a.colmax + key), __float_as_int(v[0]));
      }
      if (kt > 0) wait_or_fail(pvdone, (kt - 1) & 1);  // the previous P.V has read P
      uint32_t ph[16], pl[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        // p = hi + lo: hi = p truncated to bf16 (one mask), lo = p - hi (exact, >= 0)
        // truncated to bf16; hi + lo is within 2^-16 of p
        const float h0 = __uint_as_float(__float_as_uint(p[2 * i]) & 0xFFFF0000u);
        const float h1 = __uint_as_float(__float_as_uint(p[2 * i + 1]) & 0xFFFF0000u);
        ph[i] = hi_halves(h0, h1);
        pl[i] = hi_halves(__fsub_rn(p[2 * i], h0), __fsub_rn(p[2 * i + 1], h1));
      }
      // the row's 32 keys into the K-major swizzled A operand: 4 chunks of 8 keys
      const int half = cg >> 1;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        const int chunk = (cg & 1) * 4 + cc;
        const uint32_t off = half * kHalf + rloc * 128 + ((chunk ^ (rloc & 7)) << 4);
        *reinterpret_cast<uint4*>(sPh + off) = make_uint4(ph[4 * cc], ph[4 * cc + 1], ph[4 * cc + 2], ph[4 * cc + 3]);
        *reinterpret_cast<uint4*>(sPl + off) = make_uint4(pl[4 * cc], pl[4 * cc + 1], pl[4 * cc + 2], pl[4 * cc + 3]);
      }
      fence_proxy_async_smem();  // P is read by the tensor cores next
      __syncwarp();
      if (lane == 0) mbar_arrive(pfull);
    }
    // ---- O -> bf16 output (this warp's 32 of the 128 dims)
    wait_or_fail(pvdone, (nkt - 1) & 1);
    tc_after();
    if (__all_sync(0xffffffffu, healthy())) {
      float o[32];
      tc_ld32(tO + lane_base + cg * 32, o);
      if (row < a.P) {
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) w[i] = pack_bf16(o[2 * i], o[2 * i + 1]);
        uint4* dst = reinterpret_cast<uint4*>(a.out + (static_cast<size_t>(row) * a.Hq + h) * kD + cg * 32);
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
      }
    }
  }
  tc_before();
  __syncthreads();
  if (warp == kCWarps) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

}  // namespace pf

// ------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------
using EncodeTiledFnP = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFnP encode_fn_p() {
  static EncodeTiledFnP fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFnP>(ptr);
  }
  return fn;
}

static int map3(CUtensorMap* m, const void* ptr, cuuint64_t d0, cuuint64_t d1, cuuint64_t d2, cuuint64_t s1,
                cuuint64_t s2, cuuint32_t b1, cuuint32_t b2) {
  EncodeTiledFnP enc = encode_fn_p();
  if (!enc) return fail(kStatusCuda, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1, s2};
  cuuint32_t box[3] = {64, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(kStatusCuda, "prefill_attn: tensor map failed (%d)", static_cast<int>(r));
  return kStatusOk;
}

int prefill_attn(cudaStream_t stream, int P, int Hq, int Hkv, int D, const void* q, const void* kc, const void* vc,
                 void* out, float* colmax, int* err) {
  using namespace pf;
  if (!q || !kc || !vc || !out) return fail(kStatusArg, "prefill_attn: null pointer");
  if (D != kD) return fail(kStatusUnsupported, "prefill_attn: head_dim %d unsupported (only 128)", D);
  if (P <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv) return fail(kStatusArg, "prefill_attn: bad sizes");
  if ((P + kRows - 1) / kRows > 65535 || Hq > 65535) return fail(kStatusArg, "prefill_attn: grid too large");
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(kc) | reinterpret_cast<uintptr_t>(vc)) & 15)
    return fail(kStatusArg, "prefill_attn: q, k, v must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(out) & 15) return fail(kStatusArg, "prefill_attn: out must be 16-byte aligned");
  CUtensorMap qm, km, vm;
  // q [P][Hq][128]: dims (d, head, position), one head x 128 positions per box
  int st = map3(&qm, q, kD, Hq, P, static_cast<cuuint64_t>(kD) * 2, static_cast<cuuint64_t>(Hq) * kD * 2, 1, kRows);
  if (st) return st;
  // k, v [Hkv][P][128]: dims (d, position, kv head), 128 positions per box
  st = map3(&km, kc, kD, P, Hkv, static_cast<cuuint64_t>(kD) * 2, static_cast<cuuint64_t>(P) * kD * 2, kKeys, 1);
  if (st) return st;
  st = map3(&vm, vc, kD, P, Hkv, static_cast<cuuint64_t>(kD) * 2, static_cast<cuuint64_t>(P) * kD * 2, kKeys, 1);
  if (st) return st;
  Args a;
  a.P = P;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.G = Hq / Hkv;
  a.scale = __bfloat162float(__float2bfloat16_rn(1.0f / sqrtf(static_cast<float>(kD))));
  a.out = static_cast<__nv_bfloat16*>(out);
  a.colmax = colmax;
  a.err = err;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(prefill_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return fail(kStatusCuda, "prefill_attn: %s", cudaGetErrorString(e));
    configured = true;
  }
  dim3 grid((P + kRows - 1) / kRows, Hq);
  prefill_attn_kernel<<<grid, kThreads, kSmem, stream>>>(qm, km, vm, a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(kStatusCuda, "prefill_attn launch: %s", cudaGetErrorString(e));
  return kStatusOk;
}

}  // namespace kvbp

#include "../../include/kvbp.h"

extern "C" int kvbp_prefill_attn_score(kvbp_stream_t stream, int32_t P, int32_t Hq, int32_t Hkv, int32_t head_dim,
                                       const void* q, const void* kcache, const void* vcache, void* out,
                                       float* colmax, int32_t* dev_err) {
  return kvbp::prefill_attn(reinterpret_cast<cudaStream_t>(stream), P, Hq, Hkv, head_dim, q, kcache, vcache, out,
                            colmax, dev_err);
}
