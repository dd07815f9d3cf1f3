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
// per (sequence, kv head).  Each CTA owns a contiguous range of 64-slot tiles.  K tiles
// then V tiles stream through a 4-stage shared-memory ring filled by 2-D TMA loads
// (128-byte swizzle, no multicast).  Q.K^T runs on the tensor cores (mma.sync m16n8k16,
// slots on M, the <= 8 query heads of the group on N).  The logits of the CTA's slots
// stay in shared memory; the softmax max / sum are combined across the cluster through
// distributed shared memory, so every probability is final before P.V and the K/V
// cache is read exactly once.  P.V runs on the fp32 pipes (lane = 4 head dims), and the
// partial outputs are summed across the cluster through DSMEM.
#include <cooperative_groups.h>

#include "common.cuh"
#include "kvbp_internal.h"

namespace cg = cooperative_groups;

namespace kvbp {

constexpr int kD = 128;
constexpr int kTile = 64;
constexpr int kStages = 4;
constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kTileBytes = kTile * kD * 2;  // 16 KiB: two 64x64 bf16 boxes
constexpr int kBoxBytes = kTileBytes / 2;

struct AttnSmem {
  // byte offsets from the 1024-aligned base
  int logits, valid, opart, octa, stats, bars, total;
};

__host__ __device__ inline int align_up(int x, int a) { return (x + a - 1) / a * a; }

__host__ __device__ inline AttnSmem attn_smem_layout(int nloc_tiles) {
  AttnSmem L;
  int nloc = nloc_tiles * kTile;
  L.logits = kStages * kTileBytes;
  L.valid = L.logits + nloc * 8 * 4;
  L.opart = align_up(L.valid + nloc, 16);
  L.octa = L.opart + kWarps * 8 * kD * 4;
  L.stats = L.octa + 8 * kD * 4;
  L.bars = align_up(L.stats + 4 * 8 * 4, 8);
  L.total = L.bars + kStages * 8;
  return L;
}

struct AttnArgs {
  const __nv_bfloat16* q;  // [B, Hq, D]
  const int* slot_pos;     // [B, S]; < 0 = free slot
  __nv_bfloat16* out;      // [B, Hq, D]
  float* step_score;       // [B, S], non-negative; atomicMax target
  int* err;
  int B, Hq, Hkv, S;
  int tiles;       // ceil(S / 64)
  int cluster;     // CTAs per (sequence, kv head)
  int nloc_tiles;  // max tiles per CTA
  float scale;     // bfloat16(1/sqrt(D)) as float
};

template <int G>
__global__ void __launch_bounds__(kThreads) decode_attn_score_kernel(const __grid_constant__ CUtensorMap kmap,
                                                                     const __grid_constant__ CUtensorMap vmap,
                                                                     const AttnArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const AttnSmem L = attn_smem_layout(p.nloc_tiles);
  uint8_t* ring = base;
  float* logits = reinterpret_cast<float*>(base + L.logits);
  uint8_t* valid = base + L.valid;
  float* opart = reinterpret_cast<float*>(base + L.opart);
  float* octa = reinterpret_cast<float*>(base + L.octa);
  float* st_m = reinterpret_cast<float*>(base + L.stats);
  float* st_l = st_m + 8;
  float* fin_m = st_l + 8;
  float* fin_l = fin_m + 8;
  uint64_t* full = reinterpret_cast<uint64_t*>(base + L.bars);

  cg::cluster_group cluster = cg::this_cluster();
  const int CS = p.cluster;
  const int rank = static_cast<int>(cluster.block_rank());
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = (rank * p.tiles) / CS, t1 = ((rank + 1) * p.tiles) / CS;
  const int nt = t1 - t0, ntot = 2 * nt, nloc = nt * kTile;
  const int S = p.S;
  const int row_base = (b * p.Hkv + kvh) * S;
  const int* spos = p.slot_pos + static_cast<size_t>(b) * S;
  float* sscore = p.step_score + static_cast<size_t>(b) * S;
  const float NEG_INF = -__int_as_float(0x7f800000);

  if (tid == 0) {
    prefetch_tmap(&kmap);
    prefetch_tmap(&vmap);
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    fence_barrier_init();
  }
  __syncthreads();

  auto issue = [&](int u) {
    const int st = u % kStages;
    uint8_t* dst = ring + st * kTileBytes;
    const bool is_k = u < nt;
    const int y = row_base + (t0 + (is_k ? u : u - nt)) * kTile;
    mbar_expect_tx(&full[st], kTileBytes);
    tma_load_2d(dst, is_k ? &kmap : &vmap, &full[st], 0, y);
    tma_load_2d(dst + kBoxBytes, is_k ? &kmap : &vmap, &full[st], 64, y);
  };
  if (tid == 0)
    for (int u = 0; u < (ntot < kStages ? ntot : kStages); ++u) issue(u);

  // B operand of the QK^T mma: lane holds q[head = lane/4][k = 2*(lane%4) (+8)] pairs.
  uint32_t qb[8][2];
  {
    const int g = lane >> 2, t = lane & 3;
    const uint32_t* qrow = reinterpret_cast<const uint32_t*>(
        p.q + (static_cast<size_t>(b) * p.Hq + kvh * G + (g < G ? g : 0)) * kD);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      qb[kk][0] = g < G ? qrow[(kk * 16 + 2 * t) >> 1] : 0u;
      qb[kk][1] = g < G ? qrow[(kk * 16 + 8 + 2 * t) >> 1] : 0u;
    }
  }

  bool bad = false;
  // ---- phase 1: logits of every slot in this CTA's range -------------------------
  for (int u = 0; u < nt; ++u) {
    const int st = u % kStages;
    const uint32_t par = (u / kStages) & 1;
    if (!bad && !mbar_wait_bounded(&full[st], par)) {
      bad = true;
      set_err(p.err, kErrWaitTimeout);
    }
    if (!bad) {
      const uint8_t* tb = ring + st * kTileBytes;
      const int r0 = warp * 16;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int col = kk * 16;
        const int box = col >> 6, cb = (col & 63) >> 3;
        const int j = lane >> 3;
        const int row = r0 + (lane & 7) + ((j & 1) << 3);
        const int chunk = cb + (j >> 1);
        const uint32_t addr = smem_u32(tb + box * kBoxBytes + row * 128 + ((chunk ^ (row & 7)) << 4));
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4(addr, a0, a1, a2, a3);
        mma_bf16_16816(acc, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
      }
      const int g = lane >> 2, t = lane & 3;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int row = r0 + g + half * 8;
        const int slot = (t0 + u) * kTile + row;
        const int lt = u * kTile + row;
        const bool ok = slot < S && spos[slot] >= 0;
        float2 sv;
        sv.x = ok ? bf16r(bf16r(acc[half * 2 + 0]) * p.scale) : NEG_INF;
        sv.y = ok ? bf16r(bf16r(acc[half * 2 + 1]) * p.scale) : NEG_INF;
        *reinterpret_cast<float2*>(&logits[lt * 8 + 2 * t]) = sv;
        if (t == 0) valid[lt] = ok ? 1 : 0;
      }
    }
    bad = __syncthreads_or(bad);
    if (tid == 0 && !bad && u + kStages < ntot) issue(u + kStages);
  }

  // ---- softmax statistics, combined across the cluster ---------------------------
  for (int h = warp; h < G; h += kWarps) {
    float m = NEG_INF;
    for (int i = lane; i < nloc; i += 32) m = fmaxf(m, logits[i * 8 + h]);
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) st_m[h] = bad ? NEG_INF : m;
  }
  cluster.sync();
  if (tid < G) {
    float M = NEG_INF;
    for (int r = 0; r < CS; ++r) M = fmaxf(M, cluster.map_shared_rank(st_m, r)[tid]);
    fin_m[tid] = M;
  }
  __syncthreads();
  for (int h = warp; h < G; h += kWarps) {
    const float M = fin_m[h];
    float sum = 0.f;
    for (int i = lane; i < nloc; i += 32) {
      const float s = logits[i * 8 + h];
      const float e = (s == NEG_INF || M == NEG_INF) ? 0.f : expf(s - M);
      logits[i * 8 + h] = e;
      sum += e;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) st_l[h] = bad ? 0.f : sum;
  }
  cluster.sync();
  if (tid < G) {
    float Lsum = 0.f;
    for (int r = 0; r < CS; ++r) Lsum += cluster.map_shared_rank(st_l, r)[tid];
    fin_l[tid] = Lsum;
    if (Lsum <= 0.f && rank == 0) set_err(p.err, kErrNoValidSlot);
  }
  __syncthreads();
  for (int i = tid; i < nloc; i += kThreads) {
    if (valid[i] && !bad) {
      float mx = 0.f;
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float l = fin_l[h];
        const float pr = l > 0.f ? logits[i * 8 + h] / l : 0.f;
        logits[i * 8 + h] = pr;
        mx = fmaxf(mx, pr);
      }
      if (mx != mx) set_err(p.err, kErrNanScore);
      atomicMax(reinterpret_cast<int*>(&sscore[t0 * kTile + i]), __float_as_int(mx));
    } else {
#pragma unroll
      for (int h = 0; h < 8; ++h) logits[i * 8 + h] = 0.f;
    }
  }
  __syncthreads();

  // ---- phase 2: P . V ----------------------------------------------------------
  float o[G][4];
#pragma unroll
  for (int h = 0; h < G; ++h) o[h][0] = o[h][1] = o[h][2] = o[h][3] = 0.f;
  for (int u = nt; u < ntot; ++u) {
    const int st = u % kStages;
    const uint32_t par = (u / kStages) & 1;
    if (!bad && !mbar_wait_bounded(&full[st], par)) {
      bad = true;
      set_err(p.err, kErrWaitTimeout);
    }
    if (!bad) {
      const uint8_t* tb = ring + st * kTileBytes;
      const int ul = u - nt;
      const int box = lane >> 4, chunk = (lane & 15) >> 1;
      for (int r = 0; r < 16; ++r) {
        const int row = warp * 16 + r;
        const int lt = ul * kTile + row;
        if (!valid[lt]) continue;
        const float4 p0 = *reinterpret_cast<const float4*>(&logits[lt * 8]);
        const float4 p1 = *reinterpret_cast<const float4*>(&logits[lt * 8 + 4]);
        const float pv[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
        const uint2 w = *reinterpret_cast<const uint2*>(tb + box * kBoxBytes + row * 128 +
                                                        ((chunk ^ (row & 7)) << 4) + ((lane & 1) << 3));
        const float v0 = bf16lo(w.x), v1 = bf16hi(w.x), v2 = bf16lo(w.y), v3 = bf16hi(w.y);
#pragma unroll
        for (int h = 0; h < G; ++h) {
          o[h][0] = fmaf(pv[h], v0, o[h][0]);
          o[h][1] = fmaf(pv[h], v1, o[h][1]);
          o[h][2] = fmaf(pv[h], v2, o[h][2]);
          o[h][3] = fmaf(pv[h], v3, o[h][3]);
        }
      }
    }
    bad = __syncthreads_or(bad);
    if (tid == 0 && !bad && u + kStages < ntot) issue(u + kStages);
  }

  // ---- reduce P.V partials: warps -> CTA -> cluster ------------------------------
#pragma unroll
  for (int h = 0; h < G; ++h)
    *reinterpret_cast<float4*>(&opart[(warp * 8 + h) * kD + 4 * lane]) = make_float4(o[h][0], o[h][1], o[h][2], o[h][3]);
  __syncthreads();
  for (int e = tid; e < G * kD; e += kThreads) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) acc += opart[w * 8 * kD + e];
    octa[e] = acc;
  }
  cluster.sync();
  {
    const int per = (G * kD + CS - 1) / CS;
    const int e0 = rank * per;
    const int e1 = (e0 + per < G * kD) ? e0 + per : G * kD;
    __nv_bfloat16* orow = p.out + (static_cast<size_t>(b) * p.Hq + kvh * G) * kD;
    for (int e = e0 + tid; e < e1; e += kThreads) {
      float acc = 0.f;
      for (int r = 0; r < CS; ++r) acc += cluster.map_shared_rank(octa, r)[e];
      orow[e] = __float2bfloat16_rn(acc);
    }
  }
  cluster.sync();  // peers may still be reading this CTA's shared memory
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

// [rows, 128] bf16 view of a [B, Hkv, S, 128] cache; 64x64 boxes with 128-byte swizzle.
static int make_cache_map(CUtensorMap* map, const void* ptr, long long rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return fail(kStatusCuda, "cuTensorMapEncodeTiled unavailable (driver too old or no GPU)");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(kD * 2)};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(kTile)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(kStatusCuda, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return kStatusOk;
}

// Choose CTAs per (sequence, kv head): minimise (total tiles + per-CTA overhead)
// spread over ~2 resident CTAs per SM, plus the tail of one CTA.
static int choose_cluster(int pairs, int tiles, int sms, int max_nloc_tiles) {
  int best = 8;
  double best_t = 1e30;
  for (int cs = 1; cs <= 8; ++cs) {
    const int per = (tiles + cs - 1) / cs;
    if (per > max_nloc_tiles) continue;
    const double slots = 2.0 * sms;
    const double ctas = static_cast<double>(pairs) * cs;
    const double t = (static_cast<double>(pairs) * tiles + ctas * 1.0) / slots + per + 1.0;
    if (t < best_t - 1e-9) {
      best_t = t;
      best = cs;
    }
  }
  return best;
}

template <int G>
static cudaError_t launch_g(cudaStream_t stream, const CUtensorMap& km, const CUtensorMap& vm, const AttnArgs& a,
                            int smem) {
  auto kern = decode_attn_score_kernel<G>;
  static int configured_smem = 0;
  if (smem > configured_smem) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured_smem = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.cluster, a.Hkv, a.B);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = a.cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, km, vm, a);
}

int decode_attn_score(cudaStream_t stream, int B, int Hq, int Hkv, int D, int S, const void* q, const void* kcache,
                      const void* vcache, const int* slot_pos, void* out, float* step_score, int* err,
                      int cluster_override) {
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
  int st = make_cache_map(&km, kcache, rows);
  if (st) return st;
  st = make_cache_map(&vm, vcache, rows);
  if (st) return st;

  AttnArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.slot_pos = slot_pos;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.step_score = step_score;
  a.err = err;
  a.B = B;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.S = S;
  a.tiles = tiles;
  a.cluster = cs;
  a.nloc_tiles = nloc_tiles;
  a.scale = __bfloat162float(__float2bfloat16_rn(1.0f / sqrtf(static_cast<float>(kD))));
  const int smem = attn_smem_layout(nloc_tiles).total + 1024;

  cudaError_t e;
  switch (G) {
    case 1: e = launch_g<1>(stream, km, vm, a, smem); break;
    case 2: e = launch_g<2>(stream, km, vm, a, smem); break;
    case 3: e = launch_g<3>(stream, km, vm, a, smem); break;
    case 4: e = launch_g<4>(stream, km, vm, a, smem); break;
    case 5: e = launch_g<5>(stream, km, vm, a, smem); break;
    case 6: e = launch_g<6>(stream, km, vm, a, smem); break;
    case 7: e = launch_g<7>(stream, km, vm, a, smem); break;
    default: e = launch_g<8>(stream, km, vm, a, smem); break;
  }
  if (e != cudaSuccess) return fail(kStatusCuda, "decode_attn_score launch: %s", cudaGetErrorString(e));
  return kStatusOk;
}

}  // namespace kvbp

#include "../../include/kvbp.h"

extern "C" int kvbp_decode_attn_score(kvbp_stream_t stream, int32_t B, int32_t Hq, int32_t Hkv, int32_t head_dim,
                                      int32_t S, const void* q, const void* kcache, const void* vcache,
                                      const int32_t* slot_pos, void* out, float* step_score, int32_t* dev_err) {
  return kvbp::decode_attn_score(reinterpret_cast<cudaStream_t>(stream), B, Hq, Hkv, head_dim, S, q, kcache, vcache,
                                 slot_pos, out, step_score, dev_err, 0);
}

// Same as kvbp_decode_attn_score with an explicit cluster size (CTAs per sequence and
// kv head, 1..8); 0 selects automatically.  Used by tests and tuning sweeps.
extern "C" int kvbp_decode_attn_score_cs(kvbp_stream_t stream, int32_t B, int32_t Hq, int32_t Hkv, int32_t head_dim,
                                         int32_t S, const void* q, const void* kcache, const void* vcache,
                                         const int32_t* slot_pos, void* out, float* step_score, int32_t* dev_err,
                                         int32_t cluster) {
  return kvbp::decode_attn_score(reinterpret_cast<cudaStream_t>(stream), B, Hq, Hkv, head_dim, S, q, kcache, vcache,
                                 slot_pos, out, step_score, dev_err, cluster);
}
