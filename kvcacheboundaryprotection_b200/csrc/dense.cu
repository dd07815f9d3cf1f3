// Per-token kernels around the GEMMs of one decoder step: embedding gather, fused
// residual-add + RMSNorm, the QKV epilogue (bias, q/k RMSNorm, RoPE, scatter of the
// new K/V into its cache slot), SwiGLU and greedy argmax.  Rounding points follow
// src/counterfact_kv_eviction/jax_inference.py (rms_norm :609-618, rotary_embedding
// :621-637, bias add :953-956, q/k norm :975-978, cache write :1011-1012, silu/mlp
// :702-704,1089-1107, residual adds :1280,1325, greedy sampling at
// kv_coupled_generator.py:344).
#include "common.cuh"
#include "kvbp_internal.h"

namespace kvbp {

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide float sum; every thread receives the total.  ``red`` holds 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
  t = warp_sum(t);
  return t;
}

// ---- embedding gather --------------------------------------------------------------
__global__ void embed_kernel(const __nv_bfloat16* __restrict__ table, const int* __restrict__ ids, int V, int H,
                             __nv_bfloat16* __restrict__ out, int* err) {
  pdl_launch_dependents();
  pdl_wait();
  const int r = blockIdx.x;
  const int id = ids[r];
  if (id < 0 || id >= V) {
    set_err(err, kErrIndex);
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(table + static_cast<size_t>(id) * H);
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(r) * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

// ---- per-row sum of squares (feeds the RMSNorm prologue of the decode GEMM) -----------
__global__ void row_sumsq_kernel(const __nv_bfloat16* __restrict__ h, int H, float* __restrict__ ss_out) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float red[32];
  const size_t r = blockIdx.x;
  float ss = 0.f;
  for (int i = threadIdx.x * 2; i < H; i += blockDim.x * 2) {
    const uint32_t hv = *reinterpret_cast<const uint32_t*>(h + r * H + i);
    ss += bf16lo(hv) * bf16lo(hv) + bf16hi(hv) * bf16hi(hv);
  }
  ss = block_sum(ss, red);
  if (threadIdx.x == 0) ss_out[r] = ss;
}

// ---- h = bf16(h + delta); out = bf16(rmsnorm(h) * w) ---------------------------------
__global__ void add_rmsnorm_kernel(__nv_bfloat16* __restrict__ h, const __nv_bfloat16* __restrict__ delta,
                                   const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out, int H,
                                   float eps) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float red[32];
  const size_t r = blockIdx.x;
  __nv_bfloat16* hr = h + r * H;
  const __nv_bfloat16* dr = delta ? delta + r * H : nullptr;
  float ss = 0.f;
  for (int i = threadIdx.x * 2; i < H; i += blockDim.x * 2) {
    const uint32_t hv = *reinterpret_cast<const uint32_t*>(hr + i);
    float x0 = bf16lo(hv), x1 = bf16hi(hv);
    if (dr) {
      const uint32_t dv = *reinterpret_cast<const uint32_t*>(dr + i);
      x0 = bf16r(x0 + bf16lo(dv));
      x1 = bf16r(x1 + bf16hi(dv));
      *reinterpret_cast<uint32_t*>(hr + i) = pack_bf16(x0, x1);
    }
    ss += x0 * x0 + x1 * x1;
  }
  ss = block_sum(ss, red);
  const float var = ss / static_cast<float>(H);
  const float inv = 1.0f / sqrtf(var + eps);
  for (int i = threadIdx.x * 2; i < H; i += blockDim.x * 2) {
    const uint32_t hv = *reinterpret_cast<const uint32_t*>(hr + i);
    const uint32_t wv = *reinterpret_cast<const uint32_t*>(w + i);
    *reinterpret_cast<uint32_t*>(out + r * H + i) =
        pack_bf16((bf16lo(hv) * inv) * bf16lo(wv), (bf16hi(hv) * inv) * bf16hi(wv));
  }
}

// ---- QKV epilogue -----------------------------------------------------------------
// One block (8 warps) per row.  The row's RoPE cos/sin (64 frequencies) are formed once in
// shared memory; warp w finishes heads w, w + 8, ...; lane l owns the RoPE pairs
// (l, l + 64) and (l + 32, l + 96) of the head.
__global__ void __launch_bounds__(256) qkv_epilogue_kernel(
    const __nv_bfloat16* __restrict__ qkv, int ldq, const __nv_bfloat16* __restrict__ bias,
    const __nv_bfloat16* __restrict__ qnw, const __nv_bfloat16* __restrict__ knw, float eps,
    const float* __restrict__ inv_freq, const int* __restrict__ positions, const int* __restrict__ write_slot,
    int rows_per_seq, int Hq, int Hkv, int S, __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ kcache,
    __nv_bfloat16* __restrict__ vcache, int* err) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float cs[64], sn[64];
  const int r = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid < 64) {
    const float ang = static_cast<float>(positions[r]) * inv_freq[tid];
    cs[tid] = bf16r(cosf(ang));
    sn[tid] = bf16r(sinf(ang));
  }
  __syncthreads();
  const int slot = write_slot[r];
  const int seq = r / rows_per_seq;
  const int nh = Hq + 2 * Hkv;
  for (int hh = warp; hh < nh; hh += 8) {
    const __nv_bfloat16* src = qkv + static_cast<size_t>(r) * ldq + hh * 128;
    float x0[2], x1[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int i = lane + 32 * u;
      x0[u] = __bfloat162float(src[i]);
      x1[u] = __bfloat162float(src[i + 64]);
      if (bias) {
        x0[u] = bf16r(x0[u] + __bfloat162float(bias[hh * 128 + i]));
        x1[u] = bf16r(x1[u] + __bfloat162float(bias[hh * 128 + i + 64]));
      }
    }
    const bool is_q = hh < Hq, is_k = !is_q && hh < Hq + Hkv;
    if (is_q || is_k) {
      const __nv_bfloat16* nw = is_q ? qnw : knw;
      if (nw) {  // warp-uniform branch: RMSNorm over the head's 128 features
        const float ss = warp_sum(x0[0] * x0[0] + x1[0] * x1[0] + x0[1] * x0[1] + x1[1] * x1[1]);
        const float inv = 1.0f / sqrtf(ss / 128.0f + eps);
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int i = lane + 32 * u;
          x0[u] = bf16r((x0[u] * inv) * __bfloat162float(nw[i]));
          x1[u] = bf16r((x1[u] * inv) * __bfloat162float(nw[i + 64]));
        }
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int i = lane + 32 * u;
        const float c = cs[i], sv = sn[i];
        const float y0 = bf16r(bf16r(x0[u] * c) - bf16r(x1[u] * sv));
        const float y1 = bf16r(bf16r(x1[u] * c) + bf16r(x0[u] * sv));
        x0[u] = y0;
        x1[u] = y1;
      }
    }
    __nv_bfloat16* dst;
    if (is_q) {
      dst = q_out + (static_cast<size_t>(r) * Hq + hh) * 128;
    } else {
      if (slot < 0) continue;  // position evicted before its forward: nothing to store
      if (slot >= S) {
        if (lane == 0) set_err(err, kErrIndex);
        continue;
      }
      const int kvh = is_k ? hh - Hq : hh - Hq - Hkv;
      dst = (is_k ? kcache : vcache) + ((static_cast<size_t>(seq) * Hkv + kvh) * S + slot) * 128;
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int i = lane + 32 * u;
      dst[i] = __float2bfloat16_rn(x0[u]);
      dst[i + 64] = __float2bfloat16_rn(x1[u]);
    }
  }
}

// ---- SwiGLU: act = bf16(bf16(g * bf16(sigmoid(g))) * u) -------------------------------
__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ gu, int F, long long n,
                                __nv_bfloat16* __restrict__ act) {
  pdl_launch_dependents();
  pdl_wait();
  for (long long e = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 2; e < n;
       e += static_cast<long long>(gridDim.x) * blockDim.x * 2) {
    const long long r = e / F, c = e % F;
    const uint32_t gv = *reinterpret_cast<const uint32_t*>(gu + r * 2 * F + c);
    const uint32_t uv = *reinterpret_cast<const uint32_t*>(gu + r * 2 * F + F + c);
    float out[2];
    const float g[2] = {bf16lo(gv), bf16hi(gv)};
    const float u[2] = {bf16lo(uv), bf16hi(uv)};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float sig = bf16r(1.0f / (1.0f + expf(-g[j])));
      out[j] = bf16r(bf16r(g[j] * sig) * u[j]);
    }
    *reinterpret_cast<uint32_t*>(act + r * F + c) = pack_bf16(out[0], out[1]);
  }
}

// ---- greedy argmax: first index of the maximum (numpy.argmax semantics) ----------------
struct ArgBest {
  float v;
  int i;
};

__device__ __forceinline__ bool arg_better(float av, int ai, float bv, int bi) {
  const bool an = av != av, bn = bv != bv;
  if (an != bn) return an;  // numpy.argmax returns the first NaN
  if (an) return ai < bi;
  return av > bv || (av == bv && ai < bi);
}

// Grid (CS, rows), a cluster of CS CTAs per row: CTA c scans vectors [c, c + 1) * nvec / CS
// of the row, and cluster rank 0 reduces the CTAs' winners over distributed shared memory.
__global__ void argmax_kernel(const __nv_bfloat16* __restrict__ logits, long long ld, int V, int* __restrict__ out,
                              long long* __restrict__ keys, int index_offset) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float sv[32];
  __shared__ int si[32];
  __shared__ float cta_v;  // this CTA's winner, read by cluster rank 0
  __shared__ int cta_i;
  const int r = blockIdx.y, CS = gridDim.x, c = blockIdx.x;
  const __nv_bfloat16* row = logits + r * ld;
  float bv = -__int_as_float(0x7f800000);
  int bi = 0x7fffffff;
  const int nvec = V / 8;
  const uint4* rv = reinterpret_cast<const uint4*>(row);
  auto visit = [&](const uint4 w, int j) {  // the 8 logits of vector j
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float a = bf16lo(ws[k]), b = bf16hi(ws[k]);
      const int ia = j * 8 + 2 * k;
      if (arg_better(a, ia, bv, bi)) bv = a, bi = ia;
      if (arg_better(b, ia + 1, bv, bi)) bv = b, bi = ia + 1;
    }
  };
  // four independent loads in flight per thread (the winner does not depend on the order
  // in which candidates are visited: larger value, then smaller index)
  const int v1 = static_cast<int>((static_cast<long long>(c + 1) * nvec) / CS);
  int j = static_cast<int>((static_cast<long long>(c) * nvec) / CS) + threadIdx.x;
  const int stride = blockDim.x;
  for (; j + 3 * stride < v1; j += 4 * stride) {
    uint4 w[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) w[q] = rv[j + q * stride];
#pragma unroll
    for (int q = 0; q < 4; ++q) visit(w[q], j + q * stride);
  }
  for (; j < v1; j += stride) visit(rv[j], j);
  if (c == CS - 1)
    for (int k = nvec * 8 + threadIdx.x; k < V; k += stride) {
      const float a = __bfloat162float(row[k]);
      if (arg_better(a, k, bv, bi)) bv = a, bi = k;
    }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (arg_better(ov, oi, bv, bi)) bv = ov, bi = oi;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) sv[warp] = bv, si[warp] = bi;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    bv = lane < nw ? sv[lane] : -__int_as_float(0x7f800000);
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (arg_better(ov, oi, bv, bi)) bv = ov, bi = oi;
    }
    if (lane == 0) cta_v = bv, cta_i = bi;
  }
  if (CS > 1) cluster_sync_all();  // every CTA's winner is in its shared memory
  if (threadIdx.x == 0 && c == 0) {
    bv = cta_v;
    bi = cta_i;
    for (int q = 1; q < CS; ++q) {
      const float ov = ld_dsmem_f32(mapa_u32(smem_u32(&cta_v), q));
      const int oi = __float_as_int(ld_dsmem_f32(mapa_u32(smem_u32(&cta_i), q)));
      if (arg_better(ov, oi, bv, bi)) bv = ov, bi = oi;
    }
    if (out) out[r] = bi;
    if (keys) {
      // (value, lowest index) as one integer: the largest key over vocabulary shards is
      // the global first maximum.  -0 becomes +0 (numpy ranks them equal, so the lower
      // index must decide) and every NaN one positive NaN above +inf (numpy.argmax takes
      // the first NaN, whatever its sign or payload).
      // The value's bits are mapped to an order-preserving unsigned word, then the top
      // bit is flipped so that the keys also order correctly as SIGNED int64 (the
      // allreduce-MAX compares int64): a shard whose maximum is negative ranks below one
      // whose maximum is positive.
      uint32_t u = __float_as_uint(bv);
      if (bv != bv) u = 0x7fc00000u;
      else if (u == 0x80000000u) u = 0u;
      u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
      u ^= 0x80000000u;
      const uint32_t idx = static_cast<uint32_t>(bi + index_offset);
      keys[r] = static_cast<long long>((static_cast<unsigned long long>(u) << 32) | (0xFFFFFFFFu - idx));
    }
  }
  if (CS > 1) cluster_sync_all();  // no CTA leaves while rank 0 may still read its winner
}

__global__ void key_to_token_kernel(const long long* __restrict__ keys, int rows, int* __restrict__ tokens) {
  pdl_launch_dependents();
  pdl_wait();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r < rows)
    tokens[r] = static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(static_cast<unsigned long long>(keys[r]) & 0xFFFFFFFFull));
}

// ---- residual add of a reduced fp32 delta: h = bf16(h + bf16(delta)), plus the
// per-128-column-tile sums of squares of the new h (the next norm prologue's input) ----
__global__ void residual_add_kernel(__nv_bfloat16* __restrict__ h, const float* __restrict__ delta, int rows, int H,
                                    float* __restrict__ ss_out) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float red[4][32];
  const int tile = blockIdx.x, c = threadIdx.x, lane = c & 31, warp = c >> 5;
  const int col = tile * 128 + c;
  for (int r = 0; r < 32; ++r) {
    float ss = 0.f;
    if (r < rows) {
      const size_t i = static_cast<size_t>(r) * H + col;
      const float x = bf16r(__bfloat162float(h[i]) + bf16r(delta[i]));
      h[i] = __float2bfloat16_rn(x);
      ss = x * x;
    }
    ss = warp_sum(ss);
    if (lane == 0) red[warp][r] = ss;
  }
  __syncthreads();
  if (c < 32) ss_out[tile * 32 + c] = (c < rows) ? (red[0][c] + red[1][c]) + (red[2][c] + red[3][c]) : 0.f;
}

// ------------------------------------------------------------------------------------
static int check_launch(const char* what, cudaError_t e0 = cudaSuccess) {
  cudaError_t e = e0 != cudaSuccess ? e0 : cudaGetLastError();
  if (e != cudaSuccess) return fail(kStatusCuda, "%s launch: %s", what, cudaGetErrorString(e));
  return kStatusOk;
}

int embed(cudaStream_t st, int rows, int V, int H, const void* table, const int* ids, void* out, int* err) {
  if (!table || !ids || !out) return fail(kStatusArg, "embed: null pointer");
  if (rows <= 0 || H <= 0 || V <= 0 || H % 8) return fail(kStatusArg, "embed: bad size (H must be a multiple of 8)");
  const cudaError_t le = launch_pdl(embed_kernel, dim3(rows), dim3(128), 0, st, dim3(0), static_cast<const __nv_bfloat16*>(table), ids, V, H,
                                     static_cast<__nv_bfloat16*>(out), err);
  return check_launch("embed", le);
}

int add_rmsnorm(cudaStream_t st, int rows, int H, void* h, const void* delta, const void* w, void* out, float eps) {
  if (!h || !w || !out) return fail(kStatusArg, "add_rmsnorm: null pointer");
  if (rows <= 0 || H <= 0 || H % 2) return fail(kStatusArg, "add_rmsnorm: bad size");
  const cudaError_t le = launch_pdl(add_rmsnorm_kernel, dim3(rows), dim3(256), 0, st, dim3(0), static_cast<__nv_bfloat16*>(h), static_cast<const __nv_bfloat16*>(delta),
                                           static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(out), H,
                                           eps);
  return check_launch("add_rmsnorm", le);
}

int qkv_epilogue(cudaStream_t st, int rows, int rows_per_seq, int Hq, int Hkv, int D, int S, const void* qkv, int ldq,
                 const void* bias, const void* qnw, const void* knw, float eps, const float* inv_freq,
                 const int* positions, const int* write_slot, void* q_out, void* kcache, void* vcache, int* err) {
  if (!qkv || !inv_freq || !positions || !write_slot || !q_out || !kcache || !vcache)
    return fail(kStatusArg, "qkv_epilogue: null pointer");
  if (D != 128) return fail(kStatusUnsupported, "qkv_epilogue: head_dim %d unsupported (only 128)", D);
  if (rows <= 0 || rows_per_seq <= 0 || Hq <= 0 || Hkv <= 0 || S <= 0 || ldq < (Hq + 2 * Hkv) * D)
    return fail(kStatusArg, "qkv_epilogue: bad size");
  if ((Hq + 2 * Hkv) > 65535) return fail(kStatusArg, "qkv_epilogue: too many heads");
  const cudaError_t le = launch_pdl(qkv_epilogue_kernel, dim3(rows), dim3(256), 0, st, dim3(0),
      static_cast<const __nv_bfloat16*>(qkv), ldq, static_cast<const __nv_bfloat16*>(bias),
      static_cast<const __nv_bfloat16*>(qnw), static_cast<const __nv_bfloat16*>(knw), eps, inv_freq, positions,
      write_slot, rows_per_seq, Hq, Hkv, S, static_cast<__nv_bfloat16*>(q_out), static_cast<__nv_bfloat16*>(kcache),
      static_cast<__nv_bfloat16*>(vcache), err);
  return check_launch("qkv_epilogue", le);
}

int row_sumsq(cudaStream_t st, int rows, int H, const void* h, float* ss_out) {
  if (!h || !ss_out) return fail(kStatusArg, "row_sumsq: null pointer");
  if (rows <= 0 || rows > 32 || H <= 0 || H % 2) return fail(kStatusArg, "row_sumsq: bad size (rows 1..32)");
  const cudaError_t le = launch_pdl(row_sumsq_kernel, dim3(rows), dim3(256), 0, st, dim3(0), static_cast<const __nv_bfloat16*>(h), H, ss_out);
  return check_launch("row_sumsq", le);
}

int silu_mul(cudaStream_t st, int rows, int F, const void* gu, void* act) {
  if (!gu || !act) return fail(kStatusArg, "silu_mul: null pointer");
  if (rows <= 0 || F <= 0 || F % 2) return fail(kStatusArg, "silu_mul: bad size");
  const long long n = static_cast<long long>(rows) * F;
  long long blocks = (n / 2 + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  const cudaError_t le = launch_pdl(silu_mul_kernel, dim3(static_cast<int>(blocks)), dim3(256), 0, st, dim3(0), static_cast<const __nv_bfloat16*>(gu), F, n,
                                                             static_cast<__nv_bfloat16*>(act));
  return check_launch("silu_mul", le);
}

// CTAs per row: one per 2048 16-byte vectors, 1..8 (a portable cluster)
static int argmax_cluster(int V) {
  int cs = (V / 8) / 2048;
  return cs < 1 ? 1 : (cs > 8 ? 8 : cs);
}

int argmax_rows(cudaStream_t st, int rows, int V, long long ld, const void* logits, int* out) {
  if (!logits || !out) return fail(kStatusArg, "argmax: null pointer");
  if (rows <= 0 || V <= 0 || ld < V) return fail(kStatusArg, "argmax: bad size");
  if ((ld % 8) || (reinterpret_cast<uintptr_t>(logits) & 15))
    return fail(kStatusArg, "argmax: rows must be 16-byte aligned (ld % 8 == 0)");
  if (rows > 65535) return fail(kStatusArg, "argmax: %d rows exceed 65535", rows);
  const int cs = argmax_cluster(V);
  const cudaError_t le = launch_pdl(argmax_kernel, dim3(cs, rows), dim3(512), 0, st, cs > 1 ? dim3(cs, 1, 1) : dim3(0),
                                    static_cast<const __nv_bfloat16*>(logits), ld, V, out,
                                    static_cast<long long*>(nullptr), 0);
  return check_launch("argmax", le);
}

int argmax_key(cudaStream_t st, int rows, int V, long long ld, const void* logits, int index_offset,
               long long* keys) {
  if (!logits || !keys) return fail(kStatusArg, "argmax_key: null pointer");
  if (rows <= 0 || V <= 0 || ld < V || index_offset < 0) return fail(kStatusArg, "argmax_key: bad size");
  if ((ld % 8) || (reinterpret_cast<uintptr_t>(logits) & 15))
    return fail(kStatusArg, "argmax_key: rows must be 16-byte aligned (ld % 8 == 0)");
  if (rows > 65535) return fail(kStatusArg, "argmax_key: %d rows exceed 65535", rows);
  const int cs = argmax_cluster(V);
  const cudaError_t le = launch_pdl(argmax_kernel, dim3(cs, rows), dim3(512), 0, st, cs > 1 ? dim3(cs, 1, 1) : dim3(0),
                                    static_cast<const __nv_bfloat16*>(logits), ld, V, static_cast<int*>(nullptr),
                                    keys, index_offset);
  return check_launch("argmax_key", le);
}

int key_to_token(cudaStream_t st, int rows, const long long* keys, int* tokens) {
  if (!keys || !tokens) return fail(kStatusArg, "key_to_token: null pointer");
  if (rows <= 0) return fail(kStatusArg, "key_to_token: bad size");
  const cudaError_t le = launch_pdl(key_to_token_kernel, dim3((rows + 127) / 128), dim3(128), 0, st, dim3(0), keys,
                                    rows, tokens);
  return check_launch("key_to_token", le);
}

int residual_add(cudaStream_t st, int rows, int H, void* h, const float* delta, float* ss_out) {
  if (!h || !delta || !ss_out) return fail(kStatusArg, "residual_add: null pointer");
  if (rows <= 0 || rows > 32 || H <= 0 || H % 128) return fail(kStatusArg, "residual_add: rows 1..32, hidden % 128");
  const cudaError_t le = launch_pdl(residual_add_kernel, dim3(H / 128), dim3(128), 0, st, dim3(0),
                                    static_cast<__nv_bfloat16*>(h), delta, rows, H, ss_out);
  return check_launch("residual_add", le);
}

// ---- lossy int8 demotion of cache rows (online_credit_generator.py:643-704) ----------
// Per (layer, sequence, kv head, slot) row of K and of V: absmax int8 round trip with the
// reference's bf16 arithmetic -- every op computed in fp32 and rounded to bf16:
//   scale = bf16(max|x| / 127), q = clip(round_half_even(bf16(x / max(scale, bf16(1e-10)))),
//   -127, 127), x' = bf16(q * scale).  One warp per row, four elements per lane.
__global__ void demote_int8_kernel(__nv_bfloat16* __restrict__ kc, __nv_bfloat16* __restrict__ vc, int B, int Hkv,
                                   int S, const int* __restrict__ slots, int stride, const int* __restrict__ counts,
                                   int* err) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int layer = blockIdx.z, b = blockIdx.y;
  const int n = counts[b] < stride ? counts[b] : stride;
  const int rows = n * Hkv * 2;
  const float tiny = bf16r(1e-10f);
  for (int r = blockIdx.x * (blockDim.x >> 5) + warp; r < rows; r += gridDim.x * (blockDim.x >> 5)) {
    const int which = r % 2, h = (r / 2) % Hkv, j = r / (2 * Hkv);
    const int slot = slots[static_cast<size_t>(b) * stride + j];
    if (slot < 0 || slot >= S) {
      if (lane == 0) set_err(err, kErrIndex);
      continue;
    }
    __nv_bfloat16* row = (which ? vc : kc) + (((static_cast<size_t>(layer) * B + b) * Hkv + h) * S + slot) * 128;
    uint2 raw = *reinterpret_cast<const uint2*>(row + lane * 4);
    float x[4] = {bf16lo(raw.x), bf16hi(raw.x), bf16lo(raw.y), bf16hi(raw.y)};
    float amax = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float scale = bf16r(amax / 127.0f);
    const float den = fmaxf(scale, tiny);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float q = fminf(fmaxf(rintf(bf16r(x[i] / den)), -127.0f), 127.0f);
      x[i] = bf16r(q * scale);
    }
    raw.x = pack_bf16(x[0], x[1]);
    raw.y = pack_bf16(x[2], x[3]);
    *reinterpret_cast<uint2*>(row + lane * 4) = raw;
  }
}

int demote_int8(cudaStream_t st, void* kc, void* vc, int layers, int B, int Hkv, int S, const int* slots, int stride,
                const int* counts, int* err) {
  if (!kc || !vc || !slots || !counts) return fail(kStatusArg, "demote_int8: null pointer");
  if (layers <= 0 || B <= 0 || Hkv <= 0 || S <= 0 || stride <= 0 || layers > 65535 || B > 65535)
    return fail(kStatusArg, "demote_int8: bad size");
  if ((reinterpret_cast<uintptr_t>(kc) | reinterpret_cast<uintptr_t>(vc)) & 7)
    return fail(kStatusArg, "demote_int8: caches must be 8-byte aligned");
  const int rows = stride * Hkv * 2;
  const int blocks = (rows + 7) / 8 < 64 ? (rows + 7) / 8 : 64;
  const cudaError_t le = launch_pdl(demote_int8_kernel, dim3(blocks, B, layers), dim3(256), 0, st, dim3(0),
                                    static_cast<__nv_bfloat16*>(kc), static_cast<__nv_bfloat16*>(vc), B, Hkv, S, slots,
                                    stride, counts, err);
  return check_launch("demote_int8", le);
}

}  // namespace kvbp

// ------------------------------------------------------------------------------------
// C ABI
// ------------------------------------------------------------------------------------
#include "../../include/kvbp.h"

extern "C" {

int kvbp_embed(kvbp_stream_t stream, int32_t rows, int32_t vocab, int32_t hidden, const void* table,
               const int32_t* ids, void* out, int32_t* dev_err) {
  return kvbp::embed(reinterpret_cast<cudaStream_t>(stream), rows, vocab, hidden, table, ids, out, dev_err);
}

int kvbp_add_rmsnorm(kvbp_stream_t stream, int32_t rows, int32_t hidden, void* h, const void* delta, const void* w,
                     void* out, float eps) {
  return kvbp::add_rmsnorm(reinterpret_cast<cudaStream_t>(stream), rows, hidden, h, delta, w, out, eps);
}

int kvbp_row_sumsq(kvbp_stream_t stream, int32_t rows, int32_t hidden, const void* h, float* ss_out) {
  return kvbp::row_sumsq(reinterpret_cast<cudaStream_t>(stream), rows, hidden, h, ss_out);
}

int kvbp_silu_mul(kvbp_stream_t stream, int32_t rows, int32_t ffn, const void* gu, void* act) {
  return kvbp::silu_mul(reinterpret_cast<cudaStream_t>(stream), rows, ffn, gu, act);
}

int kvbp_argmax(kvbp_stream_t stream, int32_t rows, int32_t vocab, int64_t ld, const void* logits, int32_t* out_ids) {
  return kvbp::argmax_rows(reinterpret_cast<cudaStream_t>(stream), rows, vocab, ld, logits, out_ids);
}

int kvbp_argmax_key(kvbp_stream_t stream, int32_t rows, int32_t vocab, int64_t ld, const void* logits,
                    int32_t index_offset, int64_t* keys_out) {
  return kvbp::argmax_key(reinterpret_cast<cudaStream_t>(stream), rows, vocab, ld, logits, index_offset,
                          reinterpret_cast<long long*>(keys_out));
}

int kvbp_key_to_token(kvbp_stream_t stream, int32_t rows, const int64_t* keys, int32_t* tokens) {
  return kvbp::key_to_token(reinterpret_cast<cudaStream_t>(stream), rows, reinterpret_cast<const long long*>(keys),
                            tokens);
}

int kvbp_demote_int8(kvbp_stream_t stream, void* kcache, void* vcache, int32_t layers, int32_t B, int32_t Hkv,
                     int32_t S, const int32_t* slots, int32_t stride, const int32_t* counts, int32_t* dev_err) {
  return kvbp::demote_int8(reinterpret_cast<cudaStream_t>(stream), kcache, vcache, layers, B, Hkv, S, slots, stride,
                           counts, dev_err);
}

int kvbp_residual_add(kvbp_stream_t stream, int32_t rows, int32_t hidden, void* h, const float* delta,
                      float* ss_out) {
  return kvbp::residual_add(reinterpret_cast<cudaStream_t>(stream), rows, hidden, h, delta, ss_out);
}

int kvbp_qkv_rope_scatter(kvbp_stream_t stream, int32_t rows, int32_t rows_per_seq, int32_t Hq, int32_t Hkv,
                          int32_t head_dim, int32_t S, const void* qkv, int32_t ldq, const void* bias,
                          const void* q_norm_w, const void* k_norm_w, float eps, const float* inv_freq,
                          const int32_t* positions, const int32_t* write_slot, void* q_out, void* kcache,
                          void* vcache, int32_t* dev_err) {
  return kvbp::qkv_epilogue(reinterpret_cast<cudaStream_t>(stream), rows, rows_per_seq, Hq, Hkv, head_dim, S, qkv,
                            ldq, bias, q_norm_w, k_norm_w, eps, inv_freq, positions, write_slot, q_out, kcache,
                            vcache, dev_err);
}

}  // extern "C"
