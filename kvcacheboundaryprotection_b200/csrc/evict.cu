// Eviction bookkeeping of the capped KV cache: per-step score update, slot allocation
// for the new position, cadence victim selection (structural prefix/suffix protection +
// policy top-k + hard-capacity guardrail), and the step-0 selection/compaction after
// prefill.  Every decision is integer or float64 arithmetic done exactly as the
// reference's Python does it, so victims are bit-exact given equal scores:
//
//  * score update      src/counterfact_kv_eviction/kv_coupled_generator.py:504-516
//  * cadence + count   kv_coupled_generator.py:549-586 (_maybe_evict)
//  * hard-cap fallback kv_coupled_generator.py:588-604
//  * protection        scripts/run_v3_jax.py:113-136 (ProtectedPolicyWrapper)
//  * policy keys       src/counterfact_kv_eviction/policies.py:181-196 (lru),
//                      :1190-1218 (h2o), :1267-1335 (snapkv, snapkv_faithful),
//                      :1338-1367 (h2o_faithful), :1375-1449 (adakv, quest),
//                      :1221-1264 (streamingllm)
//
// Slot layout rule (the reference has none; defined here): retained prompt positions
// fill slots 0..R-1 in ascending position order after step 0; each decode step's new
// position takes the lowest free slot before that step's eviction; victims' slots
// become free.
#include "common.cuh"
#include "kvbp_internal.h"

namespace kvbp {

struct SeqState {
  int* slot_pos;     // [S]   position held by the slot, -1 = free
  int* insert_step;  // [S]
  int* last_access;  // [S]
  int* access_count; // [S]
  float* attn;       // [S]
  float* max_attn;   // [S]
  double* cumul;     // [S]
  float* prefill;    // [S]
  uint32_t* posmap;  // [W] bit p set <=> position p retained
};

struct StateArgs {
  int B, S, W;
  int* slot_pos;
  int* insert_step;
  int* last_access;
  int* access_count;
  float* attn;
  float* max_attn;
  double* cumul;
  float* prefill;
  uint32_t* posmap;
  __device__ SeqState seq(int b) const {
    const size_t o = static_cast<size_t>(b) * S;
    return SeqState{slot_pos + o, insert_step + o, last_access + o, access_count + o, attn + o,
                    max_attn + o, cumul + o,     prefill + o,     posmap + static_cast<size_t>(b) * W};
  }
};

// Composite eviction key of one position (smaller = evicted first).
__device__ __forceinline__ Key3 policy_key(int policy, int step, int pos, int ins, int last, float attn, float maxa,
                                           double cumul, float pre, int* err) {
  const uint64_t li = (static_cast<uint64_t>(ord_i32(last)) << 32) | ord_i32(ins);
  const uint64_t lo = static_cast<uint64_t>(ord_i32(last)) << 32;
  const uint64_t lx = lex_code(pos);
  // Python max(attention_score, max_attention_score)
  const double sig = (static_cast<double>(maxa) > static_cast<double>(attn)) ? static_cast<double>(maxa)
                                                                              : static_cast<double>(attn);
  double keep = 0.0;
  switch (policy) {
    case kPolicyLRU:
    case kPolicyStreamingLLM:
      return Key3{li, lx, 0};
    case kPolicyH2OFaithful:
      keep = cumul;
      break;
    case kPolicyH2O: {
      const double recent = (step - last) <= 64 ? 1.0 : 0.0;
      keep = __dadd_rn(__dadd_rn(__dmul_rn(0.7, cumul), __dmul_rn(0.1, sig)), __dmul_rn(1.0, recent));
      break;
    }
    case kPolicySnapKV:
      keep = __dadd_rn(cumul, sig);
      break;
    case kPolicySnapKVFaithful:
      keep = static_cast<double>(pre);
      break;
    case kPolicyAdaKV:
      keep = __dadd_rn(cumul, __dmul_rn(0.5, static_cast<double>(maxa)));
      break;
    case kPolicyQuest:
      keep = static_cast<double>(attn);
      break;
    default:
      return Key3{li, lx, 0};
  }
  if (keep != keep) set_err(err, kErrNanScore);
  if (policy == kPolicyH2OFaithful || policy == kPolicyH2O) return Key3{ord_f64(keep), li, lx};
  return Key3{ord_f64(keep), lo, lx};
}

__device__ __forceinline__ Key3 sink_key(int pos, int ins) { return Key3{ord_i32(ins), lex_code(pos), 0}; }

__device__ __forceinline__ Key3 hardcap_key(int pos, int ins, int last) {
  return Key3{(static_cast<uint64_t>(ord_i32(last)) << 32) | ord_i32(ins), static_cast<uint64_t>(pos), 0};
}

// ------------------------------------------------------------------------------------
// block-level helpers (blockDim.x == kEvictThreads)
// ------------------------------------------------------------------------------------
constexpr int kEvictThreads = 512;
constexpr int kMaxPerThread = 32;  // taken-bitmask width: S <= 16384

__device__ int block_sum_int(int v, int* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  int t = lane < (kEvictThreads >> 5) ? red[lane] : 0;
#pragma unroll
  for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return t;
}

__device__ int block_min_int(int v, int* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  int t = lane < (kEvictThreads >> 5) ? red[lane] : 0x7fffffff;
#pragma unroll
  for (int o = 16; o; o >>= 1) t = min(t, __shfl_xor_sync(0xffffffffu, t, o));
  return t;
}

__device__ float block_max_float(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
#pragma unroll
  for (int o = 16; o; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
  return t;
}

struct KeySlot {
  Key3 k;
  int slot;
};

__device__ __forceinline__ bool ks_less(const KeySlot& x, const KeySlot& y) {
  if (key_less(x.k, y.k)) return true;
  if (key_less(y.k, x.k)) return false;
  return x.slot < y.slot;
}

__device__ __forceinline__ KeySlot shfl_ks(const KeySlot& v, int o) {
  KeySlot r;
  r.k.a = __shfl_xor_sync(0xffffffffu, v.k.a, o);
  r.k.b = __shfl_xor_sync(0xffffffffu, v.k.b, o);
  r.k.c = __shfl_xor_sync(0xffffffffu, v.k.c, o);
  r.slot = __shfl_xor_sync(0xffffffffu, v.slot, o);
  return r;
}

// Block argmin of (key, slot); every thread receives the winner.
__device__ KeySlot block_argmin(KeySlot v, KeySlot* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const KeySlot w = shfl_ks(v, o);
    if (ks_less(w, v)) v = w;
  }
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  KeySlot t = lane < (kEvictThreads >> 5) ? red[lane] : KeySlot{key_max(), 0x7fffffff};
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const KeySlot w = shfl_ks(t, o);
    if (ks_less(w, t)) t = w;
  }
  return t;
}

// One round of block top-k: the smallest (key, slot) among this thread's strided
// slots i = tid + j * kEvictThreads that pass ``elig`` and are not yet taken (bit j of
// ``taken``), reduced over the block.  The owner of the winner marks it taken.
template <typename KeyF, typename EligF>
__device__ KeySlot take_min(int S, uint32_t& taken, KeyF keyf, EligF elig, KeySlot* red) {
  KeySlot best{key_max(), 0x7fffffff};
  for (int j = 0, i = threadIdx.x; i < S; ++j, i += kEvictThreads) {
    if ((taken >> j) & 1u) continue;
    if (!elig(i)) continue;
    const KeySlot c{keyf(i), i};
    if (ks_less(c, best)) best = c;
  }
  const KeySlot w = block_argmin(best, red);
  if (w.slot != 0x7fffffff && (w.slot % kEvictThreads) == static_cast<int>(threadIdx.x))
    taken |= 1u << (w.slot / kEvictThreads);
  return w;
}

// This thread's smallest (key, slot) among its eligible slots not yet taken.
template <typename KeyF, typename EligF>
__device__ KeySlot local_min(int S, uint32_t taken, KeyF keyf, EligF elig) {
  KeySlot best{key_max(), 0x7fffffff};
  for (int j = 0, i = threadIdx.x; i < S; ++j, i += kEvictThreads) {
    if ((taken >> j) & 1u) continue;
    if (!elig(i)) continue;
    const KeySlot c{keyf(i), i};
    if (ks_less(c, best)) best = c;
  }
  return best;
}

// Position of the k-th (0-based) set bit of the W-word bitmap; INT_MAX if none.
// Executed by one full warp.
__device__ int select_bit_warp(const uint32_t* words, int W, int k) {
  const int lane = threadIdx.x & 31;
  int base = 0;
  for (int w0 = 0; w0 < W; w0 += 32) {
    const uint32_t word = (w0 + lane < W) ? words[w0 + lane] : 0u;
    const int c = __popc(word);
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    const int total = __shfl_sync(0xffffffffu, incl, 31);
    if (base + total > k) {
      const int excl = incl - c;
      int found = 0x7fffffff;
      if (base + excl <= k && k < base + incl) {
        uint32_t m = word;
        for (int j = 0; j < k - base - excl; ++j) m &= m - 1;
        found = (w0 + lane) * 32 + (__ffs(m) - 1);
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) found = min(found, __shfl_xor_sync(0xffffffffu, found, o));
      return found;
    }
    base += total;
  }
  return 0x7fffffff;
}

// ------------------------------------------------------------------------------------
// score update: kv_coupled_generator.py:504-516, over the valid slots of one sequence.
// The slots of a sequence are split over a cluster of CTAs: each forms the maximum of
// its share, the CTAs exchange them through DSMEM (the access threshold needs the
// sequence-wide maximum), then each updates its share.
// ------------------------------------------------------------------------------------
constexpr int kScoreThreads = 256;

__global__ void __launch_bounds__(kScoreThreads) score_update_kernel(StateArgs st, const int* __restrict__ seq_step,
                                                                     float* __restrict__ step_score, int* err) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float red[32];
  __shared__ float cta_max;
  const int b = blockIdx.y, CS = gridDim.x;
  uint32_t rank;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  const int lo = (static_cast<int>(rank) * st.S) / CS, hi = ((static_cast<int>(rank) + 1) * st.S) / CS;
  const SeqState s = st.seq(b);
  const int* __restrict__ spos = s.slot_pos;
  float* __restrict__ sc = step_score + static_cast<size_t>(b) * st.S;
  float mx = 0.f;
  for (int i = lo + threadIdx.x; i < hi; i += kScoreThreads)
    if (spos[i] >= 0) mx = fmaxf(mx, sc[i]);
  mx = block_max_float(mx, red);
  if (threadIdx.x == 0) cta_max = mx;
  cluster_sync_all();
  const uint32_t local = smem_u32(&cta_max);
  float pm[8];  // every peer's maximum loaded before the first compare (CS <= 8)
#pragma unroll
  for (int q = 0; q < 8; ++q) pm[q] = q < CS ? ld_dsmem_f32(mapa_u32(local, q)) : 0.f;
  float gmx = 0.f;
#pragma unroll
  for (int q = 0; q < 8; ++q) gmx = fmaxf(gmx, pm[q]);
  const float thr = static_cast<float>(0.05 * static_cast<double>(gmx));
  const int step = seq_step[b];
  float* __restrict__ attn = s.attn;
  float* __restrict__ maxa = s.max_attn;
  double* __restrict__ cumul = s.cumul;
  int* __restrict__ last = s.last_access;
  int* __restrict__ cnt = s.access_count;
  for (int i = lo + threadIdx.x; i < hi; i += kScoreThreads) {
    const float ks = sc[i];
    if (spos[i] >= 0) {
      if (ks != ks) set_err(err, kErrNanScore);
      attn[i] = ks;
      maxa[i] = fmaxf(maxa[i], ks);
      cumul[i] = __dadd_rn(cumul[i], static_cast<double>(ks));
      if (ks > thr) {
        last[i] = step;
        cnt[i] += 1;
      }
    }
    sc[i] = 0.f;
  }
  cluster_sync_all();  // peers have read cta_max before this CTA leaves
}

// ------------------------------------------------------------------------------------
// append the new position + cadence eviction (one block per sequence)
// ------------------------------------------------------------------------------------
struct AppendArgs {
  StateArgs st;
  int C, E, policy, protect, n_prefix, n_suffix, decode_regime;
  int* seq_step;    // [B] incremented here
  int* next_pos;    // [B] incremented here
  int* cur_pos;     // [B] out: position of the token being forwarded
  int* write_slot;  // [B] out: its slot, -1 if it was evicted at this step
  const int* tokens;    // [B] token sampled for this step (may be null)
  int* token_log;       // [B][log_steps] (may be null)
  int log_steps;
  int* evlog;           // [B][evcap] evicted positions in eviction order
  int* evcount;         // [B]
  int evcap;
  int* retained_log;    // [B][log_steps + 1] retained count after step s (may be null)
  int* err;
  // victims chosen on the host (the random policy): [B][ext_stride] positions, ext_n [B]
  const int* ext_pos;
  const int* ext_n;
  int ext_stride;
  int no_hardcap;  // listed victims only: skip the hard-capacity guardrail (per-head mode has none)
  // previous step's score update run first (null upd_score: none): the scores the layers of
  // that step max-accumulated into upd_score [B][S]; upd_pending [B] = 1 once a step's
  // scores are pending (the kernel sets it, the first decode step after prefill has 0)
  float* upd_score;
  int* upd_pending;
  int pm_smem;   // the position bitmap fits in shared memory after the victim list
  int key_smem;  // byte offset of the [S] composite keys in shared memory (0: local memory)
};

__device__ void log_victim(const AppendArgs& a, int b, int pos) {
  int n = a.evcount[b];
  if (n < a.evcap)
    a.evlog[static_cast<size_t>(b) * a.evcap + n] = pos;
  else
    set_err(a.err, kErrLogOverflow);
  a.evcount[b] = n + 1;
}

__global__ void __launch_bounds__(kEvictThreads) append_evict_kernel(AppendArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ int s_vict[];  // [S] victim slots of this call, in eviction order
  __shared__ int red_i[32];
  __shared__ KeySlot red_k[32];
  __shared__ int sh[8];
  const int b = blockIdx.x, tid = threadIdx.x;
  const int S = a.st.S;
  SeqState s = a.st.seq(b);
  if (tid == 0) {
    sh[0] = a.seq_step[b] + 1;
    sh[1] = a.next_pos[b];
    sh[6] = a.upd_score ? a.upd_pending[b] : 0;
  }
  // one pass over the slot positions (kU slots per thread with their loads in flight
  // together: one block per sequence walks S slots, and a loop of dependent loads would pay
  // the memory latency per slot) finds the lowest free slot and, for a pending score
  // update, the maximum of the previous step's scores over the retained slots
  constexpr int kU = 10;  // one iteration per pass up to 5120 slots
  float* sc = a.upd_score ? a.upd_score + static_cast<size_t>(b) * S : nullptr;
  // up to kU * kEvictThreads slots the update's other inputs are loaded in the same pass
  // and kept in registers, so the update itself needs no second round trip
  const bool one_pass = S <= kU * kEvictThreads;
  int mine = 0x7fffffff;
  float mx = 0.f;
  float v[kU], ma[kU];
  double cu[kU];
  int ps[kU], cn[kU];
  for (int i0 = tid; i0 < S; i0 += kU * kEvictThreads) {
    const bool keep = sc && one_pass;
#pragma unroll
    for (int k = 0; k < kU; ++k) {
      const int i = i0 + k * kEvictThreads;
      const bool in = i < S;
      ps[k] = in ? s.slot_pos[i] : 0;
      v[k] = (sc && in) ? sc[i] : 0.f;
      ma[k] = (keep && in) ? s.max_attn[i] : 0.f;
      cu[k] = (keep && in) ? s.cumul[i] : 0.0;
      cn[k] = (keep && in) ? s.access_count[i] : 0;
    }
#pragma unroll
    for (int k = 0; k < kU; ++k) {
      const int i = i0 + k * kEvictThreads;
      if (i >= S) continue;
      if (ps[k] >= 0)
        mx = fmaxf(mx, v[k]);
      else if (i < mine)
        mine = i;
    }
  }
  __syncthreads();
  const int step = sh[0], pos = sh[1];

  if (sc) {
    // ---- the previous step's score update (kv_coupled_generator.py:504-516) over the
    // slots that step attended, before this step's append and eviction, as the reference
    // orders them; the same arithmetic as score_update_kernel --------------------------
    if (sh[6]) {
      __shared__ float red_f[32];
      mx = block_max_float(mx, red_f);
      const float thr = static_cast<float>(0.05 * static_cast<double>(mx));
      const int prev = step - 1;
      auto update = [&](int i, int p_i, float ks, float ma_i, double cu_i, int cn_i) {
        if (p_i >= 0) {
          if (ks != ks) set_err(a.err, kErrNanScore);
          s.attn[i] = ks;
          s.max_attn[i] = fmaxf(ma_i, ks);
          s.cumul[i] = __dadd_rn(cu_i, static_cast<double>(ks));
          if (ks > thr) {
            s.last_access[i] = prev;
            s.access_count[i] = cn_i + 1;
          }
        }
        sc[i] = 0.f;  // this step's layers accumulate from zero
      };
      if (one_pass) {
#pragma unroll
        for (int k = 0; k < kU; ++k) {
          const int i = tid + k * kEvictThreads;
          if (i < S) update(i, ps[k], v[k], ma[k], cu[k], cn[k]);
        }
      } else {
        for (int i0 = tid; i0 < S; i0 += kU * kEvictThreads) {
          float ks2[kU], ma2[kU];
          double cu2[kU];
          int ps2[kU], cn2[kU];
#pragma unroll
          for (int k = 0; k < kU; ++k) {
            const int i = i0 + k * kEvictThreads;
            const bool in = i < S;
            ps2[k] = in ? s.slot_pos[i] : -1;
            ks2[k] = in ? sc[i] : 0.f;
            ma2[k] = in ? s.max_attn[i] : 0.f;
            cu2[k] = in ? s.cumul[i] : 0.0;
            cn2[k] = in ? s.access_count[i] : 0;
          }
#pragma unroll
          for (int k = 0; k < kU; ++k) {
            const int i = i0 + k * kEvictThreads;
            if (i < S) update(i, ps2[k], ks2[k], ma2[k], cu2[k], cn2[k]);
          }
        }
      }
    } else {
      for (int i = tid; i < S; i += kEvictThreads) sc[i] = 0.f;
    }
  }

  // lowest free slot (found in the pass above)
  const int slot = block_min_int(mine, red_i);
  if (slot == 0x7fffffff) {
    if (tid == 0) {
      set_err(a.err, kErrNoFreeSlot);
      a.write_slot[b] = -1;
      a.cur_pos[b] = pos;
      a.seq_step[b] = step;
      a.next_pos[b] = pos + 1;
      if (a.upd_score) a.upd_pending[b] = 1;
    }
    return;
  }
  if (tid == 0) {
    s.slot_pos[slot] = pos;
    s.insert_step[slot] = step;
    s.last_access[slot] = step;
    s.access_count[slot] = 1;
    s.attn[slot] = 0.f;
    s.max_attn[slot] = 0.f;
    s.cumul[slot] = 0.0;
    s.prefill[slot] = 0.f;
    if ((pos >> 5) < a.st.W)
      s.posmap[pos >> 5] |= 1u << (pos & 31);
    else
      set_err(a.err, kErrIndex);
    a.seq_step[b] = step;
    a.next_pos[b] = pos + 1;
    a.cur_pos[b] = pos;
    if (a.token_log && a.tokens && step <= a.log_steps)
      a.token_log[static_cast<size_t>(b) * a.log_steps + step - 1] = a.tokens[b];
  }
  __syncthreads();

  int n_vict = 0;
  if (a.decode_regime && step % a.E == 0) {
    // ---- retained count and evict_count -----------------------------------------
    int cnt = 0;
    for (int i = tid; i < S; i += kEvictThreads) cnt += s.slot_pos[i] >= 0;
    const int R = block_sum_int(cnt, red_i);
    const int k_req = R - a.C > 0 ? R - a.C : 0;
    // ---- structural protection (ProtectedPolicyWrapper) ---------------------------
    int thr_lo = -1, thr_hi = 0x7fffffff;  // eligible <=> thr_lo <= pos < thr_hi
    bool none = false;
    if (a.protect) {
      if (k_req <= 0 || a.n_suffix == 0 || a.n_suffix >= R || a.n_prefix >= R) {
        none = true;  // wrapper returns [] (n_suffix == 0 slices the whole list)
      } else {
        // the position bitmap staged in shared memory first (all threads, loads in flight
        // together): the two selecting warps walk it 32 words per step, which from global
        // memory was one dependent round trip per step
        const uint32_t* pm = s.posmap;
        if (a.pm_smem) {
          uint32_t* spm = reinterpret_cast<uint32_t*>(s_vict + S);
          for (int w0 = tid; w0 < a.st.W; w0 += 4 * kEvictThreads) {
            uint32_t v4[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int w = w0 + q * kEvictThreads;
              v4[q] = w < a.st.W ? s.posmap[w] : 0u;
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int w = w0 + q * kEvictThreads;
              if (w < a.st.W) spm[w] = v4[q];
            }
          }
          __syncthreads();
          pm = spm;
        }
        const int warp = tid >> 5;
        if (warp == 0) {
          const int v = select_bit_warp(pm, a.st.W, a.n_prefix);
          if ((tid & 31) == 0) sh[2] = v;
        } else if (warp == 1) {
          const int v = select_bit_warp(pm, a.st.W, R - a.n_suffix);
          if ((tid & 31) == 0) sh[3] = v;
        }
        __syncthreads();
        thr_lo = sh[2];
        thr_hi = sh[3];
      }
    }
    __syncthreads();
    int k = 0;
    if (a.ext_pos) {
      // victims listed by the host, in its order: look up each position's slot
      int nl = a.ext_n[b];
      nl = nl < a.ext_stride ? nl : a.ext_stride;
      for (int j = 0; j < nl; ++j) {
        const int p = a.ext_pos[static_cast<size_t>(b) * a.ext_stride + j];
        int hit = 0x7fffffff;
        for (int i = tid; i < S; i += kEvictThreads)
          if (s.slot_pos[i] == p && p >= 0) {
            hit = i;
            break;
          }
        const int sl = block_min_int(hit, red_i);
        if (tid == 0) {
          bool dup = false;
          for (int q = 0; q < n_vict; ++q) dup |= s_vict[q] == sl;
          if (sl == 0x7fffffff)
            set_err(a.err, kErrIndex);
          else if (!dup)
            s_vict[n_vict] = sl;
          sh[5] = (sl != 0x7fffffff && !dup) ? 1 : 0;
        }
        __syncthreads();
        n_vict += sh[5];
        __syncthreads();
      }
    } else if (!none && k_req > 0) {
      auto elig = [&](int i) {
        const int p = s.slot_pos[i];
        return p >= 0 && p >= thr_lo && p < thr_hi;
      };
      int ne = 0;
      for (int i = tid; i < S; i += kEvictThreads) ne += elig(i);
      const int n_elig = block_sum_int(ne, red_i);
      k = k_req < n_elig ? k_req : n_elig;
      if (a.policy == kPolicyStreamingLLM && k > 0) {
        // sink: the 4 smallest by (insert_step, str(pos)); recent: the C-4 largest by
        // (last, insert, str(pos)); candidates = the rest, or everything if empty.
        auto skey = [&](int i) { return sink_key(s.slot_pos[i], s.insert_step[i]); };
        auto okey = [&](int i) {
          return policy_key(kPolicyLRU, step, s.slot_pos[i], s.insert_step[i], s.last_access[i], 0.f, 0.f, 0.0, 0.f,
                            a.err);
        };
        uint32_t taken = 0;
        const int n_sink = n_elig < 4 ? n_elig : 4;
        for (int r = 0; r < n_sink; ++r) {
          const KeySlot w = take_min(S, taken, skey, elig, red_k);
          if (tid == 0) sh[4 + r] = w.slot;
        }
        __syncthreads();
        const int recent_n = a.C - 4 > 0 ? a.C - 4 : 0;
        const int n_notrecent = n_elig - recent_n > 0 ? n_elig - recent_n : 0;
        taken = 0;
        for (int r = 0; r < n_notrecent && n_vict < k; ++r) {
          const KeySlot w = take_min(S, taken, okey, elig, red_k);
          bool is_sink = false;
          for (int j = 0; j < n_sink; ++j) is_sink |= (sh[4 + j] == w.slot);
          if (!is_sink) {
            if (tid == 0) s_vict[n_vict] = w.slot;
            ++n_vict;
          }
        }
        if (n_vict == 0) {  // no candidates outside sink/recent: rank all eligible
          taken = 0;
          for (int r = 0; r < k; ++r) {
            const KeySlot w = take_min(S, taken, okey, elig, red_k);
            if (tid == 0) s_vict[n_vict] = w.slot;
            ++n_vict;
          }
        }
      } else if (k > 0) {
        // k rounds of block argmin.  Each thread forms the keys of its slots once (the loads
        // of kQ slots in flight together) and keeps them -- in shared memory when they fit
        // (a local array of 512 threads does not stay in L1); a thread's minimum changes only
        // when it owned a round's winner, and then it rescans its cached keys (a rescan from
        // global memory put every round's latency on the critical path: 4.7 us per round at
        // 4104 slots).  A warp-first top-k (each warp its k smallest, then one warp over the
        // 16 x k candidates) measured slower than these block rounds.
        Key3* kcs = a.key_smem ? reinterpret_cast<Key3*>(reinterpret_cast<uint8_t*>(s_vict) + a.key_smem) : nullptr;
        Key3 kc_local[kMaxPerThread];
        auto kc = [&](int j) -> Key3& { return kcs ? kcs[tid + j * kEvictThreads] : kc_local[j]; };
        uint32_t skip = 0;  // bit j: slot tid + j * kEvictThreads ineligible or already taken
        const int nj = tid < S ? (S - tid + kEvictThreads - 1) / kEvictThreads : 0;
        // only the fields the policy's key reads are loaded
        const int pol = a.policy;
        const bool need_cu = pol == kPolicyH2OFaithful || pol == kPolicyH2O || pol == kPolicySnapKV || pol == kPolicyAdaKV;
        const bool need_at = pol == kPolicyH2O || pol == kPolicySnapKV || pol == kPolicyQuest;
        const bool need_ma = pol == kPolicyH2O || pol == kPolicySnapKV || pol == kPolicyAdaKV;
        const bool need_pr = pol == kPolicySnapKVFaithful;
        constexpr int kQ = 4;  // slots per batch of loads
        for (int j0 = 0; j0 < nj; j0 += kQ) {
          int pp[kQ], ins[kQ], lst[kQ];
          float at[kQ], ma[kQ], pr[kQ];
          double cu[kQ];
#pragma unroll
          for (int q = 0; q < kQ; ++q) {
            const int j = j0 + q, i = tid + j * kEvictThreads;
            const bool in = j < nj;
            pp[q] = in ? s.slot_pos[i] : -1;
            ins[q] = in ? s.insert_step[i] : 0;
            lst[q] = in ? s.last_access[i] : 0;
            at[q] = (in && need_at) ? s.attn[i] : 0.f;
            ma[q] = (in && need_ma) ? s.max_attn[i] : 0.f;
            pr[q] = (in && need_pr) ? s.prefill[i] : 0.f;
            cu[q] = (in && need_cu) ? s.cumul[i] : 0.0;
          }
#pragma unroll
          for (int q = 0; q < kQ; ++q) {
            const int j = j0 + q;
            if (j >= nj) break;
            const bool e = pp[q] >= 0 && pp[q] >= thr_lo && pp[q] < thr_hi;
            if (e)
              kc(j) = policy_key(a.policy, step, pp[q], ins[q], lst[q], at[q], ma[q], cu[q], pr[q], a.err);
            else
              skip |= 1u << j;
          }
        }
        auto cached_min = [&]() {
          KeySlot best{key_max(), 0x7fffffff};
          for (int j = 0; j < nj; ++j) {
            if ((skip >> j) & 1u) continue;
            const KeySlot c{kc(j), tid + j * kEvictThreads};
            if (ks_less(c, best)) best = c;
          }
          return best;
        };
        KeySlot mine = cached_min();
        for (int r = 0; r < k; ++r) {
          const KeySlot w = block_argmin(mine, red_k);
          if (w.slot != 0x7fffffff && (w.slot % kEvictThreads) == tid) {
            skip |= 1u << (w.slot / kEvictThreads);
            mine = cached_min();
          }
          if (tid == 0) s_vict[n_vict] = w.slot;
          ++n_vict;
        }
      }
    }
    __syncthreads();
    if (tid == 0) {
      for (int j = 0; j < n_vict; ++j) {
        const int sl = s_vict[j];
        const int p = s.slot_pos[sl];
        log_victim(a, b, p);
        s.posmap[p >> 5] &= ~(1u << (p & 31));
        s.slot_pos[sl] = -1;
      }
    }
    __syncthreads();
    // ---- hard-capacity guardrail ------------------------------------------------
    const int overflow = a.no_hardcap ? 0 : (R - n_vict) - a.C;
    if (overflow > 0) {
      auto live = [&](int i) { return s.slot_pos[i] >= 0; };
      auto hkey = [&](int i) { return hardcap_key(s.slot_pos[i], s.insert_step[i], s.last_access[i]); };
      uint32_t taken = 0;
      for (int r = 0; r < overflow; ++r) {
        const KeySlot w = take_min(S, taken, hkey, live, red_k);
        if (tid == 0) s_vict[r] = w.slot;
      }
      __syncthreads();
      if (tid == 0) {
        for (int j = 0; j < overflow; ++j) {
          const int sl = s_vict[j];
          const int p = s.slot_pos[sl];
          log_victim(a, b, p);
          s.posmap[p >> 5] &= ~(1u << (p & 31));
          s.slot_pos[sl] = -1;
        }
      }
      n_vict += overflow;
    }
    __syncthreads();
    if (tid == 0 && a.retained_log && step <= a.log_steps)
      a.retained_log[static_cast<size_t>(b) * (a.log_steps + 1) + step] = R - n_vict;
  } else if (tid == 0 && a.retained_log && step <= a.log_steps) {
    // retained count = previous count + 1 (no eviction this step)
    const size_t o = static_cast<size_t>(b) * (a.log_steps + 1);
    a.retained_log[o + step] = a.retained_log[o + step - 1] + 1;
  }
  __syncthreads();
  if (tid == 0) a.write_slot[b] = (s.slot_pos[slot] == pos) ? slot : -1;
  if (tid == 0 && a.upd_score) a.upd_pending[b] = 1;  // this step's scores are applied by the next call
}

// ------------------------------------------------------------------------------------
// step 0: rank-based selection over the prompt positions 0..P-1 (all retained)
// ------------------------------------------------------------------------------------
struct PrefillSelArgs {
  int B, P, policy;
  int n_prefix, n_suffix, protect_all;  // protected <=> pos < n_prefix || pos >= P - n_suffix
  int lo, hi;                           // victim <=> lo <= rank < hi; victim index = rank - lo
  const float* scores;                  // [B][P] prefill scores (null = all zero)
  uint8_t* victim;                      // [B][P] out
  int* evlog;                           // [B][evcap]
  int evcap;
  int* err;
};

__device__ __forceinline__ bool pf_eligible(const PrefillSelArgs& a, int p) {
  return !a.protect_all && p >= a.n_prefix && p < a.P - a.n_suffix;
}

__device__ __forceinline__ Key3 pf_key(const PrefillSelArgs& a, int b, int p) {
  const float sc = a.scores ? a.scores[static_cast<size_t>(b) * a.P + p] : 0.f;
  // step-0 metadata: insert = last = 0, attn = max = prefill = score, cumul = score
  return policy_key(a.policy, 0, p, 0, 0, sc, sc, static_cast<double>(sc), sc, a.err);
}

__global__ void __launch_bounds__(256) prefill_rank_kernel(PrefillSelArgs a) {
  __shared__ Key3 tile[256];
  __shared__ uint8_t tile_ok[256];
  const int b = blockIdx.y;
  const int i = blockIdx.x * 256 + threadIdx.x;
  const bool mine_ok = i < a.P && pf_eligible(a, i);
  const Key3 mk = mine_ok ? pf_key(a, b, i) : key_max();
  int rank = 0;
  for (int j0 = 0; j0 < a.P; j0 += 256) {
    const int j = j0 + threadIdx.x;
    const bool ok = j < a.P && pf_eligible(a, j);
    tile_ok[threadIdx.x] = ok;
    tile[threadIdx.x] = ok ? pf_key(a, b, j) : key_max();
    __syncthreads();
    if (mine_ok) {
      const int n = a.P - j0 < 256 ? a.P - j0 : 256;
      for (int t = 0; t < n; ++t) rank += (tile_ok[t] && key_less(tile[t], mk));
    }
    __syncthreads();
  }
  if (i < a.P) {
    const bool v = mine_ok && rank >= a.lo && rank < a.hi;
    a.victim[static_cast<size_t>(b) * a.P + i] = v;
    if (v) {
      const int idx = rank - a.lo;
      if (idx < a.evcap)
        a.evlog[static_cast<size_t>(b) * a.evcap + idx] = i;
      else
        set_err(a.err, kErrLogOverflow);
    }
  }
}

// Compaction: retained prompt positions -> slots 0..R-1 (ascending), after dropping the
// hard-cap overflow (the smallest remaining positions, kv_coupled_generator.py:590-604).
struct CompactArgs {
  StateArgs st;
  int P, C, n_policy_victims;
  const uint8_t* victim;  // [B][P]
  const float* scores;    // [B][P] or null
  int* gather_src;        // [B][S] out: prompt position held by each slot (-1 = none)
  int* evlog;
  int evcap;
  int* evcount;
  int* seq_step;
  int* next_pos;
  int* retained_log;  // [B][log_steps + 1] (may be null)
  int log_steps;
  float* step_score;  // [B][S] zeroed
  int* err;
};

__global__ void __launch_bounds__(1024) prefill_compact_kernel(CompactArgs a) {
  __shared__ int warp_tot[32];
  __shared__ int carry;
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int S = a.st.S;
  SeqState s = a.st.seq(b);
  const int remaining = a.P - a.n_policy_victims;
  const int overflow = remaining - a.C > 0 ? remaining - a.C : 0;
  for (int i = tid; i < S; i += blockDim.x) {
    s.slot_pos[i] = -1;
    a.gather_src[static_cast<size_t>(b) * S + i] = -1;
    a.step_score[static_cast<size_t>(b) * S + i] = 0.f;
  }
  for (int w = tid; w < a.st.W; w += blockDim.x) s.posmap[w] = 0u;
  if (tid == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < a.P; base += blockDim.x) {
    const int i = base + tid;
    const int keep = (i < a.P) && !a.victim[static_cast<size_t>(b) * a.P + i];
    int incl = keep;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int v = lane < (blockDim.x >> 5) ? warp_tot[lane] : 0;
      int inc2 = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, inc2, o);
        if (lane >= o) inc2 += t;
      }
      warp_tot[lane] = inc2 - v;  // exclusive warp offsets
    }
    __syncthreads();
    const int r = carry + warp_tot[warp] + incl - keep;  // rank among remaining positions
    if (keep) {
      if (r < overflow) {
        const int idx = a.n_policy_victims + r;
        if (idx < a.evcap)
          a.evlog[static_cast<size_t>(b) * a.evcap + idx] = i;
        else
          set_err(a.err, kErrLogOverflow);
      } else {
        const int sl = r - overflow;
        if (sl < S) {
          const float sc = a.scores ? a.scores[static_cast<size_t>(b) * a.P + i] : 0.f;
          s.slot_pos[sl] = i;
          s.insert_step[sl] = 0;
          s.last_access[sl] = 0;
          s.access_count[sl] = 1;
          s.attn[sl] = sc;
          s.max_attn[sl] = sc;
          s.cumul[sl] = static_cast<double>(sc);
          s.prefill[sl] = sc;
          atomicOr(&s.posmap[i >> 5], 1u << (i & 31));
          a.gather_src[static_cast<size_t>(b) * S + sl] = i;
        } else {
          set_err(a.err, kErrNoFreeSlot);
        }
      }
    }
    __syncthreads();
    if (tid == blockDim.x - 1) carry = r + keep;
    __syncthreads();
  }
  if (tid == 0) {
    a.evcount[b] = a.n_policy_victims + overflow;
    a.seq_step[b] = 0;
    a.next_pos[b] = a.P;
    if (a.retained_log) a.retained_log[static_cast<size_t>(b) * (a.log_steps + 1)] = remaining - overflow;
  }
}

// Gather the retained prompt K/V rows into their slots for every layer.
__global__ void gather_kv_kernel(const __nv_bfloat16* __restrict__ src_k, const __nv_bfloat16* __restrict__ src_v,
                                 __nv_bfloat16* __restrict__ dst_k, __nv_bfloat16* __restrict__ dst_v,
                                 const int* __restrict__ gather_src, int B, int Hkv, int P, int S, int layers) {
  const int slot = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int kvh = blockIdx.y;
  const int lb = blockIdx.z;  // layer * B + b
  const int b = lb % B;
  if (slot >= S) return;
  const int p = gather_src[static_cast<size_t>(b) * S + slot];
  if (p < 0 || p >= P) return;
  const size_t src = ((static_cast<size_t>(lb) * Hkv + kvh) * P + p) * 128;
  const size_t dst = ((static_cast<size_t>(lb) * Hkv + kvh) * S + slot) * 128;
  const int lane = threadIdx.x & 31;
  reinterpret_cast<uint2*>(dst_k + dst)[lane] = reinterpret_cast<const uint2*>(src_k + src)[lane];
  reinterpret_cast<uint2*>(dst_v + dst)[lane] = reinterpret_cast<const uint2*>(src_v + src)[lane];
  (void)layers;
}

// ------------------------------------------------------------------------------------
// host launchers
// ------------------------------------------------------------------------------------
static int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(kStatusCuda, "%s launch: %s", what, cudaGetErrorString(e));
  return kStatusOk;
}

static bool state_ok(const StateArgs& s) {
  return s.slot_pos && s.insert_step && s.last_access && s.access_count && s.attn && s.max_attn && s.cumul &&
         s.prefill && s.posmap && s.B > 0 && s.S > 0 && s.W > 0;
}

int score_update(cudaStream_t stream, const StateArgs& st, const int* seq_step, float* step_score, int* err) {
  if (!state_ok(st) || !seq_step || !step_score) return fail(kStatusArg, "score_update: bad argument");
  // a cluster of up to 8 CTAs per sequence, each with at most ~512 slots
  int cs = (st.S + 511) / 512;
  if (cs > 8) cs = 8;
  if (cs < 1) cs = 1;
  if (st.B > 65535) return fail(kStatusArg, "score_update: batch %d too large", st.B);
  cudaError_t le = launch_pdl(score_update_kernel, dim3(cs, st.B), dim3(kScoreThreads), 0, stream, dim3(cs, 1, 1), st,
                              seq_step, step_score, err);
  if (le != cudaSuccess) return fail(kStatusCuda, "score_update launch: %s", cudaGetErrorString(le));
  return check_launch("score_update");
}

// per-head signals of the faithful Ada-KV / QUEST policies (kv_coupled_generator.py:
// 470-492): cumulative (float64 sum over steps) and current (this step's) attention of
// query heads 0..Hkv-1, per slot.  The slot that received this step's new position
// starts from zero (a fresh position's signal in the reference); head_score is cleared.
__global__ void head_signal_update_kernel(int Hkv, int S, const int* __restrict__ write_slot,
                                          float* __restrict__ head_score, double* __restrict__ head_cumul,
                                          float* __restrict__ head_current) {
  pdl_launch_dependents();
  pdl_wait();
  const int b = blockIdx.y;
  const int ws = write_slot[b];
  const size_t base = static_cast<size_t>(b) * Hkv * S;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < Hkv * S; i += gridDim.x * blockDim.x) {
    const float q = head_score[base + i];
    const double prev = (i % S) == ws ? 0.0 : head_cumul[base + i];
    head_cumul[base + i] = __dadd_rn(prev, static_cast<double>(q));
    head_current[base + i] = q;
    head_score[base + i] = 0.f;
  }
}

int head_signal_update(cudaStream_t stream, int B, int Hkv, int S, const int* write_slot, float* head_score,
                       double* head_cumul, float* head_current, int* err) {
  (void)err;
  const int n = Hkv * S;
  dim3 grid((n + 255) / 256 < 64 ? (n + 255) / 256 : 64, B);
  cudaError_t e = launch_pdl(head_signal_update_kernel, grid, dim3(256), 0, stream, dim3(0), Hkv, S, write_slot,
                             head_score, head_cumul, head_current);
  if (e != cudaSuccess) return fail(kStatusCuda, "head_signal_update launch: %s", cudaGetErrorString(e));
  return check_launch("head_signal_update");
}

int append_evict(cudaStream_t stream, const AppendArgs& a) {
  if (!state_ok(a.st) || !a.seq_step || !a.next_pos || !a.cur_pos || !a.write_slot || !a.evlog || !a.evcount)
    return fail(kStatusArg, "append_evict: bad argument");
  if (a.C <= 0 || a.E <= 0) return fail(kStatusArg, "append_evict: capacity and evict_every must be > 0");
  if (a.policy < 0 || a.policy >= kPolicyCount) return fail(kStatusArg, "append_evict: unknown policy %d", a.policy);
  if (a.policy == kPolicyRandom && !a.ext_pos)
    return fail(kStatusArg, "append_evict: the random policy's victims come from the host (kvbp_append_evict_listed)");
  if (a.ext_pos && (!a.ext_n || a.ext_stride <= 0))
    return fail(kStatusArg, "append_evict_listed: victim_count and victim_stride > 0 are required");
  if (a.st.S > kEvictThreads * kMaxPerThread)
    return fail(kStatusUnsupported, "append_evict: %d slots exceed %d", a.st.S, kEvictThreads * kMaxPerThread);
  if (a.n_prefix < 0 || a.n_suffix < 0) return fail(kStatusArg, "append_evict: negative protection size");
  if (a.upd_score && !a.upd_pending) return fail(kStatusArg, "update_append_evict: pending flags are required");
  AppendArgs aa = a;
  int smem = a.st.S * 4;
  aa.pm_smem = (a.st.S + a.st.W) * 4 <= 160 * 1024;
  if (aa.pm_smem) smem = (a.st.S + a.st.W) * 4;
  aa.key_smem = 0;
  const int key_off = (smem + 15) / 16 * 16;
  if (key_off + a.st.S * static_cast<int>(sizeof(Key3)) <= 200 * 1024) {
    aa.key_smem = key_off;
    smem = key_off + a.st.S * static_cast<int>(sizeof(Key3));
  }
  static int configured = 0;
  if (smem > 48 * 1024 && smem > configured) {
    cudaError_t e = cudaFuncSetAttribute(append_evict_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return fail(kStatusCuda, "append_evict: %s", cudaGetErrorString(e));
    configured = smem;
  }
  cudaError_t le = launch_pdl(append_evict_kernel, dim3(a.st.B), dim3(kEvictThreads), smem, stream, dim3(0), aa);
  if (le != cudaSuccess) return fail(kStatusCuda, "append_evict launch: %s", cudaGetErrorString(le));
  return check_launch("append_evict");
}

int prefill_select(cudaStream_t stream, const PrefillSelArgs& a) {
  if (!a.victim || !a.evlog || a.B <= 0 || a.P <= 0) return fail(kStatusArg, "prefill_select: bad argument");
  if (a.policy < 0 || a.policy >= kPolicyCount) return fail(kStatusArg, "prefill_select: unknown policy");
  dim3 grid((a.P + 255) / 256, a.B);
  if (grid.y > 65535) return fail(kStatusArg, "prefill_select: batch too large");
  prefill_rank_kernel<<<grid, 256, 0, stream>>>(a);
  return check_launch("prefill_select");
}

int prefill_compact(cudaStream_t stream, const CompactArgs& a) {
  if (!state_ok(a.st) || !a.victim || !a.gather_src || !a.evlog || !a.evcount || !a.seq_step || !a.next_pos ||
      !a.step_score)
    return fail(kStatusArg, "prefill_compact: bad argument");
  prefill_compact_kernel<<<a.st.B, 1024, 0, stream>>>(a);
  return check_launch("prefill_compact");
}

int gather_kv(cudaStream_t stream, const void* src_k, const void* src_v, void* dst_k, void* dst_v,
              const int* gather_src, int layers, int B, int Hkv, int P, int S) {
  if (!src_k || !src_v || !dst_k || !dst_v || !gather_src) return fail(kStatusArg, "gather_kv: null pointer");
  if (layers <= 0 || B <= 0 || Hkv <= 0 || P <= 0 || S <= 0) return fail(kStatusArg, "gather_kv: bad size");
  if (static_cast<long long>(layers) * B > 65535) return fail(kStatusArg, "gather_kv: layers*B too large");
  dim3 grid((S + 3) / 4, Hkv, layers * B);
  gather_kv_kernel<<<grid, 128, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(src_k), static_cast<const __nv_bfloat16*>(src_v),
      static_cast<__nv_bfloat16*>(dst_k), static_cast<__nv_bfloat16*>(dst_v), gather_src, B, Hkv, P, S, layers);
  return check_launch("gather_kv");
}

}  // namespace kvbp

// ------------------------------------------------------------------------------------
// C ABI
// ------------------------------------------------------------------------------------
#include "../../include/kvbp.h"

namespace {

kvbp::StateArgs to_state(const kvbp_state* s) {
  kvbp::StateArgs a{};
  a.B = s->B;
  a.S = s->S;
  a.W = s->W;
  a.slot_pos = s->slot_pos;
  a.insert_step = s->insert_step;
  a.last_access = s->last_access;
  a.access_count = s->access_count;
  a.attn = s->attn;
  a.max_attn = s->max_attn;
  a.cumul = s->cumul;
  a.prefill = s->prefill;
  a.posmap = s->posmap;
  return a;
}

}  // namespace

extern "C" {

int kvbp_score_update(kvbp_stream_t stream, const kvbp_state* st, const int32_t* seq_step, float* step_score,
                      int32_t* dev_err) {
  if (!st) return kvbp::fail(kvbp::kStatusArg, "score_update: null state");
  return kvbp::score_update(reinterpret_cast<cudaStream_t>(stream), to_state(st), seq_step, step_score, dev_err);
}

static int append_evict_common(kvbp_stream_t stream, const kvbp_state* st, const kvbp_evict_cfg* cfg,
                               int32_t* seq_step, int32_t* next_pos, int32_t* cur_pos, int32_t* write_slot,
                               const int32_t* tokens, int32_t* token_log, int32_t log_steps, int32_t* evlog,
                               int32_t* evcount, int32_t evcap, int32_t* retained_log, const int32_t* victim_pos,
                               const int32_t* victim_count, int32_t victim_stride, int32_t flags,
                               int32_t* dev_err, float* step_score = nullptr, int32_t* pending = nullptr) {
  if (!st || !cfg) return kvbp::fail(kvbp::kStatusArg, "append_evict: null state/config");
  kvbp::AppendArgs a{};
  a.upd_score = step_score;
  a.upd_pending = pending;
  a.ext_pos = victim_pos;
  a.ext_n = victim_count;
  a.ext_stride = victim_stride;
  a.no_hardcap = (flags & KVBP_LISTED_NO_HARDCAP) ? 1 : 0;
  a.st = to_state(st);
  a.C = cfg->capacity;
  a.E = cfg->evict_every;
  a.policy = cfg->policy;
  a.protect = cfg->protect;
  a.n_prefix = cfg->n_prefix;
  a.n_suffix = cfg->n_suffix;
  a.decode_regime = cfg->decode_regime;
  a.seq_step = seq_step;
  a.next_pos = next_pos;
  a.cur_pos = cur_pos;
  a.write_slot = write_slot;
  a.tokens = tokens;
  a.token_log = token_log;
  a.log_steps = log_steps;
  a.evlog = evlog;
  a.evcount = evcount;
  a.evcap = evcap;
  a.retained_log = retained_log;
  a.err = dev_err;
  return kvbp::append_evict(reinterpret_cast<cudaStream_t>(stream), a);
}

int kvbp_append_evict(kvbp_stream_t stream, const kvbp_state* st, const kvbp_evict_cfg* cfg, int32_t* seq_step,
                      int32_t* next_pos, int32_t* cur_pos, int32_t* write_slot, const int32_t* tokens,
                      int32_t* token_log, int32_t log_steps, int32_t* evlog, int32_t* evcount, int32_t evcap,
                      int32_t* retained_log, int32_t* dev_err) {
  return append_evict_common(stream, st, cfg, seq_step, next_pos, cur_pos, write_slot, tokens, token_log, log_steps,
                             evlog, evcount, evcap, retained_log, nullptr, nullptr, 0, 0, dev_err);
}

int kvbp_update_append_evict(kvbp_stream_t stream, const kvbp_state* st, const kvbp_evict_cfg* cfg,
                             int32_t* seq_step, int32_t* next_pos, int32_t* cur_pos, int32_t* write_slot,
                             const int32_t* tokens, int32_t* token_log, int32_t log_steps, int32_t* evlog,
                             int32_t* evcount, int32_t evcap, int32_t* retained_log, float* step_score,
                             int32_t* pending, int32_t* dev_err) {
  if (!step_score || !pending)
    return kvbp::fail(kvbp::kStatusArg, "update_append_evict: step_score and pending are required");
  return append_evict_common(stream, st, cfg, seq_step, next_pos, cur_pos, write_slot, tokens, token_log, log_steps,
                             evlog, evcount, evcap, retained_log, nullptr, nullptr, 0, 0, dev_err, step_score,
                             pending);
}

int kvbp_append_evict_listed(kvbp_stream_t stream, const kvbp_state* st, const kvbp_evict_cfg* cfg,
                             int32_t* seq_step, int32_t* next_pos, int32_t* cur_pos, int32_t* write_slot,
                             const int32_t* tokens, int32_t* token_log, int32_t log_steps, int32_t* evlog,
                             int32_t* evcount, int32_t evcap, int32_t* retained_log, const int32_t* victim_pos,
                             const int32_t* victim_count, int32_t victim_stride, int32_t flags, int32_t* dev_err) {
  if (!victim_pos) return kvbp::fail(kvbp::kStatusArg, "append_evict_listed: victim_pos is required");
  return append_evict_common(stream, st, cfg, seq_step, next_pos, cur_pos, write_slot, tokens, token_log, log_steps,
                             evlog, evcount, evcap, retained_log, victim_pos, victim_count, victim_stride, flags,
                             dev_err);
}

int kvbp_head_signal_update(kvbp_stream_t stream, int32_t B, int32_t Hkv, int32_t S, const int32_t* write_slot,
                            float* head_score, double* head_cumul, float* head_current, int32_t* dev_err) {
  if (!head_score || !head_cumul || !head_current || !write_slot)
    return kvbp::fail(kvbp::kStatusArg, "head_signal_update: null pointer");
  if (B <= 0 || Hkv <= 0 || S <= 0 || B > 65535) return kvbp::fail(kvbp::kStatusArg, "head_signal_update: bad size");
  return kvbp::head_signal_update(reinterpret_cast<cudaStream_t>(stream), B, Hkv, S, write_slot, head_score,
                                  head_cumul, head_current, dev_err);
}

int kvbp_prefill_select(kvbp_stream_t stream, int32_t B, int32_t P, const kvbp_evict_cfg* cfg, const float* scores,
                        uint8_t* victim, int32_t* evlog, int32_t evcap, int32_t* n_policy_victims,
                        int32_t* dev_err) {
  if (!cfg || !n_policy_victims) return kvbp::fail(kvbp::kStatusArg, "prefill_select: null config/output");
  if (cfg->policy < 0 || cfg->policy >= kvbp::kPolicyCount)
    return kvbp::fail(kvbp::kStatusArg, "prefill_select: unknown policy %d", cfg->policy);
  if (cfg->policy == kvbp::kPolicyRandom)
    return kvbp::fail(kvbp::kStatusArg, "prefill_select: the random policy's victims come from the host");
  if (P <= 0 || cfg->capacity <= 0) return kvbp::fail(kvbp::kStatusArg, "prefill_select: bad size");
  // _maybe_evict(step=0, force_if_over_capacity=True): evict_count = max(0, P - C)
  const int C = cfg->capacity;
  const int k_req = P - C > 0 ? P - C : 0;
  kvbp::PrefillSelArgs a{};
  a.B = B;
  a.P = P;
  a.policy = cfg->policy;
  a.scores = scores;
  a.victim = victim;
  a.evlog = evlog;
  a.evcap = evcap;
  a.err = dev_err;
  int n_elig = P;
  a.n_prefix = 0;
  a.n_suffix = 0;
  a.protect_all = 0;
  if (cfg->protect) {
    // ProtectedPolicyWrapper over positions 0..P-1: returns [] when evict_count <= 0;
    // n_suffix == 0 makes all_positions[-0:] the whole list.
    if (k_req <= 0 || cfg->n_suffix == 0 || cfg->n_suffix >= P || cfg->n_prefix >= P) {
      a.protect_all = 1;
      n_elig = 0;
    } else {
      a.n_prefix = cfg->n_prefix;
      a.n_suffix = cfg->n_suffix;
      n_elig = P - cfg->n_prefix - cfg->n_suffix;
      if (n_elig < 0) n_elig = 0;
    }
  }
  const int k = k_req < n_elig ? k_req : n_elig;
  a.lo = 0;
  a.hi = k;
  if (cfg->policy == kvbp::kPolicyStreamingLLM && k > 0) {
    // all step-0 keys tie on (insert, last) = (0, 0): order = str(pos) order.  The sink
    // is ranks 0..3, "recent" the top C-4 ranks; candidates are the ranks in between.
    const int recent_n = C - 4 > 0 ? C - 4 : 0;
    const int n_notrecent = n_elig - recent_n > 0 ? n_elig - recent_n : 0;
    const int n_sink = n_elig < 4 ? n_elig : 4;
    const int n_cand = n_notrecent - n_sink > 0 ? n_notrecent - n_sink : 0;
    if (n_cand > 0) {
      a.lo = n_sink;
      a.hi = n_sink + (k < n_cand ? k : n_cand);
    }
  }
  *n_policy_victims = a.hi - a.lo;
  if (B <= 0) return kvbp::fail(kvbp::kStatusArg, "prefill_select: bad batch");
  return kvbp::prefill_select(reinterpret_cast<cudaStream_t>(stream), a);
}

int kvbp_prefill_compact(kvbp_stream_t stream, const kvbp_state* st, int32_t P, int32_t capacity,
                         int32_t n_policy_victims, const uint8_t* victim, const float* scores, int32_t* gather_src,
                         int32_t* evlog, int32_t evcap, int32_t* evcount, int32_t* seq_step, int32_t* next_pos,
                         int32_t* retained_log, int32_t log_steps, float* step_score, int32_t* dev_err) {
  if (!st) return kvbp::fail(kvbp::kStatusArg, "prefill_compact: null state");
  if (P <= 0 || capacity <= 0 || n_policy_victims < 0 || n_policy_victims > P)
    return kvbp::fail(kvbp::kStatusArg, "prefill_compact: bad size");
  if (st->W * 32LL < P) return kvbp::fail(kvbp::kStatusArg, "prefill_compact: posmap too small for %d positions", P);
  kvbp::CompactArgs a{};
  a.st = to_state(st);
  a.P = P;
  a.C = capacity;
  a.n_policy_victims = n_policy_victims;
  a.victim = victim;
  a.scores = scores;
  a.gather_src = gather_src;
  a.evlog = evlog;
  a.evcap = evcap;
  a.evcount = evcount;
  a.seq_step = seq_step;
  a.next_pos = next_pos;
  a.retained_log = retained_log;
  a.log_steps = log_steps;
  a.step_score = step_score;
  a.err = dev_err;
  return kvbp::prefill_compact(reinterpret_cast<cudaStream_t>(stream), a);
}

int kvbp_gather_kv(kvbp_stream_t stream, const void* src_k, const void* src_v, void* dst_k, void* dst_v,
                   const int32_t* gather_src, int32_t layers, int32_t B, int32_t Hkv, int32_t P, int32_t S) {
  return kvbp::gather_kv(reinterpret_cast<cudaStream_t>(stream), src_k, src_v, dst_k, dst_v, gather_src, layers, B,
                         Hkv, P, S);
}

}  // extern "C"

// ------------------------------------------------------------------------------------
// Step-0 eviction that allocates nothing
// ------------------------------------------------------------------------------------
// Callers that cannot allocate device memory (a jax.ffi / XLA custom-call handler may only
// use the buffers XLA assigns it, and XLA usually pre-allocates most of the GPU, so a
// cudaMalloc from inside the handler bypasses its allocator and can fail) still need the
// per-position victim flags that sit between kvbp_prefill_select and kvbp_prefill_compact.
// This variant keeps them in a fixed array that every GPU loading the library holds until
// the process exits.
#include <cuda.h>

#include <mutex>

namespace {

constexpr long long kNoAllocMaxPositions = 1LL << 20;  // batch * prompt flags (1 MiB)
constexpr int kNoAllocCacheEntries = 64;

__device__ __align__(256) uint8_t g_prefill_victim_scratch[kNoAllocMaxPositions];

// Cache of the array's device address per CUDA context.  A context's ID (cuCtxGetId) is
// unique for the life of the process, so a context created after cudaDeviceReset, or a
// non-primary context on the same device, never picks up a stale address.
struct NoAllocEntry {
  unsigned long long ctx_id;
  uint8_t* ptr;
};
std::mutex g_noalloc_mu;
NoAllocEntry g_noalloc_cache[kNoAllocCacheEntries] = {};
int g_noalloc_used = 0;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

template <typename Fn>
Fn driver_fn(const char* name) {
  void* ptr = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &ptr, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
    return reinterpret_cast<Fn>(ptr);
  return nullptr;
}

// Device address of the scratch array in the current context.  In host code the array's
// name is only a host-side stand-in, so the address is looked up with the context current
// (cudaGetSymbolAddress) and cached under the context's ID.
int noalloc_scratch(uint8_t** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return kvbp::fail(kvbp::kStatusCuda, "kvbp_prefill_evict_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  static CtxGetCurrentFn get_ctx = driver_fn<CtxGetCurrentFn>("cuCtxGetCurrent");
  static CtxGetIdFn get_id = driver_fn<CtxGetIdFn>("cuCtxGetId");
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  // no context current yet on this thread: the lookup below initialises one, uncached
  const bool have_id = get_ctx && get_id && get_ctx(&ctx) == CUDA_SUCCESS && ctx && get_id(ctx, &id) == CUDA_SUCCESS;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (have_id)
    for (int i = 0; i < g_noalloc_used; ++i)
      if (g_noalloc_cache[i].ctx_id == id) {
        *out = g_noalloc_cache[i].ptr;
        return kvbp::kStatusOk;
      }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_prefill_victim_scratch);
  if (e != cudaSuccess || !p)
    return kvbp::fail(kvbp::kStatusCuda, "kvbp_prefill_evict_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
  if (have_id && g_noalloc_used < kNoAllocCacheEntries) g_noalloc_cache[g_noalloc_used++] = {id, static_cast<uint8_t*>(p)};
  *out = static_cast<uint8_t*>(p);
  return kvbp::kStatusOk;
}

}  // namespace

extern "C" int kvbp_prefill_evict_noalloc(kvbp_stream_t stream, const kvbp_state* st, int32_t P,
                                          const kvbp_evict_cfg* cfg, const float* scores, int32_t* gather_src,
                                          int32_t* evlog, int32_t evcap, int32_t* evcount, int32_t* seq_step,
                                          int32_t* next_pos, int32_t* retained_log, int32_t log_steps,
                                          float* step_score, int32_t* dev_err) {
  if (!st || !cfg) return kvbp::fail(kvbp::kStatusArg, "kvbp_prefill_evict_noalloc: null state/config");
  if (st->B <= 0 || P <= 0) return kvbp::fail(kvbp::kStatusArg, "kvbp_prefill_evict_noalloc: bad size");
  const long long n = static_cast<long long>(st->B) * P;
  if (n > kNoAllocMaxPositions)
    return kvbp::fail(kvbp::kStatusArg,
                      "kvbp_prefill_evict_noalloc: batch %d x prompt %d = %lld positions exceeds the fixed "
                      "scratch of %lld; use kvbp_prefill_select + kvbp_prefill_compact with your own buffer",
                      st->B, P, n, kNoAllocMaxPositions);
  uint8_t* scratch = nullptr;
  int s = noalloc_scratch(&scratch);
  if (s) return s;
  // kvbp_prefill_select rewrites every flag of the B*P range, so nothing needs clearing.
  int32_t n_policy = 0;
  s = kvbp_prefill_select(stream, st->B, P, cfg, scores, scratch, evlog, evcap, &n_policy, dev_err);
  if (s) return s;
  return kvbp_prefill_compact(stream, st, P, cfg->capacity, n_policy, scratch, scores, gather_src, evlog, evcap,
                              evcount, seq_step, next_pos, retained_log, log_steps, step_score, dev_err);
}
