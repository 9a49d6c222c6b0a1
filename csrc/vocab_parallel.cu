// Vocab-parallel token sampling over NVLink peer memory (sm_100a).
//
// With the LM head split over the vocabulary, rank r computes only the logits
// columns [vocab0, vocab0 + vocab_local).  Instead of all-gathering the full
// fp32 logits rows (rows x vocab x 4 bytes onto every rank), each rank reduces
// its slice to a small record per row and writes it straight into every rank's
// exchange region; the draw then runs on the records:
//
//   record (kVpHeaderBytes + 8 * cand bytes)
//     m       max of the processed slice
//     z       sum over the slice of exp(x - m)
//     tC      the cand-th largest value of the slice (-inf if the slice has <= cand tokens)
//     n       number of candidates that follow
//     gbest   argmax key: greedy rows -> (x, token); unfiltered sampling rows ->
//             (x + Gumbel(seed, step, token), token) over the whole slice
//     x[cand], token[cand]   the slice's top-cand (value, full-vocabulary token)
//
// The merge is exact where the full-row sampler's kept set lies inside the union
// of the ranks' candidates:
//   greedy                        max of the ranks' argmax keys
//   temperature only              max of the ranks' Gumbel-max keys (the noise of a
//                                 token depends only on (seed, step, token))
//   top-k <= cand (+ top-p/min-p) the global top-k is inside the union
//   top-p / min-p                 exact when the final threshold lies above every
//                                 rank's cand-th value (tC): every token above it is a
//                                 candidate.  Otherwise (flat distributions) the draw
//                                 uses the union only and the row is counted in
//                                 ``inexact``.
// The draw itself follows sample_kernel step by step (radix-select top-k, min-p,
// top-p bisection with the global normaliser, Gumbel-max), so an exact row draws
// the token the single-GPU sampler would.
//
// Ordering: the local kernel's CTAs read seq at their start; the last CTA to
// finish (all others have read seq) stores seq + 1 and release-stores it into
// flags[rank] of every peer.  Records live in two parity halves (seq & 1): a
// rank cannot be two exchanges ahead of a peer because every decode step passes
// through the model's reduce points, which wait for all ranks.
//
// Reference counterpart: the vocab-parallel LM head + logits all-gather of the
// thinker (sglang_omni/models/qwen3_omni/thinker.py:614-619, sglang's
// ParallelLMHead / LogitsProcessor), with tp_size forced to 1 there.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "omni_kernels.h"
#include "sampling.cuh"
#include "sm100.cuh"

namespace omni {
namespace {

using namespace samp;

__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct VpHeader {
  float m, z, tC;
  int n;
  unsigned long long gbest;
  unsigned long long pad;
};
static_assert(sizeof(VpHeader) == kVpHeaderBytes, "record header");

__device__ __forceinline__ char* record_at(int64_t base, const VocabSampleArgs& a, uint32_t parity, int src, int row) {
  const int64_t rec = kVpHeaderBytes + 8ll * a.cand;
  return reinterpret_cast<char*>(base) +
         ((static_cast<int64_t>(parity) * a.world + src) * a.max_rows + row) * rec;
}

struct RowRules {
  bool greedy, unfiltered;
  int topk;
  float topp, minp;
};

__device__ __forceinline__ RowRules row_rules(const VocabSampleArgs& a, int sr) {
  RowRules r;
  const float temp = a.temperature ? a.temperature[sr] : 0.f;
  r.greedy = !(temp > 0.f);
  r.topk = a.top_k ? a.top_k[sr] : 0;
  r.topp = a.top_p ? a.top_p[sr] : 1.f;
  r.minp = a.min_p ? a.min_p[sr] : 0.f;
  const bool has_k = r.topk > 0 && r.topk < a.vocab;
  r.unfiltered = !r.greedy && !has_k && !(r.topp < 1.f) && !(r.minp > 0.f);
  return r;
}

__device__ __forceinline__ float gumbel(const VocabSampleArgs& a, int sr, int token) {
  const uint64_t seed = a.seeds ? static_cast<uint64_t>(a.seeds[sr]) : 0x1234ull;
  const uint64_t step = a.step ? static_cast<uint64_t>(a.step[sr]) : 0ull;
  const float u = uniform01(seed + 0x9E37ull * step, static_cast<uint64_t>(token));
  return -logf(-logf(u));
}

// Threshold = the k-th largest of n values in shared memory (4-pass radix select
// on order-preserving keys), by the whole block.
__device__ float radix_kth(const float* xs, int n, int k, unsigned int* hist, uint32_t* s_prefix, int* s_kleft) {
  if (threadIdx.x == 0) {
    *s_prefix = 0u;
    *s_kleft = k;
  }
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    const uint32_t mask_hi = pass == 0 ? 0u : (0xffffffffu << (32 - 8 * pass));
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0u;
    __syncthreads();
    const uint32_t pref = *s_prefix;
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
      const uint32_t key = f2key(xs[j]);
      if ((key & mask_hi) == pref) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int left = *s_kleft;
      int bin = 255;
      for (; bin > 0; --bin) {
        const int c = static_cast<int>(hist[bin]);
        if (c >= left) break;
        left -= c;
      }
      *s_kleft = left;
      *s_prefix = pref | (static_cast<uint32_t>(bin) << shift);
    }
    __syncthreads();
  }
  return key2f(*s_prefix);
}

// ----------------------------------------------------------------------------- local phase
__global__ void __launch_bounds__(1024) vp_local_kernel(VocabSampleArgs a) {
  __shared__ float sred[33];
  __shared__ unsigned int hist[256];
  __shared__ uint32_t s_prefix;
  __shared__ int s_kleft;
  __shared__ unsigned long long s_best;
  __shared__ int s_ncand;
  __shared__ uint32_t s_target;
  __shared__ float cx[kVpMaxCand];
  __shared__ int ci[kVpMaxCand];
  const int row = blockIdx.x;
  if (threadIdx.x == 0) {
    s_target = *reinterpret_cast<const volatile uint32_t*>(a.seq) + 1u;
    s_best = 0ull;
    s_ncand = 0;
  }
  const int sr = a.row_slot ? a.row_slot[row] : row;
  float* lg = a.logits + static_cast<int64_t>(row) * a.logits_stride;
  const int V = a.vocab_local, g0 = a.vocab0;
  const RowRules rr = row_rules(a, sr);
  const float temp = a.temperature ? a.temperature[sr] : 0.f;
  const float rep = a.rep_penalty ? a.rep_penalty[sr] : 1.f;
  const uint8_t* seen = a.seen ? a.seen + static_cast<int64_t>(sr) * a.seen_stride + g0 : nullptr;
  const bool suppress = a.suppress_lo >= 0;
  const bool penal = seen != nullptr && rep != 1.f;
  const float inv_t = rr.greedy ? 1.f : 1.f / temp;
  __syncthreads();

  // 1) processing (in place when it changes the row) + max / greedy argmax
  unsigned long long best = 0ull;
  float m = -INFINITY;
  if (suppress || penal || !rr.greedy) {
    row_transform(lg, V, [&](int i, float x) {
      const int gi = g0 + i;
      if (suppress && gi >= a.suppress_lo && gi < a.suppress_hi && gi != a.suppress_keep) x = -INFINITY;
      if (penal && seen[i]) x = x > 0.f ? x / rep : x * rep;
      const float y = rr.greedy ? x : x * inv_t;
      m = fmaxf(m, y);
      const unsigned long long k = argmax_key(y, gi);
      best = k > best ? k : best;
      return y;
    });
  } else {
    row_for_each(lg, V, [&](int i, float x) {
      m = fmaxf(m, x);
      const unsigned long long k = argmax_key(x, g0 + i);
      best = k > best ? k : best;
    });
  }
  m = block_reduce(m, sred, MaxOp(), -INFINITY);
  float z = 0.f, tC = -INFINITY;
  if (rr.greedy) {
    atomicMax(&s_best, best);
  } else if (rr.unfiltered) {
    // Gumbel-max over the slice (tokens > 40 nats below the max cannot win in fp32)
    best = 0ull;
    row_for_each(lg, V, [&](int i, float x) {
      if (x >= m - 40.f && x > -INFINITY) {
        const unsigned long long k = argmax_key(x + gumbel(a, sr, g0 + i), g0 + i);
        best = k > best ? k : best;
      }
    });
    atomicMax(&s_best, best);
  } else {
    row_for_each(lg, V, [&](int, float x) {
      if (x > -INFINITY) z += __expf(x - m);
    });
    z = block_reduce(z, sred, SumOp(), 0.f);
    if (V > a.cand) {
      // cand-th largest key of the slice; the copy below keeps the values >= it
      if (threadIdx.x == 0) {
        s_prefix = 0u;
        s_kleft = a.cand;
      }
      for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        const uint32_t mask_hi = pass == 0 ? 0u : (0xffffffffu << (32 - 8 * pass));
        for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0u;
        __syncthreads();
        const uint32_t pref = s_prefix;
        row_for_each(lg, V, [&](int, float x) {
          const uint32_t k = f2key(x);
          if ((k & mask_hi) == pref) atomicAdd(&hist[(k >> shift) & 255u], 1u);
        });
        __syncthreads();
        if (threadIdx.x == 0) {
          int left = s_kleft;
          int bin = 255;
          for (; bin > 0; --bin) {
            const int c = static_cast<int>(hist[bin]);
            if (c >= left) break;
            left -= c;
          }
          s_kleft = left;
          s_prefix = pref | (static_cast<uint32_t>(bin) << shift);
        }
        __syncthreads();
      }
      tC = key2f(s_prefix);
    }
    // candidates: values > tC first (at most cand - 1 of them), then ties of tC
    for (int pass = 0; pass < 2; ++pass) {
      row_for_each(lg, V, [&](int i, float x) {
        const bool keep = x > -INFINITY && (pass == 0 ? x > tC : x == tC);
        const unsigned act = __activemask();
        const unsigned bal = __ballot_sync(act, keep);
        if (bal == 0u) return;
        const int leader = __ffs(act) - 1;
        const int lane = threadIdx.x & 31;
        int base = 0;
        if (lane == leader) base = atomicAdd(&s_ncand, __popc(bal));
        base = __shfl_sync(act, base, leader);
        if (keep) {
          const int slot = base + __popc(bal & ((1u << lane) - 1u));
          if (slot < a.cand) {
            cx[slot] = x;
            ci[slot] = g0 + i;
          }
        }
      });
      __syncthreads();
      if (tC == -INFINITY) break;   // the whole slice was taken in pass 0
    }
  }
  __syncthreads();

  // 2) the record into every rank's exchange region
  const int n = min(s_ncand, a.cand);
  const uint32_t parity = s_target & 1u;
  for (int p = 0; p < a.world; ++p) {
    char* rec = record_at(a.peer_xchg[p], a, parity, a.rank, row);
    if (threadIdx.x == 0) {
      VpHeader h;
      h.m = m;
      h.z = z;
      h.tC = tC;
      h.n = rr.greedy || rr.unfiltered ? 0 : n;
      h.gbest = s_best;
      h.pad = 0ull;
      *reinterpret_cast<VpHeader*>(rec) = h;
    }
    if (!rr.greedy && !rr.unfiltered) {
      float* px = reinterpret_cast<float*>(rec + kVpHeaderBytes);
      int* pi = reinterpret_cast<int*>(rec + kVpHeaderBytes + 4ll * a.cand);
      for (int j = threadIdx.x; j < n; j += blockDim.x) {
        px[j] = cx[j];
        pi[j] = ci[j];
      }
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(a.counter, 1);
    if (prev == a.rows - 1) {   // every CTA has read seq and fenced its records
      *a.counter = 0;
      *reinterpret_cast<volatile uint32_t*>(a.seq) = s_target;
      __threadfence_system();
      for (int p = 0; p < a.world; ++p)
        st_release_sys_u32(reinterpret_cast<uint32_t*>(a.peer_flags[p]) + a.rank, s_target);
    }
  }
}

// ----------------------------------------------------------------------------- merge phase
__global__ void __launch_bounds__(256) vp_merge_kernel(VocabSampleArgs a) {
  __shared__ float sred[33];
  __shared__ unsigned int hist[256];
  __shared__ uint32_t s_prefix;
  __shared__ int s_kleft;
  __shared__ unsigned long long s_best;
  __shared__ int s_fail;
  __shared__ VpHeader hd[kVpMaxWorld];
  __shared__ int hoff[kVpMaxWorld + 1];
  __shared__ float cx[kVpMaxWorld * kVpMaxCand];
  __shared__ int ci[kVpMaxWorld * kVpMaxCand];
  const int row = blockIdx.x;
  const uint32_t target = *reinterpret_cast<const volatile uint32_t*>(a.seq);
  if (threadIdx.x == 0) {
    s_fail = 0;
    s_best = 0ull;
  }
  __syncthreads();
  if (threadIdx.x < a.world) {
    const uint32_t* f = reinterpret_cast<const uint32_t*>(a.peer_flags[a.rank]) + threadIdx.x;
    const uint64_t t0 = globaltimer_ns();
    while (static_cast<int32_t>(ld_acquire_sys_u32(f) - target) < 0) {
      if (globaltimer_ns() - t0 > static_cast<uint64_t>(a.timeout_ns)) {
        record_status(a.status, kStatusPeerTimeout);
        s_fail = 1;
        break;
      }
    }
  }
  __syncthreads();
  __threadfence_system();
  const int sr = a.row_slot ? a.row_slot[row] : row;
  if (s_fail) {
    if (threadIdx.x == 0) {
      a.out_tokens[row] = 0;
      if (a.slot_tokens) a.slot_tokens[sr] = 0;
    }
    return;
  }
  const RowRules rr = row_rules(a, sr);
  const uint32_t parity = target & 1u;
  const int64_t local = a.peer_xchg[a.rank];
  if (threadIdx.x < a.world) hd[threadIdx.x] = *reinterpret_cast<const VpHeader*>(record_at(local, a, parity,
                                                                                           threadIdx.x, row));
  __syncthreads();
  if (rr.greedy || rr.unfiltered) {
    if (threadIdx.x == 0) {
      unsigned long long b = 0ull;
      for (int s = 0; s < a.world; ++s) b = hd[s].gbest > b ? hd[s].gbest : b;
      s_best = b;
    }
  } else {
    if (threadIdx.x == 0) {
      int o = 0;
      for (int s = 0; s < a.world; ++s) {
        hoff[s] = o;
        o += min(max(hd[s].n, 0), a.cand);
      }
      hoff[a.world] = o;
    }
    __syncthreads();
    float m = -INFINITY, tstar = -INFINITY;
    for (int s = 0; s < a.world; ++s) {
      m = fmaxf(m, hd[s].m);
      tstar = fmaxf(tstar, hd[s].tC);
    }
    float Z = 0.f;
    for (int s = 0; s < a.world; ++s)
      if (hd[s].m > -INFINITY) Z += hd[s].z * __expf(hd[s].m - m);
    for (int s = 0; s < a.world; ++s) {
      const char* rec = record_at(local, a, parity, s, row);
      const float* px = reinterpret_cast<const float*>(rec + kVpHeaderBytes);
      const int* pi = reinterpret_cast<const int*>(rec + kVpHeaderBytes + 4ll * a.cand);
      const int n = hoff[s + 1] - hoff[s];
      for (int j = threadIdx.x; j < n; j += blockDim.x) {
        cx[hoff[s] + j] = px[j];
        ci[hoff[s] + j] = pi[j];
      }
    }
    __syncthreads();
    const int nc = hoff[a.world];
    float thr = -INFINITY;
    bool exact_k = false;
    if (rr.topk > 0 && rr.topk < a.vocab && rr.topk <= nc) {
      thr = radix_kth(cx, nc, rr.topk, hist, &s_prefix, &s_kleft);
      exact_k = rr.topk <= a.cand;
    }
    if (rr.minp > 0.f) thr = fmaxf(thr, m + logf(rr.minp));
    if (rr.topp < 1.f) {
      float z = 0.f;
      if (thr == -INFINITY) {
        z = Z;
      } else {
        for (int j = threadIdx.x; j < nc; j += blockDim.x)
          if (cx[j] >= thr) z += __expf(cx[j] - m);
        z = block_reduce(z, sred, SumOp(), 0.f);
      }
      float lo = thr == -INFINITY ? m - 80.f : thr, hi = m;
      for (int it = 0; it < 24; ++it) {
        const float mid = 0.5f * (lo + hi);
        float sm = 0.f;
        for (int j = threadIdx.x; j < nc; j += blockDim.x)
          if (cx[j] >= thr && cx[j] >= mid) sm += __expf(cx[j] - m);
        sm = block_reduce(sm, sred, SumOp(), 0.f);
        if (sm >= rr.topp * z) lo = mid; else hi = mid;
      }
      thr = fmaxf(thr, lo);
    }
    const bool exact = exact_k || tstar == -INFINITY || thr > tstar;
    if (!exact && threadIdx.x == 0 && a.inexact) atomicAdd(a.inexact, 1);
    unsigned long long best = 0ull;
    for (int j = threadIdx.x; j < nc; j += blockDim.x) {
      const float x = cx[j];
      if (x >= thr && x > -INFINITY) {
        const unsigned long long k = argmax_key(x + gumbel(a, sr, ci[j]), ci[j]);
        best = k > best ? k : best;
      }
    }
    atomicMax(&s_best, best);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int tok = static_cast<int>(0xffffffffu - static_cast<uint32_t>(s_best & 0xffffffffull));
    if (s_best == 0ull || tok < 0 || tok >= a.vocab) tok = 0;
    a.out_tokens[row] = tok;
    if (a.slot_tokens) a.slot_tokens[sr] = tok;
    if (a.step) a.step[sr] += 1;
    if (a.seen) a.seen[static_cast<int64_t>(sr) * a.seen_stride + tok] = 1;
  }
}

bool vp_args_ok(const VocabSampleArgs& a) {
  return a.world >= 1 && a.world <= kVpMaxWorld && a.rank >= 0 && a.rank < a.world && a.cand >= 1 &&
         a.cand <= kVpMaxCand && a.rows <= a.max_rows && a.vocab_local >= 1 && a.vocab0 >= 0 &&
         a.vocab0 + a.vocab_local <= a.vocab && a.peer_xchg != nullptr && a.peer_flags != nullptr &&
         a.seq != nullptr && a.counter != nullptr;
}

}  // namespace

cudaError_t vocab_sample_local(const VocabSampleArgs& a, cudaStream_t stream) {
  if (a.rows == 0) return cudaSuccess;
  if (!vp_args_ok(a)) return cudaErrorInvalidValue;
  vp_local_kernel<<<a.rows, 1024, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t vocab_sample_merge(const VocabSampleArgs& a, cudaStream_t stream) {
  if (a.rows == 0) return cudaSuccess;
  if (!vp_args_ok(a)) return cudaErrorInvalidValue;
  vp_merge_kernel<<<a.rows, 256, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace omni
