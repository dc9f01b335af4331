// hb_sample.cuh -- on-device token selection and logprobs.
//
// Three launch shapes share one pipeline: sample_kernel (one CTA of 1024
// threads), sample_batch_kernel (one such CTA per row of a batched step) and
// sample_grid_kernel (one selection spread over every SM, cooperative
// launch, for large vocabularies); logprob_kernel gives the log_softmax
// entries of an OpenAI `logprobs` answer.
//
// The selection pipeline of the reference's Sampler.select
// (npu_llm/runtime/sampling.py:416-445) on FP32 logits already in device
// memory, so a sampled request costs no logits copy and no host argsort:
//   1. repetition / presence / frequency penalties over the unique history
//      tokens (sampling.py:327-363), in FP32 exactly as NumPy rounds them;
//   2. logit bias (:366-380);  temperature 0 -> argmax (np.argmax order);
//   3. scores / temperature;  4. top-k: keep scores >= the k-th largest
//      (np.partition threshold, ties kept, :383-389);
//   5. top-p (:392-406): the candidates sorted by (score desc, index desc),
//      the softmax over that order, the FP32 running sum taken left to right
//      as np.cumsum does, and the prefix whose mass-before is < top_p kept;
//   6. the guarded softmax in index order (:409-421), its float64
//      renormalisation and Generator.choice's draw: the first index whose
//      normalised cumulative sum exceeds u, where u is the request
//      generator's next random(), drawn on the host so the random stream
//      stays the request's own.
// Every sum whose rounding reaches the result follows NumPy's order: the
// softmax denominators replay np.add.reduce's pairwise tree (leaves of
// 64-128 elements with eight accumulators, halves split at multiples of 8),
// precomputed on the host per vocabulary size (SamplePlan) and evaluated
// level by level here.  What still differs from NumPy is the float32 exp of
// each score (CUDA's expf against NumPy's) and, with more than
// kTopPMax top-p candidates, the order of the softmax denominator in step 5:
// both move probabilities by an ulp, so only a draw or a top-p cut lying
// within ~1e-6 of a boundary can select differently.  When the top-p
// nucleus is larger than kTopPMax candidates the kernel reports
// "unsupported" and the caller selects on the host instead.
#pragma once

#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include "hb_device.cuh"

namespace hb {

constexpr int kSampThreads = 1024;
constexpr int kSampWarps = kSampThreads / 32;
constexpr int kTopPMax = 4096;       // top-p candidates sorted on chip
constexpr int kSampMaxLeaves = 4096;
constexpr int kSampMaxVocab = kSampMaxLeaves * 64;  // every pairwise leaf holds >= 64 values

struct SampleParams {
  const float *logits;  // [V], device
  float *s;             // [V] working scores
  float *e;             // [V] shifted exponentials
  int V;
  float temperature, top_p, rep, pres, freq;
  int top_k;
  int n_hist;
  const int *hist_tok;     // unique in-vocabulary history tokens
  const float *hist_cnt;   // their counts
  int n_bias;
  const int *bias_tok;     // unique in-vocabulary tokens
  const float *bias_val;
  double u;
  // NumPy's pairwise tree for V values: leaves (first, count) left to right;
  // internal nodes (left id, right id), ids 0..n_leaves-1 are the leaves and
  // n_leaves + i is node i; nodes grouped by height, level h ending at
  // level_end[h]; the root is the last node (or leaf 0 when there is one).
  const int2 *leaves;
  int n_leaves;
  const int2 *nodes;
  int n_nodes;
  const int *level_end;
  int n_levels;
  int *out;  // [0] token, [1] status: 0 selected, 1 top-p nucleus too large
};

struct SampleSmem {
  double tree[2 * kSampMaxLeaves];
  unsigned long long keys[kTopPMax];  // (score key << 32) | index, for the top-p sort
  float probs[kTopPMax];
  unsigned int hist[kSampWarps][256];
  double wscan[kSampWarps];
  float wf[kSampWarps];
  int wi[kSampWarps];
  int misc[8];
  double dmisc[2];
};

// Monotone map of a float to an unsigned key (NaN above +inf, like np.sort).
__device__ __forceinline__ uint32_t samp_key(float f) {
  if (f != f) return 0xffffffffu;
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float samp_unkey(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Visit j = threadIdx.x + k * kSampThreads for k = 0, 1, ... with the loads
// of eight consecutive visits issued before their bodies run, so one CTA
// keeps enough loads in flight to stream the vector from L2.
template <class F>
__device__ __forceinline__ void samp_map(const float *src, int V, F &&body) {
  for (int base = threadIdx.x; base < V; base += 8 * kSampThreads) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int j = base + u * kSampThreads;
      v[u] = j < V ? src[j] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int j = base + u * kSampThreads;
      if (j < V) body(j, v[u]);
    }
  }
}

__device__ __forceinline__ float samp_add(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ double samp_add(double a, double b) { return __dadd_rn(a, b); }

// Leaf sums of NumPy's pairwise tree: leaves first, first + stride, ... (in
// blocks of 128 leaves) go to groups of eight lanes; lane j of a group keeps
// accumulator j (elements j, j + 8, ... of the leaf, read coalesced across
// the group), the eight are combined as ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7))
// with shuffles, and the group's first lane adds the tail left to right.
template <class T, class F>
__device__ void leaf_sums(const SampleParams &p, F &&elem, T *out, int first, int stride) {
  const int lane = threadIdx.x & 31, j = lane & 7;
  const int group = (threadIdx.x >> 3);  // 128 groups of 8 lanes
  for (int base = first; base < p.n_leaves; base += stride) {
    const int l = base + group;
    int lo = 0, n = 0;
    if (l < p.n_leaves) {
      const int2 lf = p.leaves[l];
      lo = lf.x;
      n = lf.y;
    }
    T r = T(0);
    if (n >= 8) {  // a leaf has at most 128 values: up to 16 per lane, loaded first
      const int whole = n - n % 8;
      T v[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) v[k] = 8 * k < whole ? elem(lo + 8 * k + j) : T(0);
      r = v[0];
#pragma unroll
      for (int k = 1; k < 16; ++k)
        if (8 * k < whole) r = samp_add(r, v[k]);
    }
    const T s1 = samp_add(r, __shfl_down_sync(0xffffffffu, r, 1));
    const T s2 = samp_add(s1, __shfl_down_sync(0xffffffffu, s1, 2));
    const T s4 = samp_add(s2, __shfl_down_sync(0xffffffffu, s2, 4));
    if (j == 0 && l < p.n_leaves) {
      T res;
      int i;
      if (n < 8) {
        res = T(0);
        i = 0;
      } else {
        res = s4;
        i = n - n % 8;
      }
      for (; i < n; ++i) res = samp_add(res, elem(lo + i));
      out[l] = res;
    }
  }
}

// Combine the leaf sums already in sm.tree one tree height per step; the
// root.  All threads of the block call it.
template <class T>
__device__ T tree_combine(const SampleParams &p, SampleSmem &sm) {
  T *vals = reinterpret_cast<T *>(sm.tree);
  int start = 0;
  for (int h = 0; h < p.n_levels; ++h) {
    const int end = p.level_end[h];
    for (int i = start + threadIdx.x; i < end; i += kSampThreads) {
      const int2 nd = p.nodes[i];
      vals[p.n_leaves + i] = samp_add(vals[nd.x], vals[nd.y]);
    }
    __syncthreads();
    start = end;
  }
  const T r = vals[p.n_nodes > 0 ? p.n_leaves + p.n_nodes - 1 : 0];
  __syncthreads();
  return r;
}

// Sum of elem(0..V-1) in NumPy's pairwise order.  All threads call it.
template <class T, class F>
__device__ T tree_sum(const SampleParams &p, SampleSmem &sm, F &&elem) {
  leaf_sums<T>(p, elem, reinterpret_cast<T *>(sm.tree), 0, kSampThreads / 8);
  __syncthreads();
  return tree_combine<T>(p, sm);
}

__device__ __forceinline__ float samp_block_max(SampleSmem &sm, float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) sm.wf[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = sm.wf[0];
  for (int w = 1; w < kSampWarps; ++w) r = fmaxf(r, sm.wf[w]);
  __syncthreads();
  return r;
}

__device__ __forceinline__ int samp_block_sum(SampleSmem &sm, int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) sm.wi[threadIdx.x >> 5] = v;
  __syncthreads();
  int r = 0;
  for (int w = 0; w < kSampWarps; ++w) r += sm.wi[w];
  __syncthreads();
  return r;
}

__device__ __forceinline__ int samp_block_min(SampleSmem &sm, int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) sm.wi[threadIdx.x >> 5] = v;
  __syncthreads();
  int r = sm.wi[0];
  for (int w = 1; w < kSampWarps; ++w) r = min(r, sm.wi[w]);
  __syncthreads();
  return r;
}

// Index of the maximum of s[0..V) in np.argmax order.
__device__ int samp_argmax(const SampleParams &p, SampleSmem &sm) {
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  samp_map(p.s, p.V, [&](int j, float v) { argmax_merge(bv, bi, v, j); });
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    argmax_merge(bv, bi, ov, oi);
  }
  if ((threadIdx.x & 31) == 0) {
    sm.wf[threadIdx.x >> 5] = bv;
    sm.wi[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  float v = sm.wf[0];
  int i = sm.wi[0];
  for (int w = 1; w < kSampWarps; ++w) argmax_merge(v, i, sm.wf[w], sm.wi[w]);
  __syncthreads();
  return i;
}

// Key of the k-th largest score (1 <= k <= V), duplicates counted: four
// 8-bit radix passes, per-warp histograms with warp-aggregated increments.
__device__ uint32_t samp_kth_largest(const SampleParams &p, SampleSmem &sm, int k) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t prefix = 0, mask = 0;
  int kk = k;
  const int vpad = (p.V + kSampThreads - 1) / kSampThreads * kSampThreads;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < kSampWarps * 256; i += kSampThreads) (&sm.hist[0][0])[i] = 0u;
    __syncthreads();
    for (int b0 = threadIdx.x; b0 < vpad; b0 += 4 * kSampThreads) {
      float v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int j = b0 + u * kSampThreads;
        v[u] = j < p.V ? p.s[j] : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int j = b0 + u * kSampThreads;
        int bin = 256;
        if (j < p.V) {
          const uint32_t key = samp_key(v[u]);
          if ((key & mask) == prefix) bin = (key >> shift) & 255;
        }
        const unsigned peers = __match_any_sync(0xffffffffu, bin);
        if (bin < 256 && lane == __ffs(peers) - 1) sm.hist[warp][bin] += __popc(peers);
      }
    }
    __syncthreads();
    if (threadIdx.x < 256) {
      unsigned c = 0;
      for (int w = 0; w < kSampWarps; ++w) c += sm.hist[w][threadIdx.x];
      sm.hist[0][threadIdx.x] = c;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int acc = 0, b = 255;
      for (; b > 0; --b) {
        if (acc + static_cast<int>(sm.hist[0][b]) >= kk) break;
        acc += static_cast<int>(sm.hist[0][b]);
      }
      sm.misc[0] = b;
      sm.misc[1] = kk - acc;
    }
    __syncthreads();
    prefix |= static_cast<uint32_t>(sm.misc[0]) << shift;
    mask |= 255u << shift;
    kk = sm.misc[1];
    __syncthreads();
  }
  return prefix;
}

// One selection by the whole thread block (see the file comment).
__device__ void sample_row(const SampleParams &p, SampleSmem &sm) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int V = p.V;
  float *s = p.s;

  // 1-2. working copy, penalties, bias (each token appears once per list)
  samp_map(p.logits, V, [&](int j, float v) { s[j] = v; });
  __syncthreads();
  for (int t = tid; t < p.n_hist; t += kSampThreads) {
    const int tok = p.hist_tok[t];
    float v = s[tok];
    if (p.rep != 1.0f) v = v > 0.f ? __fdiv_rn(v, p.rep) : __fmul_rn(v, p.rep);
    v = __fsub_rn(v, __fmul_rn(p.freq, p.hist_cnt[t]));
    v = __fsub_rn(v, p.pres);
    s[tok] = v;
  }
  __syncthreads();
  for (int t = tid; t < p.n_bias; t += kSampThreads) {
    const int tok = p.bias_tok[t];
    s[tok] = __fadd_rn(s[tok], p.bias_val[t]);
  }
  __syncthreads();
  if (p.temperature == 0.0f) {
    const int best = samp_argmax(p, sm);
    if (tid == 0) {
      p.out[0] = best;
      p.out[1] = 0;
    }
    return;
  }

  // 3. temperature
  samp_map(s, V, [&](int j, float v) { s[j] = __fdiv_rn(v, p.temperature); });
  __syncthreads();

  // 4. top-k
  if (p.top_k > 0 && p.top_k < V) {
    const float thr = samp_unkey(samp_kth_largest(p, sm, p.top_k));
    samp_map(s, V, [&](int j, float v) {
      if (v < thr) s[j] = -INFINITY;
    });
    __syncthreads();
  }

  // 5. top-p
  if (p.top_p < 1.0f) {
    int cand = 0;
    float peak = -INFINITY;
    samp_map(s, V, [&](int, float v) {
      if (isfinite(v)) {
        ++cand;
        peak = fmaxf(peak, v);
      }
    });
    const int C = samp_block_sum(sm, cand);
    peak = samp_block_max(sm, peak);
    // the candidates: every finite score, or those >= the kTopPMax-th largest
    uint32_t lo_key = 0u;
    if (C > kTopPMax) lo_key = samp_kth_largest(p, sm, kTopPMax);
    if (tid == 0) sm.misc[2] = 0;
    __syncthreads();
    const int vpad = (V + kSampThreads - 1) / kSampThreads * kSampThreads;
    for (int j = tid; j < vpad; j += kSampThreads) {
      bool take = false;
      uint32_t key = 0u;
      if (j < V) {
        const float v = s[j];
        key = samp_key(v);
        take = isfinite(v) && key >= lo_key;
      }
      const unsigned ballot = __ballot_sync(0xffffffffu, take);
      int base = 0;
      if (lane == 0 && ballot) base = atomicAdd(&sm.misc[2], __popc(ballot));
      base = __shfl_sync(0xffffffffu, base, 0);
      if (take) {
        const int slot = base + __popc(ballot & ((1u << lane) - 1u));
        if (slot < kTopPMax) sm.keys[slot] = (static_cast<unsigned long long>(key) << 32) | static_cast<uint32_t>(j);
      }
    }
    __syncthreads();
    const int cnt = sm.misc[2];
    if (cnt > kTopPMax) {  // ties at the cut overflow the on-chip sort
      if (tid == 0) {
        p.out[0] = -1;
        p.out[1] = 1;
      }
      return;
    }
    int n2 = 1;
    while (n2 < cnt) n2 <<= 1;
    for (int i = cnt + tid; i < n2; i += kSampThreads) sm.keys[i] = 0ull;
    __syncthreads();
    // bitonic sort, descending: score desc, then index desc
    for (int k = 2; k <= n2; k <<= 1) {
      for (int jj = k >> 1; jj > 0; jj >>= 1) {
        for (int i = tid; i < n2; i += kSampThreads) {
          const int ixj = i ^ jj;
          if (ixj > i) {
            const unsigned long long a = sm.keys[i], b = sm.keys[ixj];
            const bool desc = (i & k) == 0;
            if (desc ? (a < b) : (a > b)) {
              sm.keys[i] = b;
              sm.keys[ixj] = a;
            }
          }
        }
        __syncthreads();
      }
    }
    // softmax over the scores in sorted order: exp(score - peak), the
    // denominator over all V positions (non-candidates are 0)
    for (int i = tid; i < cnt; i += kSampThreads)
      sm.probs[i] = expf(__fsub_rn(samp_unkey(static_cast<uint32_t>(sm.keys[i] >> 32)), peak));
    __syncthreads();
    float total;
    if (C <= kTopPMax) {
      total = tree_sum<float>(p, sm, [&](int i) { return i < cnt ? sm.probs[i] : 0.f; });
    } else {
      // the tail's order is unknown: the denominator in index order instead
      samp_map(s, V, [&](int j, float v) { p.e[j] = isfinite(v) ? expf(__fsub_rn(v, peak)) : 0.f; });
      __syncthreads();
      total = tree_sum<float>(p, sm, [&](int j) { return p.e[j]; });
    }
    const bool degenerate = !(total > 0.f) || !isfinite(total);
    for (int i = tid; i < cnt; i += kSampThreads) sm.probs[i] = __fdiv_rn(sm.probs[i], total);
    __syncthreads();
    if (tid == 0) {
      int keep = -1;
      if (degenerate) {
        keep = 1;
      } else {
        float cum = 0.f;
        for (int i = 0; i < cnt; ++i) {
          const float pi = sm.probs[i];
          cum = __fadd_rn(cum, pi);
          if (i > 0 && !(__fsub_rn(cum, pi) < p.top_p)) {
            keep = i;
            break;
          }
        }
        if (keep < 0 && C <= kTopPMax) keep = cnt;  // every candidate kept
      }
      sm.misc[3] = keep;
    }
    __syncthreads();
    const int keep = sm.misc[3];
    if (keep < 0) {  // the nucleus extends past the sorted candidates
      if (tid == 0) {
        p.out[0] = -1;
        p.out[1] = 1;
      }
      return;
    }
    const uint32_t cut_key = static_cast<uint32_t>(sm.keys[keep - 1] >> 32);
    const float cut = samp_unkey(cut_key);
    samp_map(s, V, [&](int j, float v) {
      if (v < cut) s[j] = -INFINITY;
    });
    __syncthreads();
    for (int i = keep + tid; i < cnt; i += kSampThreads)  // ties with the cut beyond it
      if (static_cast<uint32_t>(sm.keys[i] >> 32) == cut_key) s[static_cast<uint32_t>(sm.keys[i])] = -INFINITY;
    __syncthreads();
  }

  // 6. guarded softmax in index order, float64 renormalisation, the draw
  float peak = -INFINITY;
  samp_map(s, V, [&](int, float v) {
    if (isfinite(v)) peak = fmaxf(peak, v);
  });
  peak = samp_block_max(sm, peak);
  if (!isfinite(peak)) peak = 0.f;
  samp_map(s, V, [&](int j, float v) { p.e[j] = isfinite(v) ? expf(__fsub_rn(v, peak)) : 0.f; });
  __syncthreads();
  const float total = tree_sum<float>(p, sm, [&](int j) { return p.e[j]; });
  if (!(total > 0.f) || !isfinite(total)) {  // every candidate underflowed
    const int best = samp_argmax(p, sm);
    if (tid == 0) {
      p.out[0] = best;
      p.out[1] = 0;
    }
    return;
  }
  // the float32 probabilities, in place
  float *e = p.e;
  samp_map(e, V, [&](int j, float v) { e[j] = __fdiv_rn(v, total); });
  __syncthreads();
  const double s64 = tree_sum<double>(p, sm, [&](int j) { return static_cast<double>(e[j]); });
  // Cumulative sums: warp w owns the contiguous segment w of the vector and
  // reads it 32 values at a time; warp sums, a scan over the warps, then
  // each warp walks its segment to the first crossing of u.  Scaling by
  // 1/s64 and comparing run > u * last instead of dividing moves the
  // boundaries by an ulp of a double, far below the float32 effects.
  const double inv = __ddiv_rn(1.0, s64);
  const int seg = (V + kSampWarps - 1) / kSampWarps;
  const int j0 = min(V, warp * seg), j1 = min(V, j0 + seg);
  double local = 0.0;
#pragma unroll 8
  for (int j = j0 + lane; j < j1; j += 32) local = __dadd_rn(local, __dmul_rn(static_cast<double>(e[j]), inv));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) local = __dadd_rn(local, __shfl_xor_sync(0xffffffffu, local, o));
  if (lane == 0) sm.wscan[warp] = local;
  __syncthreads();
  if (tid == 0) {
    double acc = 0.0;
    for (int w = 0; w < kSampWarps; ++w) {
      const double t = sm.wscan[w];
      sm.wscan[w] = acc;
      acc = __dadd_rn(acc, t);
    }
    sm.dmisc[0] = acc;
  }
  __syncthreads();
  const double last = sm.dmisc[0];
  const double target = __dmul_rn(p.u, last);
  double run = sm.wscan[warp];
  int first = 0x7fffffff;
  if (__dadd_rn(run, local) > target) {  // the crossing is in this segment
    for (int jb = j0; jb < j1; jb += 32) {
      const int jj = jb + lane;
      double v = jj < j1 ? __dmul_rn(static_cast<double>(e[jj]), inv) : 0.0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const double t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v = __dadd_rn(v, t);
      }
      const double here = __dadd_rn(run, v);
      const unsigned hit = __ballot_sync(0xffffffffu, jj < j1 && here > target);
      if (hit) {
        first = jb + __ffs(hit) - 1;
        break;
      }
      run = __dadd_rn(run, __shfl_sync(0xffffffffu, v, 31));
    }
  }
  first = samp_block_min(sm, first);
  if (tid == 0) {
    p.out[0] = first < V ? first : V - 1;
    p.out[1] = 0;
  }
}

__global__ void __launch_bounds__(kSampThreads, 1) sample_kernel(SampleParams p) {
  extern __shared__ __align__(16) uint8_t samp_smem_raw[];
  sample_row(p, *reinterpret_cast<SampleSmem *>(samp_smem_raw));
}

// Rows of a batch side by side: CTA b selects for ps[b] (its own logits row,
// parameters, history, scratch and result words).
__global__ void __launch_bounds__(kSampThreads, 1) sample_batch_kernel(const SampleParams *ps) {
  extern __shared__ __align__(16) uint8_t samp_smem_raw[];
  const SampleParams p = ps[blockIdx.x];
  sample_row(p, *reinterpret_cast<SampleSmem *>(samp_smem_raw));
}

// ---- the same selection spread over the grid (one row) --------------------
// A cooperative launch of one CTA per SM: each CTA owns a contiguous slice
// of the vocabulary for the element-wise work and the histograms, the leaf
// sums of NumPy's tree are dealt round-robin, and the steps that need the
// whole vector (tree roots, the top-p sort and running sum, the argmax and
// the draw's crossing) meet at grid barriers.  Same arithmetic as
// sample_row; only the draw's float64 running sums are grouped differently
// (an ulp of a double).
struct SampleGrid {
  float *leaf32;             // [n_leaves]
  double *leaf64;            // [n_leaves]
  float *cta_f;              // [G]
  int *cta_i;                // [G]
  double *cta_d;             // [G]
  unsigned *hist;            // [8][256], zeroed at the start of a launch
  unsigned long long *cand;  // [kTopPMax] top-p candidates
  int *ctr;                  // [0] candidates, [1] first crossing, [2] top-p keep, [3] cut key
  float *fs;                 // [0] softmax total
  double *ds;                // [0] float64 total
};

// Key of the k-th largest score over the grid (every CTA returns it).
__device__ uint32_t grid_kth_largest(const SampleParams &p, SampleSmem &sm, unsigned *hist4, int k, int lo, int hi,
                                     cooperative_groups::grid_group &grid) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t prefix = 0, mask = 0;
  int kk = k;
  const int span = hi - lo, pad = (span + kSampThreads - 1) / kSampThreads * kSampThreads;
  for (int r = 0; r < 4; ++r) {
    const int shift = 24 - 8 * r;
    unsigned *gh = hist4 + 256 * r;
    for (int i = threadIdx.x; i < kSampWarps * 256; i += kSampThreads) (&sm.hist[0][0])[i] = 0u;
    __syncthreads();
    for (int t = threadIdx.x; t < pad; t += kSampThreads) {
      int bin = 256;
      if (t < span) {
        const uint32_t key = samp_key(p.s[lo + t]);
        if ((key & mask) == prefix) bin = (key >> shift) & 255;
      }
      const unsigned peers = __match_any_sync(0xffffffffu, bin);
      if (bin < 256 && lane == __ffs(peers) - 1) sm.hist[warp][bin] += __popc(peers);
    }
    __syncthreads();
    if (threadIdx.x < 256) {
      unsigned c = 0;
      for (int w = 0; w < kSampWarps; ++w) c += sm.hist[w][threadIdx.x];
      if (c) atomicAdd(&gh[threadIdx.x], c);
    }
    grid.sync();
    if (threadIdx.x == 0) {
      int acc = 0, b = 255;
      for (; b > 0; --b) {
        const int c = static_cast<int>(__ldcg(&gh[b]));
        if (acc + c >= kk) break;
        acc += c;
      }
      sm.misc[0] = b;
      sm.misc[1] = kk - acc;
    }
    __syncthreads();
    prefix |= static_cast<uint32_t>(sm.misc[0]) << shift;
    mask |= 255u << shift;
    kk = sm.misc[1];
    __syncthreads();
  }
  return prefix;
}

// Block-wide inclusive scan of one double per thread; *total = block sum.
__device__ __forceinline__ double samp_block_scan(SampleSmem &sm, double v, double *total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v = __dadd_rn(v, t);
  }
  if (lane == 31) sm.wscan[warp] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    double acc = 0.0;
    for (int w = 0; w < kSampWarps; ++w) {
      const double t = sm.wscan[w];
      sm.wscan[w] = acc;
      acc = __dadd_rn(acc, t);
    }
    sm.dmisc[1] = acc;
  }
  __syncthreads();
  const double r = __dadd_rn(v, sm.wscan[warp]);
  *total = sm.dmisc[1];
  __syncthreads();
  return r;
}

// np.argmax order over this CTA's slice, merged over the grid by CTA 0
// (after the caller's grid barrier) from cta_f / cta_i.
__device__ void grid_argmax_partial(const SampleParams &p, SampleSmem &sm, const SampleGrid &g, int lo, int hi) {
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int j = lo + threadIdx.x; j < hi; j += kSampThreads) argmax_merge(bv, bi, p.s[j], j);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    argmax_merge(bv, bi, ov, oi);
  }
  if ((threadIdx.x & 31) == 0) {
    sm.wf[threadIdx.x >> 5] = bv;
    sm.wi[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = sm.wf[0];
    int i = sm.wi[0];
    for (int w = 1; w < kSampWarps; ++w) argmax_merge(v, i, sm.wf[w], sm.wi[w]);
    g.cta_f[blockIdx.x] = v;
    g.cta_i[blockIdx.x] = i;
  }
  __syncthreads();
}

__device__ int grid_argmax_merge(const SampleGrid &g) {
  float v = -INFINITY;
  int i = 0x7fffffff;
  for (int c = 0; c < static_cast<int>(gridDim.x); ++c) argmax_merge(v, i, __ldcg(&g.cta_f[c]), __ldcg(&g.cta_i[c]));
  return i;
}

__global__ void __launch_bounds__(kSampThreads, 1) sample_grid_kernel(SampleParams p, SampleGrid g) {
  extern __shared__ __align__(16) uint8_t samp_smem_raw[];
  SampleSmem &sm = *reinterpret_cast<SampleSmem *>(samp_smem_raw);
  cooperative_groups::grid_group grid = cooperative_groups::this_grid();
  const int G = gridDim.x, b = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
  const int V = p.V;
  const int lo = static_cast<int>(static_cast<long long>(V) * b / G);
  const int hi = static_cast<int>(static_cast<long long>(V) * (b + 1) / G);
  float *s = p.s;
  float *e = p.e;
  if (b == 0) {  // read only after the first grid barrier
    for (int i = tid; i < 8 * 256; i += kSampThreads) g.hist[i] = 0u;
    if (tid == 0) {
      g.ctr[0] = 0;
      g.ctr[1] = 0x7fffffff;
    }
  }
  // 1-2. this CTA's slice: copy, penalties, bias
  for (int j = lo + tid; j < hi; j += kSampThreads) s[j] = p.logits[j];
  __syncthreads();
  for (int t = tid; t < p.n_hist; t += kSampThreads) {
    const int tok = p.hist_tok[t];
    if (tok < lo || tok >= hi) continue;
    float v = s[tok];
    if (p.rep != 1.0f) v = v > 0.f ? __fdiv_rn(v, p.rep) : __fmul_rn(v, p.rep);
    v = __fsub_rn(v, __fmul_rn(p.freq, p.hist_cnt[t]));
    v = __fsub_rn(v, p.pres);
    s[tok] = v;
  }
  __syncthreads();
  for (int t = tid; t < p.n_bias; t += kSampThreads) {
    const int tok = p.bias_tok[t];
    if (tok >= lo && tok < hi) s[tok] = __fadd_rn(s[tok], p.bias_val[t]);
  }
  __syncthreads();
  if (p.temperature == 0.0f) {
    grid_argmax_partial(p, sm, g, lo, hi);
    grid.sync();
    if (b == 0 && tid == 0) {
      p.out[0] = grid_argmax_merge(g);
      p.out[1] = 0;
    }
    return;
  }
  // 3. temperature
  for (int j = lo + tid; j < hi; j += kSampThreads) s[j] = __fdiv_rn(s[j], p.temperature);
  __syncthreads();
  // 4. top-k
  if (p.top_k > 0 && p.top_k < V) {
    grid.sync();  // the zeroed histograms
    const float thr = samp_unkey(grid_kth_largest(p, sm, g.hist, p.top_k, lo, hi, grid));
    for (int j = lo + tid; j < hi; j += kSampThreads)
      if (s[j] < thr) s[j] = -INFINITY;
    __syncthreads();
  }
  // 5. top-p
  if (p.top_p < 1.0f) {
    int cand = 0;
    float peak = -INFINITY;
    for (int j = lo + tid; j < hi; j += kSampThreads) {
      const float v = s[j];
      if (isfinite(v)) {
        ++cand;
        peak = fmaxf(peak, v);
      }
    }
    cand = samp_block_sum(sm, cand);
    peak = samp_block_max(sm, peak);
    if (tid == 0) {
      g.cta_i[b] = cand;
      g.cta_f[b] = peak;
    }
    grid.sync();
    if (tid == 0) {
      int c = 0;
      float pk = -INFINITY;
      for (int x = 0; x < G; ++x) {
        c += __ldcg(&g.cta_i[x]);
        pk = fmaxf(pk, __ldcg(&g.cta_f[x]));
      }
      sm.misc[4] = c;
      sm.wf[0] = pk;
    }
    __syncthreads();
    const int C = sm.misc[4];
    peak = sm.wf[0];
    __syncthreads();
    uint32_t lo_key = 0u;
    if (C > kTopPMax) lo_key = grid_kth_largest(p, sm, g.hist + 4 * 256, kTopPMax, lo, hi, grid);
    const int span = hi - lo, pad = (span + kSampThreads - 1) / kSampThreads * kSampThreads;
    for (int t = tid; t < pad; t += kSampThreads) {
      bool take = false;
      uint32_t key = 0u;
      if (t < span) {
        const float v = s[lo + t];
        key = samp_key(v);
        take = isfinite(v) && key >= lo_key;
      }
      const unsigned ballot = __ballot_sync(0xffffffffu, take);
      int base = 0;
      if (lane == 0 && ballot) base = atomicAdd(&g.ctr[0], __popc(ballot));
      base = __shfl_sync(0xffffffffu, base, 0);
      if (take) {
        const int slot = base + __popc(ballot & ((1u << lane) - 1u));
        if (slot < kTopPMax) g.cand[slot] = (static_cast<unsigned long long>(key) << 32) | static_cast<uint32_t>(lo + t);
      }
    }
    if (C > kTopPMax) {
      for (int j = lo + tid; j < hi; j += kSampThreads) {
        const float v = s[j];
        e[j] = isfinite(v) ? expf(__fsub_rn(v, peak)) : 0.f;
      }
    }
    grid.sync();
    if (C > kTopPMax) {
      leaf_sums<float>(p, [&](int j) { return __ldcg(&e[j]); }, g.leaf32, b * (kSampThreads / 8), G * (kSampThreads / 8));
      grid.sync();
    }
    if (b == 0) {
      const int cnt = __ldcg(&g.ctr[0]);
      if (cnt > kTopPMax) {
        if (tid == 0) g.ctr[2] = -1;
      } else {
        int n2 = 1;
        while (n2 < cnt) n2 <<= 1;
        for (int i = tid; i < n2; i += kSampThreads) sm.keys[i] = i < cnt ? __ldcg(&g.cand[i]) : 0ull;
        __syncthreads();
        for (int k = 2; k <= n2; k <<= 1) {
          for (int jj = k >> 1; jj > 0; jj >>= 1) {
            for (int i = tid; i < n2; i += kSampThreads) {
              const int ixj = i ^ jj;
              if (ixj > i) {
                const unsigned long long x = sm.keys[i], y = sm.keys[ixj];
                const bool desc = (i & k) == 0;
                if (desc ? (x < y) : (x > y)) {
                  sm.keys[i] = y;
                  sm.keys[ixj] = x;
                }
              }
            }
            __syncthreads();
          }
        }
        for (int i = tid; i < cnt; i += kSampThreads)
          sm.probs[i] = expf(__fsub_rn(samp_unkey(static_cast<uint32_t>(sm.keys[i] >> 32)), peak));
        __syncthreads();
        float total;
        if (C <= kTopPMax) {
          total = tree_sum<float>(p, sm, [&](int i) { return i < cnt ? sm.probs[i] : 0.f; });
        } else {
          float *vals = reinterpret_cast<float *>(sm.tree);
          for (int l = tid; l < p.n_leaves; l += kSampThreads) vals[l] = __ldcg(&g.leaf32[l]);
          __syncthreads();
          total = tree_combine<float>(p, sm);
        }
        const bool degenerate = !(total > 0.f) || !isfinite(total);
        for (int i = tid; i < cnt; i += kSampThreads) sm.probs[i] = __fdiv_rn(sm.probs[i], total);
        __syncthreads();
        if (tid == 0) {
          int keep = -1;
          if (degenerate) {
            keep = 1;
          } else {
            float cum = 0.f;
            for (int i = 0; i < cnt; ++i) {
              const float pi = sm.probs[i];
              cum = __fadd_rn(cum, pi);
              if (i > 0 && !(__fsub_rn(cum, pi) < p.top_p)) {
                keep = i;
                break;
              }
            }
            if (keep < 0 && C <= kTopPMax) keep = cnt;
          }
          sm.misc[3] = keep;
          g.ctr[2] = keep;
          if (keep > 0) g.ctr[3] = static_cast<int>(static_cast<uint32_t>(sm.keys[keep - 1] >> 32));
        }
        __syncthreads();
        const int keep = sm.misc[3];
        if (keep > 0) {
          const uint32_t cut_key = static_cast<uint32_t>(sm.keys[keep - 1] >> 32);
          for (int i = keep + tid; i < cnt; i += kSampThreads)  // ties with the cut beyond it
            if (static_cast<uint32_t>(sm.keys[i] >> 32) == cut_key) s[static_cast<uint32_t>(sm.keys[i])] = -INFINITY;
        }
      }
    }
    grid.sync();
    const int keep = __ldcg(&g.ctr[2]);
    if (keep < 0) {  // the nucleus extends past the sorted candidates
      if (b == 0 && tid == 0) {
        p.out[0] = -1;
        p.out[1] = 1;
      }
      return;
    }
    const float cut = samp_unkey(static_cast<uint32_t>(__ldcg(&g.ctr[3])));
    for (int j = lo + tid; j < hi; j += kSampThreads)
      if (s[j] < cut) s[j] = -INFINITY;
    __syncthreads();
  }
  // 6. guarded softmax in index order, float64 renormalisation, the draw
  float peak = -INFINITY;
  for (int j = lo + tid; j < hi; j += kSampThreads)
    if (isfinite(s[j])) peak = fmaxf(peak, s[j]);
  peak = samp_block_max(sm, peak);
  grid_argmax_partial(p, sm, g, lo, hi);  // for the degenerate case below
  if (tid == 0) g.cta_d[b] = static_cast<double>(peak);
  grid.sync();
  if (tid == 0) {
    double pk = -INFINITY;
    for (int x = 0; x < G; ++x) pk = fmax(pk, __ldcg(&g.cta_d[x]));
    sm.wf[0] = static_cast<float>(pk);
  }
  __syncthreads();
  peak = sm.wf[0];
  if (!isfinite(peak)) peak = 0.f;
  __syncthreads();
  for (int j = lo + tid; j < hi; j += kSampThreads) {
    const float v = s[j];
    e[j] = isfinite(v) ? expf(__fsub_rn(v, peak)) : 0.f;
  }
  grid.sync();
  leaf_sums<float>(p, [&](int j) { return __ldcg(&e[j]); }, g.leaf32, b * (kSampThreads / 8), G * (kSampThreads / 8));
  grid.sync();
  if (b == 0) {
    float *vals = reinterpret_cast<float *>(sm.tree);
    for (int l = tid; l < p.n_leaves; l += kSampThreads) vals[l] = __ldcg(&g.leaf32[l]);
    __syncthreads();
    const float total = tree_combine<float>(p, sm);
    if (tid == 0) g.fs[0] = total;
  }
  grid.sync();
  const float total = __ldcg(&g.fs[0]);
  if (!(total > 0.f) || !isfinite(total)) {  // every candidate underflowed
    if (b == 0 && tid == 0) {
      p.out[0] = grid_argmax_merge(g);
      p.out[1] = 0;
    }
    return;
  }
  for (int j = lo + tid; j < hi; j += kSampThreads) e[j] = __fdiv_rn(e[j], total);
  grid.sync();
  leaf_sums<double>(p, [&](int j) { return static_cast<double>(__ldcg(&e[j])); }, g.leaf64, b * (kSampThreads / 8),
                    G * (kSampThreads / 8));
  grid.sync();
  if (b == 0) {
    double *vals = reinterpret_cast<double *>(sm.tree);
    for (int l = tid; l < p.n_leaves; l += kSampThreads) vals[l] = __ldcg(&g.leaf64[l]);
    __syncthreads();
    const double s64 = tree_combine<double>(p, sm);
    if (tid == 0) g.ds[0] = s64;
  }
  grid.sync();
  const double inv = __ddiv_rn(1.0, __ldcg(&g.ds[0]));
  // this CTA's float64 sum, in tiles of one value per thread
  double mine = 0.0;
  for (int base = lo; base < hi; base += kSampThreads) {
    const int j = base + tid;
    double tile;
    samp_block_scan(sm, j < hi ? __dmul_rn(static_cast<double>(e[j]), inv) : 0.0, &tile);
    mine = __dadd_rn(mine, tile);
  }
  if (tid == 0) g.cta_d[b] = mine;
  grid.sync();
  if (tid == 0) {
    double before = 0.0, last = 0.0;
    for (int x = 0; x < G; ++x) {
      const double v = __ldcg(&g.cta_d[x]);
      if (x < b) before = __dadd_rn(before, v);
      last = __dadd_rn(last, v);
    }
    sm.dmisc[0] = before;
    sm.dmisc[1] = __dmul_rn(p.u, last);
  }
  __syncthreads();
  double run = sm.dmisc[0];
  const double target = sm.dmisc[1];
  __syncthreads();
  if (__dadd_rn(run, mine) > target) {  // the crossing is in this slice (block-uniform)
    for (int base = lo; base < hi; base += kSampThreads) {
      const int j = base + tid;
      double tile;
      const double incl = samp_block_scan(sm, j < hi ? __dmul_rn(static_cast<double>(e[j]), inv) : 0.0, &tile);
      const int hit = (j < hi && __dadd_rn(run, incl) > target) ? j : 0x7fffffff;
      const int first = samp_block_min(sm, hit);
      if (first != 0x7fffffff) {
        if (tid == 0) atomicMin(&g.ctr[1], first);
        break;
      }
      run = __dadd_rn(run, tile);
    }
  }
  grid.sync();
  if (b == 0 && tid == 0) {
    const int first = __ldcg(&g.ctr[1]);
    p.out[0] = first < V ? first : V - 1;
    p.out[1] = 0;
  }
}

// Log-probabilities for an OpenAI ``logprobs`` entry: the reference's
// log_softmax (npu_llm/runtime/stopping.py:101-109: float64 scores, the
// finite maximum subtracted, log of the pairwise float64 sum of exp) at
// `token`, and the n_top largest entries (np.argpartition + argsort,
// descending; equal scores by index descending).  Reads the raw logits.
// out_vals[0] = token's log-probability, out_vals[1 + i] / out_ids[i] the
// i-th largest; out_ids[n_top] = 1 when there was no finite score.
constexpr int kMaxTopLogprobs = 32;

__global__ void __launch_bounds__(kSampThreads, 1) logprob_kernel(SampleParams p, int token, int n_top,
                                                                  double *out_vals, int *out_ids) {
  extern __shared__ __align__(16) uint8_t samp_smem_raw[];
  SampleSmem &sm = *reinterpret_cast<SampleSmem *>(samp_smem_raw);
  const int tid = threadIdx.x, lane = tid & 31;
  const int V = p.V;
  float *s = p.s;
  float peak = -INFINITY;
  int finite = 0;
  samp_map(p.logits, V, [&](int j, float v) {
    s[j] = v;
    if (isfinite(v)) {
      peak = fmaxf(peak, v);
      ++finite;
    }
  });
  __syncthreads();
  peak = samp_block_max(sm, peak);
  finite = samp_block_sum(sm, finite);
  if (finite == 0) {
    if (tid == 0) out_ids[n_top] = 1;
    return;
  }
  const double dpeak = static_cast<double>(peak);
  const double total = tree_sum<double>(p, sm, [&](int j) {
    const float v = s[j];
    return isfinite(v) ? exp(__dsub_rn(static_cast<double>(v), dpeak)) : 0.0;
  });
  const double lse = log(total);
  auto logprob = [&](float v) {
    return isfinite(v) ? __dsub_rn(__dsub_rn(static_cast<double>(v), dpeak), lse) : -INFINITY;
  };
  // the n_top largest: every score >= the n_top-th largest, sorted on chip
  uint32_t thr = 0u;
  if (n_top > 0 && n_top < V) thr = samp_kth_largest(p, sm, n_top);
  if (tid == 0) sm.misc[2] = 0;
  __syncthreads();
  if (n_top > 0) {
    const int vpad = (V + kSampThreads - 1) / kSampThreads * kSampThreads;
    for (int j = tid; j < vpad; j += kSampThreads) {
      bool take = false;
      uint32_t key = 0u;
      if (j < V) {
        key = samp_key(s[j]);
        take = key >= thr;
      }
      const unsigned ballot = __ballot_sync(0xffffffffu, take);
      int base = 0;
      if (lane == 0 && ballot) base = atomicAdd(&sm.misc[2], __popc(ballot));
      base = __shfl_sync(0xffffffffu, base, 0);
      if (take) {
        const int slot = base + __popc(ballot & ((1u << lane) - 1u));
        if (slot < kTopPMax) sm.keys[slot] = (static_cast<unsigned long long>(key) << 32) | static_cast<uint32_t>(j);
      }
    }
    __syncthreads();
  }
  if (tid == 0) {
    const int cnt = min(sm.misc[2], kTopPMax);
    // selection sort of the first n_top (n_top <= kMaxTopLogprobs)
    for (int i = 0; i < n_top && i < cnt; ++i) {
      int best = i;
      for (int k = i + 1; k < cnt; ++k)
        if (sm.keys[k] > sm.keys[best]) best = k;
      const unsigned long long t = sm.keys[i];
      sm.keys[i] = sm.keys[best];
      sm.keys[best] = t;
      const int idx = static_cast<int>(static_cast<uint32_t>(sm.keys[i]));
      out_ids[i] = idx;
      out_vals[1 + i] = logprob(s[idx]);
    }
    out_vals[0] = logprob(s[token]);
    out_ids[n_top] = 0;
  }
}

}  // namespace hb
