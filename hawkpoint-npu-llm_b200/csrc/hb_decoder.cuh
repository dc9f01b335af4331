// hb_decoder.cuh -- the persistent decode kernel.
//
// One cooperative launch (one CTA per SM, all co-resident) runs a range of
// phases of one decode step for up to MB batch rows.  Per layer l:
//   1 (4l+0)  x = rmsnorm(h) ; qkv = bf16(bf16(Wqkv x) + bias)       (cpu_backend.py:131-143)
//   2 (4l+1)  RoPE on q,k ; append k,v to the KV cache ; GQA attention, one
//             (row, head) per CTA ; h1 = bf16(bf16(Wo a) + h)            (cpu_backend.py:78-151)
//   3 (4l+2)  x2 = rmsnorm(h1) ; act = bf16(silu(bf16 gate) * bf16 up) (cpu_backend.py:152-165)
//   4 (4l+3)  h' = bf16(bf16(Wdown act) + h1)                           (cpu_backend.py:166-171)
// and after the last layer
//   E (4L)    logits = W_lm rmsnorm(h) (FP32) ; argmax, first maximum
//                                                    (cpu_backend.py:173-181, generate.py:709-714)
// Each phase's CTAs own a contiguous share of the projection rows.  Results
// move between CTAs through "LL" words in global memory: one 64-bit store of
// {32-bit payload, 32-bit epoch}, read with 64-bit loads until the epoch
// matches this launch's.  A reader therefore needs no barrier and no fence:
// a word is valid exactly when its epoch is current.  Every (layer, phase)
// has its own buffer, so no word is rewritten within a launch.
//
// A producer warp streams every weight chunk through the shared-memory ring
// (hb_stream.cuh) without waiting on activations, so HBM keeps streaming
// while consumers wait for the previous phase's words.  Phase 2 splits the
// attention into (batch row, q head) units, one per CTA: the unit copies its
// K/V history from the cache (L2) with cp.async while it waits for q/k/v,
// publishes its 64 outputs as LL words, and every CTA gathers all heads for
// the o-projection.
//
// KV cache layout per (slot, layer, kv head): K [CTX][64] then V [CTX][64],
// each row of 128 bytes with its eight 16-byte blocks XOR-swizzled by the
// position (block cb of row s at s*128 + (cb ^ (s & 7))*16), so tensor-core
// fragment loads (ldmatrix) of 8 consecutive positions are bank-conflict
// free.
//
// Contexts longer than 64 positions (paged mode) keep the cache in pages of
// 64 positions, each laid out as one 64-position slot above
// ([L][KVH][K | V][64][128 B], same swizzle); a per-slot page table maps
// position s to page table[slot][s / 64].  The attention phase then splits
// each (row, q head) unit's positions over up to G / (rows * QH) CTAs: each
// split publishes its partial (max, sum of exp, unnormalised P.V) to global
// scratch, and the last split to arrive combines them and publishes the
// head's outputs.
#pragma once

#include "hb_attn.cuh"
#include "hb_stream.cuh"

namespace hb {

constexpr int kMaxBatch = 8;
constexpr int kHeadDim = 64;
constexpr int kPagePositions = 64;    // positions per KV page (paged mode)
constexpr int kMaxPagedContext = 4096;
constexpr int kSplitPositions = 128;  // positions per attention split, at least
constexpr int kPartStride = 68;       // floats per split partial: P.V [64], max, sum
constexpr int kMaxHPerThread = 8;  // hidden <= 8 * 224 = 1792 (two word pairs per thread)

struct LayerPtrs {
  const float *gamma_in, *gamma_post, *bias;
  const uint8_t *w_qkv;
  const float *s_qkv;
  const uint8_t *w_o;
  const float *s_o;
  const uint8_t *w_gu;
  const float *s_gu;
  const uint8_t *w_down;
  const float *s_down;
};

// Inputs of a step, in device memory.  In chained mode (device-resident
// greedy generation) the last CTA also advances row 0: next position, next
// token (the prompt's, or this step's argmax).
struct StepState {
  int token[kMaxBatch];
  int pos[kMaxBatch];
  int slot[kMaxBatch];
  int rows;
  int chained;
  int n_prompt;
  int n_out;
};

// Result block, read back with one device->host copy per call.
struct Result {
  Ctrl ctrl;
  int out_token[kMaxBatch];
};

struct DecParams {
  int H, I, QH, KVH, L, V, CTX, QKV, group, has_bias;
  float eps;
  int kc_h, kc_i;   // 16-byte chunk columns of K = hidden, intermediate
  const LayerPtrs *layers;
  const float *gamma_final;
  const uint8_t *w_lm;
  const float *s_lm;
  const __nv_bfloat16 *embed;
  const float *rope_cos, *rope_sin;  // [CTX][32]
  __nv_bfloat16 *kv;                 // [slots][L][KVH][K CTXx64 | V CTXx64], swizzled rows
                                     // (paged: [pages][L][KVH][K 64x64 | V 64x64])
  uint64_t *ll;                      // LL words, see ll_* below
  float *logits;                     // [MB][V]
  float *part_val;                   // [G][kMaxBatch]
  int *part_idx;
  Result *result;
  StepState *st;
  unsigned int *epoch;               // tags this launch's LL words; the last CTA increments it
  const int *prompt;                 // chained: token of each prompt position
  int *gen_out;                      // chained: generated tokens
  int phase_begin, phase_end;
  int write_logits;
  int red_rows;
  int nslots;
  int xs_elems;                      // BF16 elements per batch row of xs
  uint64_t limit_ns;
  uint64_t stall_ns;
  unsigned long long *trace;         // optional [G][4L+2][4] phase timestamps
  int paged;                         // CTX > 64: the cache is paged (the PG kernels)
  int pages_per_slot, n_pages;
  const int *page_table;             // paged: [slots][pages_per_slot] page ids
  float *att_part;                   // paged: [G][kPartStride] split partials
  int *att_cnt;                      // paged: [kMaxBatch * QH] split arrivals (reset by the last)
};

// LL buffer layout: per layer a block of kMaxBatch rows of each kind
// (q/k/v, h1, act, h_out, attention output).
__host__ __device__ inline size_t ll_layer_words(int H, int I, int QKV) {
  return static_cast<size_t>(kMaxBatch) * (QKV + 3 * H + I) / 2;
}

struct SmemPlan {
  size_t ring, full, empty, xs, hx, red, att, kv, misc, total;
};

__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Attention scratch of one (row, head) unit: its q/k/v words [96], rotated
// q [64], scores / probabilities [64], P.V partial sums [4][64] (FP32), and
// the k/v words of up to kMaxBatch - 1 earlier positions of the same slot in
// this launch [7][64].
constexpr int kUnitWords = 96 + 64 + 64 + 256;
__host__ __device__ inline size_t att_bytes(int /*QH*/, int /*ctx*/) {
  return (static_cast<size_t>(kUnitWords) + (kMaxBatch - 1) * 64) * 4;
}

__host__ __device__ inline SmemPlan smem_plan(int nslots, int mb, int xs_elems, int H, int QKV,
                                              int QH, int KVH, int red_rows, int ctx, bool paged) {
  SmemPlan s;
  size_t o = 0;
  s.ring = o;
  o += static_cast<size_t>(nslots) * kSlotBytes;
  s.full = o;
  o += 8 * nslots;
  s.empty = o;
  o += 8 * nslots;
  o = align_up(o, 128);
  s.xs = o;  // xs[m] = BF16 GEMV input of row m
  o += align_up(static_cast<size_t>(mb) * xs_elems * 2, 128);
  // hx[m] = BF16 residual row (the phase's norm input / residual)
  s.hx = o;
  o += align_up(static_cast<size_t>(mb) * H * 2, 128);
  // attention scratch and the split-K partials share one region: attention
  // ends (barrier) before the phase's GEMV writes partials, and the next
  // attention starts after the previous phase's epilogue read them
  const size_t red_bytes = align_up(static_cast<size_t>(kWarps) * mb * red_rows * 4, 128);
  const size_t att_b = align_up(att_bytes(QH, ctx), 128);
  // paged mode: K/V rows of this launch's positions [2][8][128 B], the
  // per-warp P.V partials [kWarps][64] and the split's scores [ctx]
  const size_t kv_b = paged
                          ? align_up(static_cast<size_t>(2) * kMaxBatch * 128 + kWarps * 64 * 4 + 4 * ctx, 128)
                          : align_up(static_cast<size_t>(2) * ctx * 128, 128);
  s.red = o;
  s.att = o;
  s.kv = o + att_b;  // K then V history of one (row, kv head): [2][ctx][128 B]
  o += red_bytes > att_b + kv_b ? red_bytes : att_b + kv_b;
  s.misc = o;
  o += 1024;
  s.total = o;
  return s;
}

// ---- LL words ---------------------------------------------------------------
__device__ __forceinline__ void ll_store(uint64_t *p, uint32_t data, uint32_t epoch) {
  const uint64_t v = (static_cast<uint64_t>(epoch) << 32) | data;
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ll_load(const uint64_t *p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Two adjacent LL words in one 16-byte load (p 16-byte aligned).  Each
// 8-byte half is read whole, so each word's payload and epoch still agree;
// the two halves may come from different epochs and are checked apart.
__device__ __forceinline__ void ll_load2(const uint64_t *p, uint64_t &a, uint64_t &b) {
  asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}


// All consumer threads: wait until words [0, words) of each of `rows` rows
// (row m at src + m * row_words) carry `epoch`, and pass each payload to
// sink(m, word, payload).  Words travel in aligned pairs, one 16-byte load
// per pair (words even and < 65536, row_words even, src 16-byte aligned): pair p of every
// row goes to thread p % kConsumerThreads, so a thread owns the same words
// (2p, 2p + 1) of each row.  All rows are polled together, up to U pairs per
// thread in flight: 6 for one row (the 4,864-value activation gather in one
// round instead of two: 0.492 against 0.496 ms a decode step; 8 pushed the
// kernel to 254 registers and slowed its GEMV loops), 8 for 8 rows,
// where the deeper queue halves the rounds of the 8 x 4864 activation gather
// (6 in the int8-weight 8-row kernel, which has fewer registers to spare).
template <int U, class Sink>
__device__ __forceinline__ bool ll_gather(const uint64_t *src, size_t row_words, int words, int rows,
                                          uint32_t epoch, Ctrl *ctrl, uint64_t limit_ns, Sink &&sink) {
  const int tid = threadIdx.x;
  const int pairs = words >> 1;
  const int per_row = (pairs + kConsumerThreads - 1) / kConsumerThreads;  // pairs per thread and row
  const int total = rows * per_row;
  for (int base = 0; base < total; base += U) {
    uint32_t pend = 0;  // bits 2u and 2u + 1: the two words of slot u
    int rc[U];          // (row << 16) | first word of the pair
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int e = base + u;
      const int m = e / per_row, k = e - m * per_row;
      const int col = 2 * (tid + k * kConsumerThreads);
      rc[u] = (m << 16) | (col & 0xffff);
      if (e < total && col < words) pend |= 3u << (2 * u);
    }
    uint64_t start = 0;
    uint32_t spins = 0;
    while (pend) {
      uint64_t v0[U], v1[U];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (pend & (3u << (2 * u))) ll_load2(src + (rc[u] >> 16) * row_words + (rc[u] & 0xffff), v0[u], v1[u]);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if ((pend & (1u << (2 * u))) && static_cast<uint32_t>(v0[u] >> 32) == epoch) {
          sink(rc[u] >> 16, rc[u] & 0xffff, static_cast<uint32_t>(v0[u]));
          pend &= ~(1u << (2 * u));
        }
        if ((pend & (2u << (2 * u))) && static_cast<uint32_t>(v1[u] >> 32) == epoch) {
          sink(rc[u] >> 16, (rc[u] & 0xffff) + 1, static_cast<uint32_t>(v1[u]));
          pend &= ~(2u << (2 * u));
        }
      }
      if (pend) {
        if (start == 0) start = globaltimer_ns();
        if ((++spins & 31u) == 0 && wait_expired(ctrl, start, limit_ns, kWhereGrid)) return false;
      }
    }
  }
  return true;
}

template <int MB, bool W8, bool PG>  // PG: paged KV cache (context > 64)
struct DecoderCta {
  const DecParams &P;
  Ring ring;
  __nv_bfloat16 *xs;
  __nv_bfloat16 *hx;  // BF16 residual rows [MB][H]
  float *red, *att;
  uint8_t *kvs;       // K/V history of the current batch row (attention phase)
  int *s_tok, *s_pos, *s_slot, *s_misc;
  float *s_norm;      // [kWarps * kMaxBatch] partial sums, then [kMaxBatch] inverse rms
  float *s_bestv;     // [kWarps * kMaxBatch]
  int *s_besti;
  int cta, G, mrows, tid;
  uint32_t epoch;
  size_t lw;          // LL words per layer block

  __device__ DecoderCta(const DecParams &p, uint8_t *smem) : P(p) {
    const SmemPlan sp = smem_plan(P.nslots, MB, P.xs_elems, P.H, P.QKV, P.QH, P.KVH, P.red_rows, P.CTX, PG);
    ring.slots = smem + sp.ring;
    ring.full = reinterpret_cast<uint64_t *>(smem + sp.full);
    ring.empty = reinterpret_cast<uint64_t *>(smem + sp.empty);
    ring.nslots = P.nslots;
    ring.slot = 0;
    ring.parity = 0;
    xs = reinterpret_cast<__nv_bfloat16 *>(smem + sp.xs);
    hx = reinterpret_cast<__nv_bfloat16 *>(smem + sp.hx);
    red = reinterpret_cast<float *>(smem + sp.red);
    att = reinterpret_cast<float *>(smem + sp.att);
    kvs = smem + sp.kv;
    int *mi = reinterpret_cast<int *>(smem + sp.misc);
    s_tok = mi;
    s_pos = mi + kMaxBatch;
    s_slot = mi + 2 * kMaxBatch;
    s_misc = mi + 3 * kMaxBatch;  // [0] rows, [1] last-CTA flag, [2] epoch
    s_norm = reinterpret_cast<float *>(mi + 4 * kMaxBatch);
    s_bestv = s_norm + kWarps * kMaxBatch + kMaxBatch;
    s_besti = reinterpret_cast<int *>(s_bestv + kWarps * kMaxBatch);
    cta = blockIdx.x;
    G = gridDim.x;
    tid = threadIdx.x;
    mrows = 0;
    epoch = 0;
    lw = ll_layer_words(P.H, P.I, P.QKV);
  }

  // ---- LL buffers of layer l, batch row m ----------------------------------
  __device__ uint64_t *ll_qkv(int l, int m) const { return P.ll + l * lw + static_cast<size_t>(m) * P.QKV / 2; }
  __device__ uint64_t *ll_h1(int l, int m) const {
    return P.ll + l * lw + static_cast<size_t>(kMaxBatch) * P.QKV / 2 + static_cast<size_t>(m) * P.H / 2;
  }
  __device__ uint64_t *ll_act(int l, int m) const {
    return P.ll + l * lw + static_cast<size_t>(kMaxBatch) * (P.QKV + P.H) / 2 + static_cast<size_t>(m) * P.I / 2;
  }
  __device__ uint64_t *ll_hout(int l, int m) const {
    return P.ll + l * lw + static_cast<size_t>(kMaxBatch) * (P.QKV + P.H + P.I) / 2 +
           static_cast<size_t>(m) * P.H / 2;
  }
  __device__ uint64_t *ll_att(int l, int m) const {
    return P.ll + l * lw + static_cast<size_t>(kMaxBatch) * (P.QKV + 2 * P.H + P.I) / 2 +
           static_cast<size_t>(m) * P.H / 2;
  }

  // ---- work split -------------------------------------------------------------
  // Gate/up pair blocks [gu_lo(n, c), gu_lo(n, c + 1)) of CTA c: n / G each,
  // and the n % G left over go to CTAs that own no down-projection row group
  // (down gives CTA c split_lo(H/8, G, c + 1) - split_lo(H/8, G, c) groups,
  // 0 or 1), so no CTA streams both an extra gate/up block and a down row
  // group in one layer: the largest per-layer weight share a CTA's ring must
  // hold drops from qkv + o + 5 gate/up blocks + down to 4 blocks + down.
  // When the leftover exceeds those CTAs, the plain balanced split.
  __device__ int gu_lo(int n, int c) const {
    const int hg = P.H / 8, base = n / G, rem = n - base * G;
    if (hg > G || rem > G - hg) return split_lo(n, G, c);
    const int nodown = c - split_lo(hg, G, c);  // CTAs before c without a down group
    return base * c + min(rem, nodown);
  }

  __device__ MatRange phase_range(int k) const {
    if (k >= 4 * P.L) {
      const int n = P.V / 8;
      return MatRange{P.w_lm, split_lo(n, G, cta), split_lo(n, G, cta + 1), P.kc_h};
    }
    const LayerPtrs &lp = P.layers[k >> 2];
    switch (k & 3) {
      case 0: {
        const int n = P.QKV / 8;
        return MatRange{lp.w_qkv, split_lo(n, G, cta), split_lo(n, G, cta + 1), P.kc_h};
      }
      case 1: {
        const int n = P.H / 8;
        return MatRange{lp.w_o, split_lo(n, G, cta), split_lo(n, G, cta + 1), P.kc_h};
      }
      case 2: {
        const int n = P.I / 8;  // gate/up pair blocks
        return MatRange{lp.w_gu, 2 * gu_lo(n, cta), 2 * gu_lo(n, cta + 1), P.kc_h};
      }
      default: {
        const int n = P.H / 8;
        return MatRange{lp.w_down, split_lo(n, G, cta), split_lo(n, G, cta + 1), P.kc_i};
      }
    }
  }

  // K (kind 0) or V (kind 1) block of one kv head of one slot/layer.
  __device__ __nv_bfloat16 *kv_block(int slot, int layer, int kvh, int kind) const {
    return P.kv + (((static_cast<size_t>(slot) * P.L + layer) * P.KVH + kvh) * 2 + kind) *
                      static_cast<size_t>(P.CTX) * kHeadDim;
  }

  // trace point (0 start, 1 inputs ready, 6 prologue (norm / attention)
  // done, 2 weights consumed, 3 outputs stored; slot 5 holds the producer's
  // first issue of the phase, slots 4 and 7 are unused)
  __device__ __forceinline__ void mark(int k, int point) const {
    if (P.trace && tid == 0) {
      unsigned long long *t = P.trace + (static_cast<size_t>(cta) * (4 * P.L + 2) + k) * 8;
      t[point] = globaltimer_ns();
    }
  }

  // ---- helpers -------------------------------------------------------------------
  // Per-thread registers of a norm weight vector: the thread owns the
  // hidden-vector words (element pairs) 2p and 2p + 1 of the word pairs
  // p = tid + kConsumerThreads * j, the same words ll_gather hands it, so
  // gather and norm need no barrier between them.  Word n of the thread is
  // word 2 (tid + kConsumerThreads (n / 2)) + n % 2 of the row.
  static constexpr int kNormWords = kMaxHPerThread / 2;
  __device__ __forceinline__ int norm_word(int n) const { return 2 * (tid + (n >> 1) * kConsumerThreads) + (n & 1); }
  struct Gamma {
    float v[kMaxHPerThread];
  };
  __device__ Gamma load_gamma(const float *g) const {
    Gamma r;
#pragma unroll
    for (int j = 0; j < kNormWords; ++j) {
      const int w = norm_word(j);
      const bool in = 2 * w < P.H;
      r.v[2 * j] = in ? g[2 * w] : 0.f;
      r.v[2 * j + 1] = in ? g[2 * w + 1] : 0.f;
    }
    return r;
  }
  // Two consecutive per-row constants (bias / W8 scales) of this thread's
  // first epilogue pair, loaded early; 0 when absent.
  __device__ float2 load_pair(const float *base, int row0, int npairs) const {
    float2 r = make_float2(0.f, 0.f);
    if (base != nullptr && tid < npairs) {
      r.x = base[row0 + 2 * tid];
      r.y = base[row0 + 2 * tid + 1];
    }
    return r;
  }

  // xs[m][i] = bf16((v * inv_rms) * gamma) for v = hx[m][:]  (cpu_backend.py:71-76).
  // Each thread reads and writes only its own words of hx / xs; the per-warp
  // sums of squares meet in shared memory and every thread finishes the
  // mean itself.  Ends with a barrier (xs is read across threads next).
  __device__ void norm_rows(const Gamma &gamma) {
    const int warp = tid >> 5, lane = tid & 31;
    // the rows run side by side (independent chains), each with exactly the
    // arithmetic of a single row, so one row's result does not depend on MB
    float ss[MB];
#pragma unroll
    for (int m = 0; m < MB; ++m) {
      ss[m] = 0.f;
      if (m < mrows) {
#pragma unroll
        for (int j = 0; j < kNormWords; ++j) {
          const int w = norm_word(j);
          if (2 * w < P.H) {
            const uint32_t hw = reinterpret_cast<const uint32_t *>(hx + m * P.H)[w];
            const float a = bf_lo(hw), b = bf_hi(hw);
            ss[m] = fmaf(a, a, ss[m]);
            ss[m] = fmaf(b, b, ss[m]);
          }
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
      for (int m = 0; m < MB; ++m) ss[m] += __shfl_xor_sync(0xffffffffu, ss[m], o);
    }
    if (lane == 0) {
#pragma unroll
      for (int m = 0; m < MB; ++m)
        if (m < mrows) s_norm[warp * kMaxBatch + m] = ss[m];
    }
    consumer_sync(kConsumerThreads);
#pragma unroll
    for (int m = 0; m < MB; ++m) {
      if (m < mrows) {
        float total = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) total += s_norm[w * kMaxBatch + m];
        const float mean = __fdiv_rn(total, static_cast<float>(P.H));
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, P.eps)));
#pragma unroll
        for (int j = 0; j < kNormWords; ++j) {
          const int w = norm_word(j);
          if (2 * w < P.H) {
            const uint32_t hw = reinterpret_cast<const uint32_t *>(hx + m * P.H)[w];
            const float a = __fmul_rn(__fmul_rn(bf_lo(hw), inv), gamma.v[2 * j]);
            const float b = __fmul_rn(__fmul_rn(bf_hi(hw), inv), gamma.v[2 * j + 1]);
            *reinterpret_cast<uint32_t *>(xs + m * P.xs_elems + 2 * w) = pack_bf16x2(a, b);
          }
        }
      }
    }
    consumer_sync(kConsumerThreads);
  }

  __device__ __forceinline__ float red_sum(int m, int local) const {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v += red[(w * MB + m) * P.red_rows + local];
    return v;
  }

  // hx[m][:] = the BF16 vector in the LL words at src (row m at
  // src + m * row_words).
  __device__ bool gather_to_hx(const uint64_t *src, size_t row_words, int nvals) {
    return gather_raw(src, row_words, nvals / 2, reinterpret_cast<uint32_t *>(hx), P.H / 2);
  }

  // Raw payloads of the LL words (BF16 pairs) into dst[m * dst_words + i].
  __device__ bool gather_raw(const uint64_t *src, size_t row_words, int words, uint32_t *dst,
                                          size_t dst_words) {
    return ll_gather<(MB > 1 ? (W8 ? 6 : 8) : 6)>(src, row_words, words, mrows, epoch, &P.result->ctrl, P.limit_ns,
                     [&](int m, int i, uint32_t d) { dst[m * dst_words + i] = d; });
  }

  // ---- phases -------------------------------------------------------------------

  // ---- attention (cpu_backend.py:78-129) ---------------------------------------
  // The attention phase splits its work into (batch row m, q head h) units,
  // one per CTA (unit = cta); each unit publishes its 64 outputs as LL words
  // and every CTA then gathers all heads of all rows for the o-projection.
  __device__ bool has_unit() const { return cta < mrows * P.QH; }

  // First row of the run of rows that continue row m's sequence in this
  // launch (same slot, consecutive positions): batched prefill puts up to
  // kMaxBatch consecutive positions of one slot in one launch.
  __device__ int run_start(int m) const {
    int f = m;
    while (f > 0 && s_slot[f - 1] == s_slot[m] && s_pos[f - 1] == s_pos[f] - 1) --f;
    return f;
  }

  // Start copying the K and V history of row m, kv head j from the cache
  // into kvs with cp.async: positions before the row's run (later ones are
  // computed in this launch and come from the run's q/k/v words).
  __device__ void kv_prefetch_unit(int layer, int m, int j) {
    const int p = s_pos[run_start(m)], slot = s_slot[m];
    const int pieces = p * 8;  // 16-byte pieces per block
    for (int i = tid; i < 2 * pieces; i += kConsumerThreads) {
      const int kind = i >= pieces ? 1 : 0, rem = i - kind * pieces;
      const size_t off = static_cast<size_t>(rem >> 3) * 128 + (rem & 7) * 16;
      cp_async16(kvs + static_cast<size_t>(kind) * P.CTX * 128 + off,
                 reinterpret_cast<const uint8_t *>(kv_block(slot, layer, j, kind)) + off);
    }
    cp_async_commit();
  }

  // Decode (no earlier rows in the run): the 96 q/k/v words of row m, one
  // per thread.
  __device__ bool gather_unit_row(int layer, int m, int h, int j, uint32_t *u96) {
    if (tid >= 96) return true;
    const int seg = tid >> 5, i = tid & 31;
    const int head = seg == 0 ? h : seg == 1 ? P.QH + j : P.QH + P.KVH + j;
    const uint64_t *src = ll_qkv(layer, m) + head * 32 + i;
    uint64_t start = 0;
    for (uint32_t spins = 0;; ++spins) {
      const uint64_t v = ll_load(src);
      if (static_cast<uint32_t>(v >> 32) == epoch) {
        u96[tid] = static_cast<uint32_t>(v);
        return true;
      }
      if (start == 0) start = globaltimer_ns();
      if ((spins & 31u) == 31u && wait_expired(&P.result->ctrl, start, P.limit_ns, kWhereGrid)) return false;
    }
  }

  // The unit's words into u96: q (head h), k and v (kv head j) of row m at
  // [0, 96), then k and v of each earlier row of its run at 96 + 64 * r.
  __device__ bool gather_unit(int layer, int m, int h, int j, uint32_t *u96) {
    const int f = run_start(m);
    if (f == m) return gather_unit_row(layer, m, h, j, u96);
    const int n = 96 + 64 * (m - f);
    constexpr int U = 4;
    const uint64_t *src[U];
    int dst[U];
    uint32_t pend = 0;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = tid + u * kConsumerThreads;
      dst[u] = i < 96 ? i : kUnitWords + (i - 96);
      src[u] = nullptr;
      if (i < n) {
        int row = m, head, w;
        if (i < 96) {
          const int seg = i >> 5;
          head = seg == 0 ? h : seg == 1 ? P.QH + j : P.QH + P.KVH + j;
          w = i & 31;
        } else {
          const int e = i - 96;
          row = f + (e >> 6);
          head = (e & 63) < 32 ? P.QH + j : P.QH + P.KVH + j;
          w = e & 31;
        }
        src[u] = ll_qkv(layer, row) + head * 32 + w;
        pend |= 1u << u;
      }
    }
    uint64_t start = 0;
    for (uint32_t spins = 0; pend; ++spins) {
      uint64_t v[U];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (pend & (1u << u)) v[u] = ll_load(src[u]);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if ((pend & (1u << u)) && static_cast<uint32_t>(v[u] >> 32) == epoch) {
          u96[dst[u]] = static_cast<uint32_t>(v[u]);
          pend &= ~(1u << u);
        }
      }
      if (pend) {
        if (start == 0) start = globaltimer_ns();
        if ((spins & 31u) == 31u && wait_expired(&P.result->ctrl, start, P.limit_ns, kWhereGrid)) return false;
      }
    }
    return true;
  }

  __device__ __forceinline__ void rope_pair(const uint32_t *w32, int pr, int d, __nv_bfloat16 &lo,
                                            __nv_bfloat16 &hi) const {
    rope_pair_cs(w32, d, P.rope_cos[pr * 32 + d], P.rope_sin[pr * 32 + d], lo, hi);
  }

  __device__ __forceinline__ uint32_t attend(const float *qf, float *sc, const uint8_t *kb, const uint8_t *vb,
                                             int p) const {
    return attend_warp(qf, sc, kb, vb, p);
  }

  // One unit: RoPE (rotate-half, unfused mul/add, BF16), K/V append, then
  // attend(); publishes the bf16 outputs to ll_att(layer, m) + h * 32.
  // Called by every consumer thread (one block barrier publishes the
  // cp.async history); warp 0 does the work -- one head is a few thousand
  // FMAs, so block barriers would cost more than the math.
  __device__ void attention_unit(int layer, int m, int h, int j, uint32_t *u96, float rc, float rs) {
    const int p = s_pos[m];
    float *qf = reinterpret_cast<float *>(u96 + 96);
    float *sc = qf + kHeadDim;
    uint8_t *kb = kvs, *vb = kvs + static_cast<size_t>(P.CTX) * 128;
    cp_async_wait_all();
    consumer_sync(kConsumerThreads);  // every thread's history copies (and u96) are visible
    if (tid >= 32) return;
    const int lane = tid;
    {
      __nv_bfloat16 lo, hi;
      rope_pair_cs(u96, lane, rc, rs, lo, hi);  // q
      qf[lane] = bf2f(lo);
      qf[lane + 32] = bf2f(hi);
      rope_pair_cs(u96 + 32, lane, rc, rs, lo, hi);  // k
      put_kv(kb, vb, p, lane, lo, hi, u96[64 + lane]);
      // batched prefill: k and v of the earlier rows of the run
      const int f = run_start(m);
      for (int r = f; r < m; ++r) {
        const uint32_t *w = u96 + kUnitWords + 64 * (r - f);
        rope_pair(w, s_pos[r], lane, lo, hi);
        put_kv(kb, vb, s_pos[r], lane, lo, hi, w[32 + lane]);
      }
    }
    __syncwarp();
    // the first q head of kv group j appends row p of K and V to the cache
    if (h % P.group == 0 && lane < 16) {
      const int kind = lane >> 3, cb = lane & 7;
      const uint8_t *srow = (kind ? vb : kb) + kv_off(p, cb);
      uint8_t *dst = reinterpret_cast<uint8_t *>(kv_block(s_slot[m], layer, j, kind)) + kv_off(p, cb);
      *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(srow);
    }
    ll_store(ll_att(layer, m) + h * 32 + lane, attend(qf, sc, kb, vb, p), epoch);
  }

  // ---- paged attention (contexts longer than 64 positions) ---------------------
  // Splits of each (row, q head) unit's positions: one per kSplitPositions
  // positions of the longest row, at most as many as leave every split its
  // own CTA.  The same value in every CTA (it depends only on the step).
  __device__ int att_splits() const {
    int n = 0;
    for (int m = 0; m < mrows; ++m) n = max(n, s_pos[m] + 1);
    const int want = (n + kSplitPositions - 1) / kSplitPositions;
    const int cap = G / (mrows * P.QH);
    return max(1, min(want, cap));
  }

  // Page holding position s of a slot; -1 (and the launch's error raised)
  // when the table entry lies outside the pool -- the host maps every page
  // a step reads or writes before the launch, so this guards only the
  // bounds of the accesses below.
  __device__ int kv_page(int slot, int s) const {
    const int pg = __ldg(P.page_table + static_cast<size_t>(slot) * P.pages_per_slot + (s >> 6));
    if (static_cast<unsigned>(pg) >= static_cast<unsigned>(P.n_pages)) {
      raise_error(&P.result->ctrl, kErrBadPage, kWhereKvPage);
      return -1;
    }
    return pg;
  }

  // The 64 K (kind 0) or V (kind 1) rows of one (layer, kv head) in page pg.
  __device__ const uint8_t *page_rows(int pg, int layer, int kvh, int kind) const {
    return reinterpret_cast<const uint8_t *>(P.kv) +
           ((((static_cast<size_t>(pg) * P.L + layer) * P.KVH + kvh) * 2 + kind) << 13);
  }

  // One (row m, q head h, split sp of S) unit in paged mode: RoPE of q and
  // of this launch's k rows (kept in shared memory, 128-byte rows in
  // logical block order), the K/V append (split 0 of the group's first q
  // head), then over the split's positions [lo, hi): scores q.k * 0.125,
  // max, exp(score - max), their sum and the unnormalised P.V, all seven
  // warps sharing the positions.  One split publishes o = P.V / sum; with
  // several, each leaves (P.V, max, sum) in att_part and the last to arrive
  // rescales them to the common max and publishes sum(w P.V) / sum(w sum).
  __device__ void attention_paged(int layer, int m, int h, int j, int sp, int S, uint32_t *u96) {
    const int p = s_pos[m], slot = s_slot[m];
    const int f = run_start(m), p0 = s_pos[f];  // positions >= p0 are computed in this launch
    const int n = p + 1;
    int chunk = (n + S - 1) / S;
    chunk = (chunk + 31) & ~31;
    const int lo = min(n, sp * chunk), hi = min(n, lo + chunk);
    float *qf = reinterpret_cast<float *>(u96 + 96);
    float *rmax = qf + kHeadDim;  // [kWarps]
    float *rsum = rmax + 8;       // [kWarps]
    int *flag = reinterpret_cast<int *>(rsum + 8);
    uint8_t *stk = kvs, *stv = kvs + kMaxBatch * 128;
    float *pv = reinterpret_cast<float *>(kvs + 2 * kMaxBatch * 128);  // [kWarps][64]
    float *sc = pv + kWarps * kHeadDim;                               // [hi - lo]
    const int warp = tid >> 5, lane = tid & 31;
    consumer_sync(kConsumerThreads);  // u96 complete
    if (warp == 0) {
      auto rope_pair = [&](const uint32_t *w32, int pr, int d, __nv_bfloat16 &rlo, __nv_bfloat16 &rhi) {
        const uint32_t a = w32[d >> 1], b = w32[(d + 32) >> 1];
        const float x0 = (d & 1) ? bf_hi(a) : bf_lo(a), x1 = (d & 1) ? bf_hi(b) : bf_lo(b);
        const float c = P.rope_cos[pr * 32 + d], sn = P.rope_sin[pr * 32 + d];
        rlo = f2bf(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)));
        rhi = f2bf(__fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, sn)));
      };
      auto put_row = [&](int lr, __nv_bfloat16 klo, __nv_bfloat16 khi, uint32_t vword) {
        reinterpret_cast<__nv_bfloat16 *>(stk + lr * 128)[lane] = klo;
        reinterpret_cast<__nv_bfloat16 *>(stk + lr * 128)[lane + 32] = khi;
        reinterpret_cast<uint32_t *>(stv + lr * 128)[lane] = vword;
      };
      __nv_bfloat16 rlo, rhi;
      rope_pair(u96, p, lane, rlo, rhi);  // q
      qf[lane] = bf2f(rlo);
      qf[lane + 32] = bf2f(rhi);
      rope_pair(u96 + 32, p, lane, rlo, rhi);  // k of row m
      put_row(m - f, rlo, rhi, u96[64 + lane]);
      for (int r = f; r < m; ++r) {  // batched prefill: the run's earlier rows
        const uint32_t *w = u96 + kUnitWords + 64 * (r - f);
        rope_pair(w, s_pos[r], lane, rlo, rhi);
        put_row(r - f, rlo, rhi, w[32 + lane]);
      }
      __syncwarp();
      if (sp == 0 && h % P.group == 0 && lane < 16) {
        const int kind = lane >> 3, cb = lane & 7;
        const int pg = kv_page(slot, p);
        if (pg >= 0) {
          const uint8_t *src = (kind ? stv : stk) + (m - f) * 128 + cb * 16;
          uint8_t *dst = const_cast<uint8_t *>(page_rows(pg, layer, j, kind)) + kv_off(p & 63, cb);
          *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(src);
        }
      }
    }
    consumer_sync(kConsumerThreads);  // qf and the launch's rows visible
    // scores: thread per position, two rows in flight (one in the 8-row
    // kernels, whose GEMV leaves fewer registers)
    constexpr int kRowsInFlight = MB == 1 ? 2 : 1;
    float tmax = -INFINITY;
    for (int s0 = lo + tid; s0 < hi; s0 += kRowsInFlight * kConsumerThreads) {
      uint4 kw[kRowsInFlight][8];
#pragma unroll
      for (int e = 0; e < kRowsInFlight; ++e) {
        const int s = s0 + e * kConsumerThreads;
        if (s < hi && s < p0) {
          const int pg = kv_page(slot, s);
          const uint8_t *row = pg >= 0 ? page_rows(pg, layer, j, 0) + (s & 63) * 128 : nullptr;
#pragma unroll
          for (int cb = 0; cb < 8; ++cb)
            kw[e][cb] = row ? __ldcg(reinterpret_cast<const uint4 *>(row + ((cb ^ (s & 7)) << 4)))
                            : make_uint4(0u, 0u, 0u, 0u);
        } else if (s < hi) {
#pragma unroll
          for (int cb = 0; cb < 8; ++cb) kw[e][cb] = reinterpret_cast<const uint4 *>(stk + (s - p0) * 128)[cb];
        }
      }
#pragma unroll
      for (int e = 0; e < kRowsInFlight; ++e) {
        const int s = s0 + e * kConsumerThreads;
        if (s < hi) {
          float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int cb = 0; cb < 8; ++cb) {
            const uint4 k = kw[e][cb];
            const float *q = qf + 8 * cb;
            float &a = acc[cb & 3];
            a = fmaf(bf_lo(k.x), q[0], a);
            a = fmaf(bf_hi(k.x), q[1], a);
            a = fmaf(bf_lo(k.y), q[2], a);
            a = fmaf(bf_hi(k.y), q[3], a);
            a = fmaf(bf_lo(k.z), q[4], a);
            a = fmaf(bf_hi(k.z), q[5], a);
            a = fmaf(bf_lo(k.w), q[6], a);
            a = fmaf(bf_hi(k.w), q[7], a);
          }
          const float score = ((acc[0] + acc[1]) + (acc[2] + acc[3])) * 0.125f;
          sc[s - lo] = score;
          tmax = fmaxf(tmax, score);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
    if (lane == 0) rmax[warp] = tmax;
    consumer_sync(kConsumerThreads);
    float mx = rmax[0];
    for (int w = 1; w < kWarps; ++w) mx = fmaxf(mx, rmax[w]);
    float tsum = 0.f;
    for (int s = lo + tid; s < hi; s += kConsumerThreads) {
      const float e = expf(__fsub_rn(sc[s - lo], mx));
      sc[s - lo] = e;
      tsum += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tsum += __shfl_xor_sync(0xffffffffu, tsum, o);
    if (lane == 0) rsum[warp] = tsum;
    consumer_sync(kConsumerThreads);  // sc (weights) and rsum visible
    float sum = 0.f;
    for (int w = 0; w < kWarps; ++w) sum += rsum[w];
    // P.V: a quarter warp per position (lane: 8 dims of block cb), two
    // positions per lane in flight
    const int q4 = lane >> 3, cb = lane & 7;
    float o8[8];
#pragma unroll
    for (int d = 0; d < 8; ++d) o8[d] = 0.f;
    constexpr int kStride = kWarps * 4;
    for (int s0 = lo + warp * 4 + q4; s0 < hi; s0 += 2 * kStride) {
      uint4 vw[2];
      float wt[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int s = s0 + e * kStride;
        vw[e] = make_uint4(0u, 0u, 0u, 0u);
        wt[e] = 0.f;
        if (s < hi) {
          wt[e] = sc[s - lo];
          if (s < p0) {
            const int pg = kv_page(slot, s);
            if (pg >= 0)
              vw[e] = __ldcg(reinterpret_cast<const uint4 *>(page_rows(pg, layer, j, 1) + (s & 63) * 128 +
                                                             ((cb ^ (s & 7)) << 4)));
          } else {
            vw[e] = reinterpret_cast<const uint4 *>(stv + (s - p0) * 128)[cb];
          }
        }
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        o8[0] = fmaf(wt[e], bf_lo(vw[e].x), o8[0]);
        o8[1] = fmaf(wt[e], bf_hi(vw[e].x), o8[1]);
        o8[2] = fmaf(wt[e], bf_lo(vw[e].y), o8[2]);
        o8[3] = fmaf(wt[e], bf_hi(vw[e].y), o8[3]);
        o8[4] = fmaf(wt[e], bf_lo(vw[e].z), o8[4]);
        o8[5] = fmaf(wt[e], bf_hi(vw[e].z), o8[5]);
        o8[6] = fmaf(wt[e], bf_lo(vw[e].w), o8[6]);
        o8[7] = fmaf(wt[e], bf_hi(vw[e].w), o8[7]);
      }
    }
#pragma unroll
    for (int d = 0; d < 8; ++d) {
      o8[d] += __shfl_xor_sync(0xffffffffu, o8[d], 8);
      o8[d] += __shfl_xor_sync(0xffffffffu, o8[d], 16);
    }
    if (q4 == 0) {
#pragma unroll
      for (int d = 0; d < 8; ++d) pv[warp * kHeadDim + cb * 8 + d] = o8[d];
    }
    consumer_sync(kConsumerThreads);
    uint64_t *out = ll_att(layer, m) + h * 32;
    if (S == 1) {
      if (tid < 32) {
        float a = 0.f, b = 0.f;
        for (int w = 0; w < kWarps; ++w) {
          a += pv[w * kHeadDim + 2 * tid];
          b += pv[w * kHeadDim + 2 * tid + 1];
        }
        ll_store(out + tid, pack_bf16x2(__fdiv_rn(a, sum), __fdiv_rn(b, sum)), epoch);
      }
      return;
    }
    float *part = P.att_part + static_cast<size_t>(cta) * kPartStride;
    if (tid < kHeadDim) {
      float a = 0.f;
      for (int w = 0; w < kWarps; ++w) a += pv[w * kHeadDim + tid];
      part[tid] = a;
    } else if (tid == kHeadDim) {
      part[kHeadDim] = mx;
      part[kHeadDim + 1] = sum;
    }
    consumer_sync(kConsumerThreads);
    int *cnt = P.att_cnt + m * P.QH + h;
    if (tid == 0) {
      __threadfence();
      *flag = atomicAdd(cnt, 1) == S - 1 ? 1 : 0;
    }
    consumer_sync(kConsumerThreads);
    if (*flag == 0) return;
    // last split: every other split's partial is visible after the fence
    if (tid == 0) atomicExch(cnt, 0);
    __threadfence();
    if (tid < 32) {
      const float *base = P.att_part + static_cast<size_t>(cta - sp) * kPartStride;
      float M = -INFINITY;
      for (int q = 0; q < S; ++q) M = fmaxf(M, __ldcg(base + q * kPartStride + kHeadDim));
      float den = 0.f, a = 0.f, b = 0.f;
      for (int q = 0; q < S; ++q) {
        const float *pq = base + q * kPartStride;
        const float w = expf(__fsub_rn(__ldcg(pq + kHeadDim), M));
        den = fmaf(w, __ldcg(pq + kHeadDim + 1), den);
        a = fmaf(w, __ldcg(pq + 2 * tid), a);
        b = fmaf(w, __ldcg(pq + 2 * tid + 1), b);
      }
      ll_store(out + tid, pack_bf16x2(__fdiv_rn(a, den), __fdiv_rn(b, den)), epoch);
    }
  }

  // One phase of a layer (kind = k & 3: 0 qkv, 1 attention + o_proj,
  // 2 gate_up + SwiGLU, 3 down).  A prologue leaves the GEMV's BF16 input in
  // xs, then the GEMV over this CTA's rows -- a single call site for every
  // kind, so the hot loop's code stays resident in the instruction cache --
  // then a short epilogue publishes the results as LL words.
  __device__ bool layer_phase(int k) {
    const int layer = k >> 2, kind = k & 3;
    const LayerPtrs &lp = P.layers[layer];
    const MatRange r = phase_range(k);
    const int npairs = (r.g1 - r.g0) * 4;
    // constants of this thread's first epilogue word, fetched before the wait
    const float *bias_p = (kind == 0 && P.has_bias) ? lp.bias : nullptr;
    const float *scale_p = !W8 ? nullptr : kind == 0 ? lp.s_qkv : kind == 1 ? lp.s_o : kind == 3 ? lp.s_down : nullptr;
    const float2 bias0 = load_pair(bias_p, r.g0 * 8, npairs);
    const float2 scale0 = load_pair(scale_p, r.g0 * 8, npairs);
    Gamma gamma;
    if (kind == 0 || kind == 2) gamma = load_gamma(kind == 0 ? lp.gamma_in : lp.gamma_post);
    // attention unit of this CTA: (row um, q head uh, kv head uj), and in
    // paged mode split us of S
    int S = 1, us = 0, ucta = cta;
    if constexpr (PG) {
      if (kind == 1) {
        S = att_splits();
        ucta = cta / S;
        us = cta - ucta * S;
      }
    }
    const int um = ucta / P.QH, uh = ucta - um * P.QH, uj = uh / P.group;
    uint32_t *u96 = reinterpret_cast<uint32_t *>(att);
    bool ok = true;
    if (kind == 1) {
      // this CTA's attention unit publishes its head's outputs first
      if constexpr (PG) {
        if (ucta < mrows * P.QH) ok = gather_unit(layer, um, uh, uj, u96);
        if (!ok) return false;
        if (ucta < mrows * P.QH) attention_paged(layer, um, uh, uj, us, S, u96);
      } else if (has_unit()) {
        // this row's RoPE cos / sin (dim = lane) and the K/V history are
        // fetched while the q/k/v words are awaited
        const int lane = tid & 31;
        const float rc = P.rope_cos[s_pos[um] * 32 + lane], rs = P.rope_sin[s_pos[um] * 32 + lane];
        kv_prefetch_unit(layer, um, uj);
        ok = gather_unit(layer, um, uh, uj, u96);
        if (!ok) {
          cp_async_wait_all();
          return false;
        }
        attention_unit(layer, um, uh, uj, u96, rc, rs);
      }
    }
    // the GEMV input: the previous phase's LL words, through one gather site
    // for every kind (its code is fetched once per layer, not four times)
    const bool to_hx = kind == 0 || kind == 2;
    const uint64_t *gsrc = kind == 0 ? ll_hout(layer - 1, 0) : kind == 1 ? ll_att(layer, 0)
                         : kind == 2 ? ll_h1(layer, 0) : ll_act(layer, 0);
    const int gwords = kind == 3 ? P.I / 2 : P.H / 2;
    if (kind == 0 && layer == 0) {
      // the embedding row (generate.py:758-768), same word-pair ownership
      // as the gather (the norm reads these words next without a barrier)
      for (int m = 0; m < mrows; ++m) {
        const uint2 *e = reinterpret_cast<const uint2 *>(P.embed + static_cast<size_t>(s_tok[m]) * P.H);
        for (int w = tid; w < P.H / 4; w += kConsumerThreads) {
          reinterpret_cast<uint2 *>(hx + m * P.H)[w] = __ldg(e + w);
        }
      }
    } else {
      ok = gather_raw(gsrc, gwords, gwords, reinterpret_cast<uint32_t *>(to_hx ? hx : xs),
                      to_hx ? P.H / 2 : P.xs_elems / 2);
    }
    if (!ok) return false;
    mark(k, 1);
    if (to_hx) {
      norm_rows(gamma);  // each thread starts on its own words; the norm synchronizes
    } else {
      consumer_sync(kConsumerThreads);  // xs is read across threads next
    }
    mark(k, 6);
    if (!consume_splitk<MB, W8>(ring, r, xs, P.xs_elems, mrows, red, P.red_rows, &P.result->ctrl, P.limit_ns))
      return false;
    consumer_sync(kConsumerThreads);
    mark(k, 2);
    if (kind == 2) {
      // SwiGLU (cpu_backend.py:154-165): g / (1 + exp(-clip(g, -80, 80))) * u
      const int b0 = r.g0 / 2, nblk = (r.g1 - r.g0) / 2;
      const int per_row = nblk * 4;  // LL words (pairs of intermediate indices)
      for (int idx = tid; idx < mrows * per_row; idx += kConsumerThreads) {
        const int m = idx / per_row;
        const int rem = idx - m * per_row;
        const int blk = rem >> 2, rr = (rem & 3) * 2;
        float a[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float g = red_sum(m, blk * 16 + rr + e);
          float u = red_sum(m, blk * 16 + 8 + rr + e);
          if (W8) {
            g *= lp.s_gu[(2 * (b0 + blk)) * 8 + rr + e];
            u *= lp.s_gu[(2 * (b0 + blk) + 1) * 8 + rr + e];
          }
          g = rbf(g);
          u = rbf(u);
          const float ex = expf(-fminf(fmaxf(g, -80.f), 80.f));
          a[e] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, ex)), u);
        }
        ll_store(ll_act(layer, m) + ((b0 + blk) * 8 + rr) / 2, pack_bf16x2(a[0], a[1]), epoch);
      }
      return true;
    }
    // qkv: bf16(bf16(Wx) + bias); o_proj / down: bf16(bf16(Wx) + residual)
    for (int idx = tid; idx < mrows * npairs; idx += kConsumerThreads) {
      const int m = idx / npairs, lp2 = idx - m * npairs;
      const int row = r.g0 * 8 + 2 * lp2;
      const bool mine = lp2 == tid;
      float y[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float v = red_sum(m, 2 * lp2 + e);
        if (W8) v *= mine ? (e ? scale0.y : scale0.x) : scale_p[row + e];
        y[e] = rbf(v);
        if (kind == 0) {
          if (bias_p != nullptr) y[e] = __fadd_rn(y[e], mine ? (e ? bias0.y : bias0.x) : bias_p[row + e]);
        } else {
          y[e] = __fadd_rn(y[e], bf2f(hx[m * P.H + row + e]));
        }
      }
      uint64_t *dst = kind == 0 ? ll_qkv(layer, m) : kind == 1 ? ll_h1(layer, m) : ll_hout(layer, m);
      ll_store(dst + row / 2, pack_bf16x2(y[0], y[1]), epoch);
    }
    return true;
  }

  __device__ bool phase_head() {
    const int warp = tid >> 5, lane = tid & 31;
    const Gamma gamma = load_gamma(P.gamma_final);
    if (!gather_to_hx(ll_hout(P.L - 1, 0), P.H / 2, P.H)) return false;
    mark(4 * P.L, 1);
    norm_rows(gamma);
    mark(4 * P.L, 6);
    float bv[MB];
    int bi[MB];
#pragma unroll
    for (int m = 0; m < MB; ++m) {
      bv[m] = -INFINITY;
      bi[m] = 0x7fffffff;
    }
    const MatRange r = phase_range(4 * P.L);
    float *logits = P.logits;
    const float *s_lm = P.s_lm;
    const int V = P.V;
    const bool write = P.write_logits != 0;
    const bool ok = consume_chunk_per_warp<MB, W8>(
        ring, r, xs, P.xs_elems, mrows, &P.result->ctrl, P.limit_ns, [&](int m, int row, float v) {
          if (W8) v *= s_lm[row];
          if (write) logits[static_cast<size_t>(m) * V + row] = v;
          if (argmax_better(v, row, bv[m], bi[m])) {
            bv[m] = v;
            bi[m] = row;
          }
        });
    mark(4 * P.L, 2);
#pragma unroll
    for (int m = 0; m < MB; ++m) {
      float v = bv[m];
      int i = bi[m];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, i, o);
        argmax_merge(v, i, ov, oi);
      }
      if (lane == 0) {
        s_bestv[warp * kMaxBatch + m] = v;
        s_besti[warp * kMaxBatch + m] = i;
      }
    }
    consumer_sync(kConsumerThreads);
    if (tid < mrows) {
      float v = -INFINITY;
      int i = 0x7fffffff;
      for (int w = 0; w < kWarps; ++w)
        argmax_merge(v, i, s_bestv[w * kMaxBatch + tid], s_besti[w * kMaxBatch + tid]);
      P.part_val[cta * kMaxBatch + tid] = v;
      P.part_idx[cta * kMaxBatch + tid] = i;
    }
    return ok;
  }

  // ---- consumer main ----------------------------------------------------------
  __device__ void run_consumers() {
    Ctrl *ctrl = &P.result->ctrl;
    if (tid < kMaxBatch) {
      const StepState *st = P.st;
      s_tok[tid] = __ldcg(&st->token[tid]);
      s_pos[tid] = __ldcg(&st->pos[tid]);
      s_slot[tid] = __ldcg(&st->slot[tid]);
    }
    if (tid == 0) {
      s_misc[0] = __ldcg(&P.st->rows);
      s_misc[2] = static_cast<int>(__ldcg(P.epoch));
    }
    consumer_sync(kConsumerThreads);
    mrows = min(s_misc[0], MB);
    epoch = static_cast<uint32_t>(s_misc[2]);
    if (P.stall_ns != 0 && tid == 0) stall_on_unset_flag(ctrl, P.stall_ns);
    consumer_sync(kConsumerThreads);
    bool ok = ld_volatile_int(&ctrl->abort) == 0;
    const int nph = 4 * P.L + 2;
    (void)nph;
    bool ran_head = false;
    for (int k = P.phase_begin; k < P.phase_end && ok; ++k) {
      mark(k, 0);
      if (k >= 4 * P.L) {
        ok = phase_head();
        ran_head = true;
      } else {
        ok = layer_phase(k);
      }
      consumer_sync(kConsumerThreads);
      mark(k, 3);
    }
    mark(nph - 1, 0);
    // exit protocol: the last CTA finishes the argmax and advances the state
    consumer_sync(kConsumerThreads);
    if (tid == 0) {
      __threadfence();
      const unsigned int prev = atomicAdd(&ctrl->done, 1u);
      s_misc[1] = (prev == static_cast<unsigned int>(G) - 1u) ? 1 : 0;
    }
    consumer_sync(kConsumerThreads);
    if (s_misc[1]) {
      __threadfence();
      const int warp = tid >> 5, lane = tid & 31;
      if (ran_head && warp == 0 && ld_volatile_int(&ctrl->abort) == 0) {
        for (int m = 0; m < mrows; ++m) {
          float v = -INFINITY;
          int i = 0x7fffffff;
          for (int c = lane; c < G; c += 32)
            argmax_merge(v, i, __ldcg(P.part_val + c * kMaxBatch + m), __ldcg(P.part_idx + c * kMaxBatch + m));
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, i, o);
            argmax_merge(v, i, ov, oi);
          }
          if (lane == 0) P.result->out_token[m] = i;
        }
      }
      consumer_sync(kConsumerThreads);
      if (tid == 0) {
        StepState *st = P.st;
        if (st->chained && ld_volatile_int(&ctrl->abort) == 0) {
          const int p = st->pos[0];
          int next = (p + 1 < st->n_prompt) ? P.prompt[p + 1] : -1;
          const int tok = ran_head ? P.result->out_token[0] : 0;
          if (tok < 0 || tok >= P.V) {
            // the next launch would read this row of the embedding: stop the
            // chain instead (unreachable while the argmax offers every row)
            raise_error(ctrl, kErrBadToken, kWhereToken);
          } else {
            if (ran_head) {
              P.gen_out[st->n_out] = tok;
              st->n_out = st->n_out + 1;
              if (next < 0) next = tok;
            }
            st->token[0] = next < 0 ? 0 : next;
            st->pos[0] = p + 1;
          }
        }
        unsigned int ne = *P.epoch + 1u;
        if (ne == 0u) ne = 1u;
        *P.epoch = ne;
        atomicExch(&ctrl->done, 0u);
        __threadfence();
      }
    }
  }

  // ---- producer main ----------------------------------------------------------
  // The chunk sequence of a launch: per phase, the K/V history of every row
  // (attention phases), then the phase's weight row groups.
  __device__ void run_producer() {
    Producer prod{&ring, RingPos{0, 0}, 0, &P.result->ctrl, P.limit_ns, policy_evict_first()};
    bool ok = true;
    for (int k = P.phase_begin; k < P.phase_end && ok; ++k) {
      if (P.trace) P.trace[(static_cast<size_t>(cta) * (4 * P.L + 2) + k) * 8 + 5] = globaltimer_ns();
      if (ok) ok = prod.issue_range(phase_range(k));
    }
    prod.drain();
  }
};

template <int MB, bool W8, bool PG>
__global__ void __launch_bounds__(kThreads, 1) decoder_kernel(const __grid_constant__ DecParams P) {
  extern __shared__ __align__(1024) uint8_t smem[];
  DecoderCta<MB, W8, PG> cx(P, smem);
  if (threadIdx.x == 0) {
    for (int i = 0; i < P.nslots; ++i) {
      mbar_init(&cx.ring.full[i], 1);
      mbar_init(&cx.ring.empty[i], kWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x >= kConsumerThreads) {
    if (threadIdx.x == kConsumerThreads) cx.run_producer();
    return;
  }
  cx.run_consumers();
}

}  // namespace hb
