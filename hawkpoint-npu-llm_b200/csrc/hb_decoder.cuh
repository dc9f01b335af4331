// hb_decoder.cuh -- the persistent decode kernel.
//
// One cooperative launch runs a range of "phases" of one decode step for up
// to MB batch rows.  For each layer l there are four phases, separated by a
// bounded grid barrier:
//   A (4l+0)  x = rmsnorm(h) ; qkv = bf16(bf16(Wqkv x) + bias)      (cpu_backend.py:131-143)
//   B (4l+1)  rotate q,k (RoPE) ; append k,v to the KV cache ; GQA attention
//             of one head per CTA ; that head's slice of o_proj -> FP32 partials
//                                                                    (cpu_backend.py:78-129)
//   C (4l+2)  h1 = bf16(bf16(sum of o partials) + h) ; x2 = rmsnorm(h1) ;
//             act = bf16(silu(bf16 gate) * bf16 up)                  (cpu_backend.py:145-165)
//   D (4l+3)  h = bf16(bf16(Wdown act) + h1)                          (cpu_backend.py:166-171)
// and after the last layer
//   E (4L)    logits = W_lm rmsnorm(h) (FP32) ; argmax (first maximum)
//                                                     (cpu_backend.py:173-181, generate.py:709-714)
// A producer warp streams every weight chunk of the launch through the
// shared-memory ring (hb_stream.cuh) without waiting on the barriers.
#pragma once

#include "hb_stream.cuh"

namespace hb {

constexpr int kMaxBatch = 8;
constexpr int kHeadDim = 64;

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

// Inputs of a step, in device memory.  In chained mode (device-resident greedy
// generation) the last CTA to finish advances row 0: next position, next token
// (the prompt's, or this step's argmax).
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
  int kc_h, kc_i, kc_d;   // 16-byte chunk columns of K = hidden, intermediate, head_dim
  int slab_bytes;         // bytes of one head's o_proj slab
  const LayerPtrs *layers;
  const float *gamma_final;
  const uint8_t *w_lm;
  const float *s_lm;
  const __nv_bfloat16 *embed;
  const float *rope_cos, *rope_sin;  // [CTX][32]
  __nv_bfloat16 *kv;                 // [slots][L][KVH][2][CTX][64]
  __nv_bfloat16 *hbuf;               // [MB][H]
  __nv_bfloat16 *qkv;                // [MB][QKV]
  float *opart;                      // [MB][QH][H]
  __nv_bfloat16 *act;                // [MB][I]
  float *logits;                     // [MB][V]
  float *part_val;                   // [G][MB]
  int *part_idx;                     // [G][MB]
  Result *result;
  StepState *st;
  const int *prompt;                 // chained: token of each prompt position
  int *gen_out;                      // chained: generated tokens
  int phase_begin, phase_end;
  int write_logits;
  int red_rows;
  int nslots;
  int xs_elems;                      // BF16 elements per batch row of xs
  uint64_t limit_ns;
  uint64_t stall_ns;
  unsigned long long *trace;         // optional [G][4L+2] phase timestamps
};

// Shared-memory carve-up (offsets from the dynamic smem base).
struct SmemPlan {
  size_t ring, full, empty, xs, hx, red, att, misc, total;
};

__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

__host__ __device__ inline SmemPlan smem_plan(int nslots, int mb, int xs_elems, int H, int red_rows,
                                              int ctx) {
  SmemPlan s;
  size_t o = 0;
  s.ring = o;
  o += static_cast<size_t>(nslots) * kSlotBytes;
  s.full = o;
  o += 8 * nslots;
  s.empty = o;
  o += 8 * nslots;
  o = align_up(o, 128);
  s.xs = o;
  o += align_up(static_cast<size_t>(mb) * xs_elems * 2, 128);
  s.hx = o;
  o += align_up(static_cast<size_t>(mb) * H * 4, 128);
  s.red = o;
  o += align_up(static_cast<size_t>(kWarps) * mb * red_rows * 4, 128);
  s.att = o;
  o += align_up((3 * kHeadDim + ctx + kWarps * kHeadDim) * 4, 128);
  s.misc = o;
  o += 1024;
  s.total = o;
  return s;
}

template <int MB, bool W8>
struct DecoderCta {
  const DecParams &P;
  Ring ring;
  __nv_bfloat16 *xs;
  float *hx, *red, *att;
  int *s_tok, *s_pos, *s_slot, *s_flag, *s_last;
  float *s_norm;      // [kWarps * MB] partial sums, then [MB] inverse rms
  float *s_bestv;     // [kWarps * MB]
  int *s_besti;
  int cta, G, mrows, tid;

  __device__ DecoderCta(const DecParams &p, uint8_t *smem) : P(p) {
    const SmemPlan sp = smem_plan(P.nslots, MB, P.xs_elems, P.H, P.red_rows, P.CTX);
    ring.slots = smem + sp.ring;
    ring.full = reinterpret_cast<uint64_t *>(smem + sp.full);
    ring.empty = reinterpret_cast<uint64_t *>(smem + sp.empty);
    ring.nslots = P.nslots;
    ring.counter = 0;
    xs = reinterpret_cast<__nv_bfloat16 *>(smem + sp.xs);
    hx = reinterpret_cast<float *>(smem + sp.hx);
    red = reinterpret_cast<float *>(smem + sp.red);
    att = reinterpret_cast<float *>(smem + sp.att);
    int *mi = reinterpret_cast<int *>(smem + sp.misc);
    s_tok = mi;
    s_pos = mi + kMaxBatch;
    s_slot = mi + 2 * kMaxBatch;
    s_flag = mi + 3 * kMaxBatch;
    s_last = mi + 3 * kMaxBatch + 1;
    s_norm = reinterpret_cast<float *>(mi + 4 * kMaxBatch);          // kWarps*MB + MB floats
    s_bestv = s_norm + kWarps * kMaxBatch + kMaxBatch;
    s_besti = reinterpret_cast<int *>(s_bestv + kWarps * kMaxBatch);
    cta = blockIdx.x;
    G = gridDim.x;
    tid = threadIdx.x;
    mrows = 0;
  }

  // ---- work split ------------------------------------------------------------
  __device__ int head_of(int c) const { return (c * P.QH) / G; }
  __device__ int first_cta_of_head(int h) const { return (h * G + P.QH - 1) / P.QH; }

  __device__ MatRange phase_range(int k) const {
    MatRange r{nullptr, 0, 0, 0};
    if (k >= 4 * P.L) {
      const int n = P.V / 8;
      r = MatRange{P.w_lm, split_lo(n, G, cta), split_lo(n, G, cta + 1), P.kc_h};
      return r;
    }
    const LayerPtrs &lp = P.layers[k >> 2];
    switch (k & 3) {
      case 0: {
        const int n = P.QKV / 8;
        r = MatRange{lp.w_qkv, split_lo(n, G, cta), split_lo(n, G, cta + 1), P.kc_h};
        break;
      }
      case 1: {
        const int h = head_of(cta);
        const int c0 = first_cta_of_head(h), c1 = first_cta_of_head(h + 1);
        const int n = P.H / 8;
        r = MatRange{lp.w_o + static_cast<size_t>(h) * P.slab_bytes, split_lo(n, c1 - c0, cta - c0),
                     split_lo(n, c1 - c0, cta - c0 + 1), P.kc_d};
        break;
      }
      case 2: {
        const int n = P.I / 8;  // gate/up pair blocks
        r = MatRange{lp.w_gu, 2 * split_lo(n, G, cta), 2 * split_lo(n, G, cta + 1), P.kc_h};
        break;
      }
      default: {
        const int n = P.H / 8;
        r = MatRange{lp.w_down, split_lo(n, G, cta), split_lo(n, G, cta + 1), P.kc_i};
        break;
      }
    }
    return r;
  }

  // ---- helpers ----------------------------------------------------------------
  __device__ __forceinline__ float h_in(int layer, int m, int i) const {
    if (layer == 0) return bf2f(P.embed[static_cast<size_t>(s_tok[m]) * P.H + i]);
    return bf2f(__ldcg(P.hbuf + static_cast<size_t>(m) * P.H + i));
  }

  // h1 = bf16(bf16(sum_h o_partial_h [* s_o]) + h_in): identical wherever used.
  __device__ __forceinline__ float h1_value(const LayerPtrs &lp, int layer, int m, int i) const {
    float o = 0.f;
    const float *op = P.opart + static_cast<size_t>(m) * P.QH * P.H + i;
    for (int h = 0; h < P.QH; ++h) o += __ldcg(op + static_cast<size_t>(h) * P.H);
    if (W8) o *= lp.s_o[i];
    return rbf(__fadd_rn(rbf(o), h_in(layer, m, i)));
  }

  // xs[m][i] = bf16((v * inv_rms) * gamma) for v = hx[m][:]  (cpu_backend.py:71-76)
  __device__ void norm_rows(const float *gamma) {
    const int warp = tid >> 5, lane = tid & 31;
    for (int m = 0; m < mrows; ++m) {
      float s = 0.f;
      for (int i = tid; i < P.H; i += kConsumerThreads) {
        const float v = hx[m * P.H + i];
        s = fmaf(v, v, s);
      }
      s = warp_sum(s);
      if (lane == 0) s_norm[warp * kMaxBatch + m] = s;
    }
    consumer_sync(kConsumerThreads);
    if (tid < mrows) {
      float total = 0.f;
      for (int w = 0; w < kWarps; ++w) total += s_norm[w * kMaxBatch + tid];
      const float mean = __fdiv_rn(total, static_cast<float>(P.H));
      s_norm[kWarps * kMaxBatch + tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, P.eps)));
    }
    consumer_sync(kConsumerThreads);
    for (int idx = tid; idx < mrows * P.H; idx += kConsumerThreads) {
      const int m = idx / P.H, i = idx - m * P.H;
      const float inv = s_norm[kWarps * kMaxBatch + m];
      xs[m * P.xs_elems + i] = f2bf(__fmul_rn(__fmul_rn(hx[idx], inv), gamma[i]));
    }
    consumer_sync(kConsumerThreads);
  }

  __device__ __forceinline__ float red_sum(int m, int local) const {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v += red[(w * MB + m) * P.red_rows + local];
    return v;
  }

  // ---- phases -----------------------------------------------------------------
  __device__ bool phase_a(int layer) {
    const LayerPtrs &lp = P.layers[layer];
    for (int idx = tid; idx < mrows * P.H; idx += kConsumerThreads) {
      const int m = idx / P.H, i = idx - m * P.H;
      hx[idx] = h_in(layer, m, i);
    }
    consumer_sync(kConsumerThreads);
    norm_rows(lp.gamma_in);
    const MatRange r = phase_range(4 * layer);
    if (!consume_splitk<MB, W8>(ring, r, xs, P.xs_elems, mrows, red, P.red_rows, &P.result->ctrl,
                                P.limit_ns))
      return false;
    consumer_sync(kConsumerThreads);
    const int nrows = (r.g1 - r.g0) * 8;
    for (int idx = tid; idx < mrows * nrows; idx += kConsumerThreads) {
      const int m = idx / nrows, lr = idx - m * nrows;
      const int row = r.g0 * 8 + lr;
      float v = red_sum(m, lr);
      if (W8) v *= lp.s_qkv[row];
      float y = rbf(v);
      if (P.has_bias) y = rbf(__fadd_rn(y, lp.bias[row]));
      P.qkv[static_cast<size_t>(m) * P.QKV + row] = f2bf(y);
    }
    return true;
  }

  __device__ bool phase_b(int layer) {
    const LayerPtrs &lp = P.layers[layer];
    const int warp = tid >> 5, lane = tid & 31;
    const int head = head_of(cta);
    const int kvh = head / P.group;
    const bool writer = (cta == first_cta_of_head(kvh * P.group));
    float *aq = att, *ak = att + kHeadDim, *av = att + 2 * kHeadDim;
    float *sc = att + 3 * kHeadDim;
    float *pv = sc + P.CTX;
    for (int m = 0; m < mrows; ++m) {
      const int p = s_pos[m];
      __nv_bfloat16 *kcache = P.kv + ((static_cast<size_t>(s_slot[m]) * P.L + layer) * P.KVH + kvh) *
                                         2 * P.CTX * kHeadDim;
      __nv_bfloat16 *vcache = kcache + static_cast<size_t>(P.CTX) * kHeadDim;
      const __nv_bfloat16 *row = P.qkv + static_cast<size_t>(m) * P.QKV;
      if (tid < 32) {
        const int d = tid;
        const float c = P.rope_cos[p * 32 + d], s = P.rope_sin[p * 32 + d];
        // rotate-half (cpu_backend.py:78-93), multiplies and adds unfused
        const float q0 = bf2f(__ldcg(row + head * kHeadDim + d));
        const float q1 = bf2f(__ldcg(row + head * kHeadDim + d + 32));
        aq[d] = rbf(__fsub_rn(__fmul_rn(q0, c), __fmul_rn(q1, s)));
        aq[d + 32] = rbf(__fadd_rn(__fmul_rn(q1, c), __fmul_rn(q0, s)));
        const int kb = P.QH * kHeadDim + kvh * kHeadDim;
        const float k0 = bf2f(__ldcg(row + kb + d)), k1 = bf2f(__ldcg(row + kb + d + 32));
        const float ka = rbf(__fsub_rn(__fmul_rn(k0, c), __fmul_rn(k1, s)));
        const float kz = rbf(__fadd_rn(__fmul_rn(k1, c), __fmul_rn(k0, s)));
        ak[d] = ka;
        ak[d + 32] = kz;
        const int vb = (P.QH + P.KVH) * kHeadDim + kvh * kHeadDim;
        const __nv_bfloat16 v0 = __ldcg(row + vb + d), v1 = __ldcg(row + vb + d + 32);
        av[d] = bf2f(v0);
        av[d + 32] = bf2f(v1);
        if (writer) {
          kcache[p * kHeadDim + d] = f2bf(ka);
          kcache[p * kHeadDim + d + 32] = f2bf(kz);
          vcache[p * kHeadDim + d] = v0;
          vcache[p * kHeadDim + d + 32] = v1;
        }
      }
      consumer_sync(kConsumerThreads);
      // scores: warp per position, lane per pair of dims
      for (int s = warp; s <= p; s += kWarps) {
        float k0, k1;
        if (s == p) {
          k0 = ak[2 * lane];
          k1 = ak[2 * lane + 1];
        } else {
          const uint32_t kk = __ldcg(reinterpret_cast<const unsigned int *>(kcache + s * kHeadDim) + lane);
          k0 = bf_lo(kk);
          k1 = bf_hi(kk);
        }
        float part = aq[2 * lane] * k0;
        part = fmaf(aq[2 * lane + 1], k1, part);
        part = warp_sum(part);
        if (lane == 0) sc[s] = part * 0.125f;
      }
      consumer_sync(kConsumerThreads);
      if (warp == 0) {
        float mx = -INFINITY;
        for (int s = lane; s <= p; s += 32) mx = fmaxf(mx, sc[s]);
        mx = warp_max(mx);
        float sum = 0.f;
        for (int s = lane; s <= p; s += 32) {
          const float e = expf(__fsub_rn(sc[s], mx));
          sc[s] = e;
          sum += e;
        }
        sum = warp_sum(sum);
        for (int s = lane; s <= p; s += 32) sc[s] = __fdiv_rn(sc[s], sum);
      }
      consumer_sync(kConsumerThreads);
      float a0 = 0.f, a1 = 0.f;
      for (int s = warp; s <= p; s += kWarps) {
        const float pr = sc[s];
        float v0, v1;
        if (s == p) {
          v0 = av[2 * lane];
          v1 = av[2 * lane + 1];
        } else {
          const uint32_t vv = __ldcg(reinterpret_cast<const unsigned int *>(vcache + s * kHeadDim) + lane);
          v0 = bf_lo(vv);
          v1 = bf_hi(vv);
        }
        a0 = fmaf(pr, v0, a0);
        a1 = fmaf(pr, v1, a1);
      }
      pv[warp * kHeadDim + 2 * lane] = a0;
      pv[warp * kHeadDim + 2 * lane + 1] = a1;
      consumer_sync(kConsumerThreads);
      if (tid < kHeadDim) {
        float o = 0.f;
        for (int w = 0; w < kWarps; ++w) o += pv[w * kHeadDim + tid];
        xs[m * P.xs_elems + tid] = f2bf(o);
      }
      consumer_sync(kConsumerThreads);
    }
    const MatRange r = phase_range(4 * layer + 1);
    float *opart = P.opart;
    const int QH = P.QH, H = P.H;
    return consume_rg_per_warp<MB, W8>(
        ring, r, xs, P.xs_elems, mrows, &P.result->ctrl, P.limit_ns,
        [&](int m, int row, float v) { opart[(static_cast<size_t>(m) * QH + head) * H + row] = v; });
  }

  __device__ bool phase_c(int layer) {
    const LayerPtrs &lp = P.layers[layer];
    for (int idx = tid; idx < mrows * P.H; idx += kConsumerThreads) {
      const int m = idx / P.H, i = idx - m * P.H;
      hx[idx] = h1_value(lp, layer, m, i);
    }
    consumer_sync(kConsumerThreads);
    norm_rows(lp.gamma_post);
    const MatRange r = phase_range(4 * layer + 2);
    if (!consume_splitk<MB, W8>(ring, r, xs, P.xs_elems, mrows, red, P.red_rows, &P.result->ctrl,
                                P.limit_ns))
      return false;
    consumer_sync(kConsumerThreads);
    const int b0 = r.g0 / 2, npairs = (r.g1 - r.g0) / 2;
    for (int idx = tid; idx < mrows * npairs * 8; idx += kConsumerThreads) {
      const int m = idx / (npairs * 8);
      const int rem = idx - m * npairs * 8;
      const int pr = rem >> 3, rr = rem & 7;
      float g = red_sum(m, pr * 16 + rr);
      float u = red_sum(m, pr * 16 + 8 + rr);
      if (W8) {
        g *= lp.s_gu[(2 * (b0 + pr)) * 8 + rr];
        u *= lp.s_gu[(2 * (b0 + pr) + 1) * 8 + rr];
      }
      g = rbf(g);
      u = rbf(u);
      // SwiGLU (cpu_backend.py:154-165): g / (1 + exp(-clip(g, -80, 80))) * u
      const float e = expf(-fminf(fmaxf(g, -80.f), 80.f));
      const float a = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, e)), u);
      P.act[static_cast<size_t>(m) * P.I + (b0 + pr) * 8 + rr] = f2bf(a);
    }
    return true;
  }

  __device__ bool phase_d(int layer) {
    const LayerPtrs &lp = P.layers[layer];
    const int n8 = P.I / 8;
    for (int idx = tid; idx < mrows * n8; idx += kConsumerThreads) {
      const int m = idx / n8, c = idx - m * n8;
      const uint4 v = __ldcg(reinterpret_cast<const uint4 *>(P.act + static_cast<size_t>(m) * P.I) + c);
      *reinterpret_cast<uint4 *>(xs + m * P.xs_elems + c * 8) = v;
    }
    consumer_sync(kConsumerThreads);
    const MatRange r = phase_range(4 * layer + 3);
    if (!consume_splitk<MB, W8>(ring, r, xs, P.xs_elems, mrows, red, P.red_rows, &P.result->ctrl,
                                P.limit_ns))
      return false;
    consumer_sync(kConsumerThreads);
    const int nrows = (r.g1 - r.g0) * 8;
    for (int idx = tid; idx < mrows * nrows; idx += kConsumerThreads) {
      const int m = idx / nrows, lr = idx - m * nrows;
      const int row = r.g0 * 8 + lr;
      float v = red_sum(m, lr);
      if (W8) v *= lp.s_down[row];
      const float d = rbf(v);
      const float h1 = h1_value(lp, layer, m, row);
      P.hbuf[static_cast<size_t>(m) * P.H + row] = f2bf(__fadd_rn(d, h1));
    }
    return true;
  }

  __device__ bool phase_e() {
    const int warp = tid >> 5, lane = tid & 31;
    for (int idx = tid; idx < mrows * P.H; idx += kConsumerThreads) {
      hx[idx] = bf2f(__ldcg(P.hbuf + idx));
    }
    consumer_sync(kConsumerThreads);
    norm_rows(P.gamma_final);
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
          if (v > bv[m] || (v == bv[m] && row < bi[m])) {
            bv[m] = v;
            bi[m] = row;
          }
        });
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
    if (tid == 0) *s_flag = __ldcg(&P.st->rows);
    consumer_sync(kConsumerThreads);
    mrows = min(*s_flag, MB);
    if (P.stall_ns != 0 && tid == 0) stall_on_unset_flag(ctrl, P.stall_ns);
    consumer_sync(kConsumerThreads);
    bool ok = ld_volatile_int(&ctrl->abort) == 0;
    const int nph = 4 * P.L + 2;
    unsigned int barriers = 0;
    bool ran_e = false;
    for (int k = P.phase_begin; k < P.phase_end && ok; ++k) {
      if (P.trace && tid == 0) P.trace[static_cast<size_t>(cta) * nph + k] = globaltimer_ns();
      if (k >= 4 * P.L) {
        ok = phase_e();
        ran_e = true;
      } else {
        const int layer = k >> 2;
        switch (k & 3) {
          case 0: ok = phase_a(layer); break;
          case 1: ok = phase_b(layer); break;
          case 2: ok = phase_c(layer); break;
          default: ok = phase_d(layer); break;
        }
      }
      if (ok && k + 1 < P.phase_end) {
        ++barriers;
        ok = grid_barrier(ctrl, barriers * static_cast<unsigned int>(G), kConsumerThreads, P.limit_ns,
                          s_flag);
      }
    }
    if (P.trace && tid == 0) P.trace[static_cast<size_t>(cta) * nph + nph - 1] = globaltimer_ns();
    // exit protocol: the last CTA finishes the argmax and resets the counters
    consumer_sync(kConsumerThreads);
    if (tid == 0) {
      __threadfence();
      const unsigned int prev = atomicAdd(&ctrl->done, 1u);
      *s_last = (prev == static_cast<unsigned int>(G) - 1u) ? 1 : 0;
    }
    consumer_sync(kConsumerThreads);
    if (*s_last) {
      __threadfence();
      const int warp = tid >> 5, lane = tid & 31;
      if (ran_e && warp == 0 && ld_volatile_int(&ctrl->abort) == 0) {
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
          if (ran_e) {
            const int tok = P.result->out_token[0];
            P.gen_out[st->n_out] = tok;
            st->n_out = st->n_out + 1;
            if (next < 0) next = tok;
          }
          st->token[0] = next < 0 ? 0 : next;
          st->pos[0] = p + 1;
        }
        atomicExch(&ctrl->bar, 0u);
        atomicExch(&ctrl->done, 0u);
        __threadfence();
      }
    }
  }

  // ---- producer main ----------------------------------------------------------
  __device__ void run_producer() {
    Ctrl *ctrl = &P.result->ctrl;
    const uint64_t policy = policy_evict_first();
    uint32_t issued = 0;
    for (int k = P.phase_begin; k < P.phase_end; ++k) {
      const MatRange r = phase_range(k);
      if (!produce_range(ring, r, issued, ctrl, P.limit_ns, policy)) break;
    }
    drain_ring(ring, issued, ctrl);
  }
};

template <int MB, bool W8>
__global__ void __launch_bounds__(kThreads, 1) decoder_kernel(const __grid_constant__ DecParams P) {
  extern __shared__ __align__(1024) uint8_t smem[];
  DecoderCta<MB, W8> cx(P, smem);
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
