// hb_gemv.cuh -- standalone weight-streaming GEMV (BF16 or W8 weights) for up
// to 8 activation vectors, with an optional fused argmax over the rows.
//
//   y[b][r] = bf16(sum_k W[r][k] x[b][k] [* scale[r]])   (or FP32, or not stored)
//
// Same weight stream as the decoder (hb_stream.cuh).  Small-K / few-rows
// shapes use the split-K consumer (all warps on every chunk, latency mode);
// shapes with >= 16 row groups per CTA use one warp per chunk (throughput
// mode, the LM-head case).  The argmax is finished by the last CTA to arrive
// (a done counter in the caller's scratch), so there is no grid barrier.
#pragma once

#include "hb_stream.cuh"

namespace hb {

constexpr int kMaxBatchGemv = 8;

struct GemvParams {
  const uint8_t *w;
  const float *scales;
  int rows, kc, K;
  const __nv_bfloat16 *x;   // [batch][K]
  int batch;
  void *y;                  // [batch][rows]
  int out_mode;             // 0 bf16, 1 f32, 2 none
  int argmax;
  int32_t *argmax_out;      // [batch]
  Ctrl *ctrl;
  float *part_val;          // [grid][8]
  int *part_idx;
  int nslots;
  int red_rows;
  int per_warp;
  uint64_t limit_ns;
  uint64_t stall_ns;        // test hook: CTA 0 first waits this long on a flag nothing sets
};

__host__ __device__ inline size_t gemv_smem_bytes(int nslots, int mb, int K, int red_rows) {
  size_t o = static_cast<size_t>(nslots) * kSlotBytes + 16 * nslots;
  o = align_up(o, 128);
  o += align_up(static_cast<size_t>(mb) * K * 2, 128);
  o += align_up(static_cast<size_t>(kWarps) * mb * red_rows * 4, 128);
  o += 1024;
  return o;
}

template <int MB, bool W8>
__global__ void __launch_bounds__(kThreads, 1) gemv_kernel(const __grid_constant__ GemvParams P) {
  extern __shared__ __align__(1024) uint8_t smem[];
  Ring ring;
  size_t o = 0;
  ring.slots = smem;
  o += static_cast<size_t>(P.nslots) * kSlotBytes;
  ring.full = reinterpret_cast<uint64_t *>(smem + o);
  o += 8 * P.nslots;
  ring.empty = reinterpret_cast<uint64_t *>(smem + o);
  o += 8 * P.nslots;
  o = align_up(o, 128);
  __nv_bfloat16 *xs = reinterpret_cast<__nv_bfloat16 *>(smem + o);
  o += align_up(static_cast<size_t>(MB) * P.K * 2, 128);
  float *red = reinterpret_cast<float *>(smem + o);
  o += align_up(static_cast<size_t>(kWarps) * MB * P.red_rows * 4, 128);
  float *s_bv = reinterpret_cast<float *>(smem + o);
  int *s_bi = reinterpret_cast<int *>(s_bv + kWarps * kMaxBatchGemv);
  int *s_last = s_bi + kWarps * kMaxBatchGemv;
  ring.nslots = P.nslots;
  ring.slot = 0;
  ring.parity = 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < P.nslots; ++i) {
      mbar_init(&ring.full[i], 1);
      mbar_init(&ring.empty[i], kWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  const int G = gridDim.x, cta = blockIdx.x, tid = threadIdx.x;
  const int n_rg = P.rows / 8;
  const MatRange r{P.w, split_lo(n_rg, G, cta), split_lo(n_rg, G, cta + 1), P.kc};
  Ctrl *ctrl = P.ctrl;

  if (tid >= kConsumerThreads) {
    if (tid == kConsumerThreads) {
      Producer prod{&ring, RingPos{0, 0}, 0, ctrl, P.limit_ns, policy_evict_first()};
      prod.issue_range(r);
      prod.drain();
    }
    return;
  }

  if (P.stall_ns != 0 && cta == 0 && tid == 0) stall_on_unset_flag(ctrl, P.stall_ns);
  const int mrows = min(P.batch, MB);
  const int n8 = P.K / 8;
  for (int idx = tid; idx < mrows * n8; idx += kConsumerThreads) {
    const int m = idx / n8, c = idx - m * n8;
    *reinterpret_cast<uint4 *>(xs + static_cast<size_t>(m) * P.K + c * 8) =
        reinterpret_cast<const uint4 *>(P.x + static_cast<size_t>(m) * P.K)[c];
  }
  consumer_sync(kConsumerThreads);

  float bv[MB];
  int bi[MB];
#pragma unroll
  for (int m = 0; m < MB; ++m) {
    bv[m] = -INFINITY;
    bi[m] = 0x7fffffff;
  }
  const float *scales = P.scales;
  auto emit = [&](int m, int row, float v) {
    if (W8) v *= scales[row];
    if (P.out_mode == 0)
      reinterpret_cast<__nv_bfloat16 *>(P.y)[static_cast<size_t>(m) * P.rows + row] = f2bf(v);
    else if (P.out_mode == 1)
      reinterpret_cast<float *>(P.y)[static_cast<size_t>(m) * P.rows + row] = v;
    if (argmax_better(v, row, bv[m], bi[m])) {
      bv[m] = v;
      bi[m] = row;
    }
  };
  bool ok;
  if (P.per_warp) {
    ok = consume_chunk_per_warp<MB, W8>(ring, r, xs, P.K, mrows, ctrl, P.limit_ns, emit);
  } else {
    ok = consume_splitk<MB, W8>(ring, r, xs, P.K, mrows, red, P.red_rows, ctrl, P.limit_ns);
    consumer_sync(kConsumerThreads);
    const int nrows = (r.g1 - r.g0) * 8;
    if (ok) {
      for (int idx = tid; idx < mrows * nrows; idx += kConsumerThreads) {
        const int m = idx / nrows, lr = idx - m * nrows;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) v += red[(w * MB + m) * P.red_rows + lr];
#pragma unroll
        for (int mm = 0; mm < MB; ++mm)
          if (mm == m) emit(mm, r.g0 * 8 + lr, v);
      }
    }
  }
  if (!P.argmax) return;
  const int warp = tid >> 5, lane = tid & 31;
#pragma unroll
  for (int m = 0; m < MB; ++m) {
    float v = bv[m];
    int i = bi[m];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, off);
      const int oi = __shfl_xor_sync(0xffffffffu, i, off);
      argmax_merge(v, i, ov, oi);
    }
    if (lane == 0) {
      s_bv[warp * kMaxBatchGemv + m] = v;
      s_bi[warp * kMaxBatchGemv + m] = i;
    }
  }
  consumer_sync(kConsumerThreads);
  if (tid < mrows) {
    float v = -INFINITY;
    int i = 0x7fffffff;
    for (int w = 0; w < kWarps; ++w) argmax_merge(v, i, s_bv[w * kMaxBatchGemv + tid], s_bi[w * kMaxBatchGemv + tid]);
    P.part_val[cta * kMaxBatchGemv + tid] = v;
    P.part_idx[cta * kMaxBatchGemv + tid] = i;
  }
  consumer_sync(kConsumerThreads);
  if (tid == 0) {
    __threadfence();
    const unsigned int prev = atomicAdd(&ctrl->done, 1u);
    *s_last = (prev == static_cast<unsigned int>(G) - 1u) ? 1 : 0;
  }
  consumer_sync(kConsumerThreads);
  if (*s_last && warp == 0) {
    __threadfence();
    if (ld_volatile_int(&ctrl->abort) != 0) {
      // some CTA gave up a wait: its partial is not a result, so no row's
      // argmax is one either
      if (lane < mrows) P.argmax_out[lane] = -1;
      if (lane == 0) {
        atomicExch(&ctrl->done, 0u);
        __threadfence();
      }
      return;
    }
    for (int m = 0; m < mrows; ++m) {
      float v = -INFINITY;
      int i = 0x7fffffff;
      for (int c = lane; c < G; c += 32)
        argmax_merge(v, i, __ldcg(P.part_val + c * kMaxBatchGemv + m), __ldcg(P.part_idx + c * kMaxBatchGemv + m));
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, off);
        const int oi = __shfl_xor_sync(0xffffffffu, i, off);
        argmax_merge(v, i, ov, oi);
      }
      if (lane == 0) P.argmax_out[m] = i;
    }
    if (lane == 0) {
      atomicExch(&ctrl->done, 0u);
      __threadfence();
    }
  }
  (void)ok;
}

}  // namespace hb
