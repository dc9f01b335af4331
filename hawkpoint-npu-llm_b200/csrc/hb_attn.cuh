// hb_attn.cuh -- per-head attention arithmetic shared by the persistent
// decoder kernel (hb_decoder.cuh) and the batched kernels (hb_tc.cuh), so a
// row's attention is computed by the same instructions on either path
// (cpu_backend.py:78-129).
#pragma once

#include "hb_device.cuh"

namespace hb {

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const uint32_t a = __bfloat16_as_ushort(f2bf(lo));
  const uint32_t b = __bfloat16_as_ushort(f2bf(hi));
  return a | (b << 16);
}

// Byte offset of 16-byte block cb (dims 8cb..8cb+7) of position s in a K or
// V block: rows of 128 bytes, blocks XOR-swizzled by the row so the 8 rows
// an ldmatrix reads fall in distinct banks.
__device__ __forceinline__ int kv_off(int s, int cb) { return s * 128 + ((cb ^ (s & 7)) << 4); }

// Rotate-half RoPE of the BF16 values x0 (dim d) and x1 (dim d + 32) of a
// head with the position's cos / sin of dim d (unfused mul / sub / add, as
// cpu_backend.py:78-93).
__device__ __forceinline__ void rope_vals(float x0, float x1, float c, float sn, __nv_bfloat16 &lo,
                                          __nv_bfloat16 &hi) {
  lo = f2bf(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)));
  hi = f2bf(__fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, sn)));
}

// rope_vals of elements d and d + 32 of a 64-element head held as BF16
// pairs in w32[0..32).
__device__ __forceinline__ void rope_pair_cs(const uint32_t *w32, int d, float c, float sn, __nv_bfloat16 &lo,
                                             __nv_bfloat16 &hi) {
  const uint32_t a = w32[d >> 1], b = w32[(d + 32) >> 1];
  rope_vals((d & 1) ? bf_hi(a) : bf_lo(a), (d & 1) ? bf_hi(b) : bf_lo(b), c, sn, lo, hi);
}

// Lane d's part of position pr's K row (rotated dims d, d + 32) in a
// swizzled K history block.
__device__ __forceinline__ void put_k(uint8_t *kb, int pr, int d, __nv_bfloat16 klo, __nv_bfloat16 khi) {
  *reinterpret_cast<__nv_bfloat16 *>(kb + kv_off(pr, d >> 3) + (d & 7) * 2) = klo;
  *reinterpret_cast<__nv_bfloat16 *>(kb + kv_off(pr, 4 + (d >> 3)) + (d & 7) * 2) = khi;
}

// Lane d's part of position pr's V row (dims 2d, 2d + 1) in a swizzled V
// history block.
__device__ __forceinline__ void put_v(uint8_t *vb, int pr, int d, uint32_t vword) {
  *reinterpret_cast<uint32_t *>(vb + kv_off(pr, (2 * d) >> 3) + ((2 * d) & 7) * 2) = vword;
}

__device__ __forceinline__ void put_kv(uint8_t *kb, uint8_t *vb, int pr, int d, __nv_bfloat16 klo,
                                       __nv_bfloat16 khi, uint32_t vword) {
  put_k(kb, pr, d, klo, khi);
  put_v(vb, pr, d, vword);
}

// One warp: scores q.k * 0.125 over positions <= p of a K / V history in
// shared memory (qf: the rotated q in FP32, sc: 64 floats of scratch),
// softmax (max-subtract, exp, IEEE divide) and P.V in FP32; returns this
// lane's output dims 2 * lane, 2 * lane + 1 as a BF16 pair
// (cpu_backend.py:95-129).
__device__ __forceinline__ uint32_t attend_warp(const float *qf, float *sc, const uint8_t *kb, const uint8_t *vb,
                                            int p) {
  const int lane = threadIdx.x & 31;
  // scores: lane takes positions lane and lane + 32
  float s2[2];  // (indexed by unrolled e only)
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int sp = lane + 32 * e;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    if (sp <= p) {
#pragma unroll
      for (int cb = 0; cb < 8; ++cb) {
        const uint4 kw = *reinterpret_cast<const uint4 *>(kb + kv_off(sp, cb));
        const float *q = qf + 8 * cb;
        float &a = acc[cb & 3];
        a = fmaf(bf_lo(kw.x), q[0], a);
        a = fmaf(bf_hi(kw.x), q[1], a);
        a = fmaf(bf_lo(kw.y), q[2], a);
        a = fmaf(bf_hi(kw.y), q[3], a);
        a = fmaf(bf_lo(kw.z), q[4], a);
        a = fmaf(bf_hi(kw.z), q[5], a);
        a = fmaf(bf_lo(kw.w), q[6], a);
        a = fmaf(bf_hi(kw.w), q[7], a);
      }
    }
    s2[e] = sp <= p ? ((acc[0] + acc[1]) + (acc[2] + acc[3])) * 0.125f : -INFINITY;
  }
  float mx = fmaxf(s2[0], s2[1]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const float e0 = lane <= p ? expf(__fsub_rn(s2[0], mx)) : 0.f;
  const float e1 = lane + 32 <= p ? expf(__fsub_rn(s2[1], mx)) : 0.f;
  float sum = e0 + e1;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  sc[lane] = __fdiv_rn(e0, sum);
  sc[lane + 32] = __fdiv_rn(e1, sum);
  __syncwarp();
  // P.V: lane takes dims 2*lane, 2*lane+1; two chains over even / odd positions
  float o00 = 0.f, o01 = 0.f, o10 = 0.f, o11 = 0.f;
  const int cbv = (2 * lane) >> 3, offv = ((2 * lane) & 7) * 2;
  int sp = 0;
  for (; sp + 1 <= p; sp += 2) {
    const float w0 = sc[sp], w1 = sc[sp + 1];
    const uint32_t v0 = *reinterpret_cast<const uint32_t *>(vb + kv_off(sp, cbv) + offv);
    const uint32_t v1 = *reinterpret_cast<const uint32_t *>(vb + kv_off(sp + 1, cbv) + offv);
    o00 = fmaf(w0, bf_lo(v0), o00);
    o01 = fmaf(w0, bf_hi(v0), o01);
    o10 = fmaf(w1, bf_lo(v1), o10);
    o11 = fmaf(w1, bf_hi(v1), o11);
  }
  if (sp <= p) {
    const float w0 = sc[sp];
    const uint32_t v0 = *reinterpret_cast<const uint32_t *>(vb + kv_off(sp, cbv) + offv);
    o00 = fmaf(w0, bf_lo(v0), o00);
    o01 = fmaf(w0, bf_hi(v0), o01);
  }
  return pack_bf16x2(o00 + o10, o01 + o11);
}


}  // namespace hb
