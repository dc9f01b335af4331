// hb_stream.cuh -- the weight stream shared by the decoder and GEMV kernels.
//
// Each CTA owns a contiguous run of row groups of every projection it works
// on.  One producer thread copies that run, chunk by chunk, into a ring of
// shared-memory slots with cp.async.bulk (completion on a per-slot "full"
// mbarrier); the consumer warps compute on a slot and release it on its
// "empty" mbarrier.  The producer never waits on activations, so it keeps
// streaming weights for the next phases while the consumers wait for their
// inputs: that latency hides under the HBM stream.
//
// Packed projection layout (runtime/layout.py): row group g (8 rows) at
// g * kc * 128 bytes, then chunk column j (16 bytes of each of the 8 rows) at
// j * 128 + r * 16.  A chunk is either several whole row groups or, when one
// row group is larger than a slot, a K-slice of kPartCols chunk columns.
//
// BF16 dot products run on the tensor cores (mma.m16n8k16, FP32 accumulate):
// the weights of a row group are the B operand as stored, so nothing is
// converted; W8 weights use FP32 CUDA-core FMAs.
#pragma once

#include "hb_device.cuh"

namespace hb {

constexpr int kWarps = 7;                  // consumer warps
constexpr int kConsumerThreads = kWarps * 32;
constexpr int kThreads = kConsumerThreads + 32;  // + producer warp
constexpr uint32_t kSlotBytes = 16384;
constexpr int kPartCols = 128;             // chunk columns per K-slice (kSlotBytes / 128)
constexpr int kColGroups = kWarps * 4;     // split-K column groups per CTA

struct MatRange {
  const uint8_t *base;  // row group 0 of the matrix
  int g0, g1;           // row-group range owned by this CTA
  int kc;               // 16-byte chunk columns per row
};

// Balanced contiguous split of n units over parts.
__device__ __forceinline__ int split_lo(int n, int parts, int idx) {
  return static_cast<int>((static_cast<long long>(n) * idx) / parts);
}

// The chunks of a range, in stream order: whole row groups packed into a
// slot, or -- when one row group exceeds a slot -- K-slices of kPartCols
// chunk columns.  f(rg, nrg, col0, ncols, last_part) returns false to stop.
// Producer and consumers walk the same sequence.
template <class F>
__device__ __forceinline__ bool for_each_chunk(const MatRange &r, F &&f) {
  if (r.base == nullptr || r.g1 <= r.g0) return true;
  const int rgb = r.kc * 128;
  if (rgb <= static_cast<int>(kSlotBytes)) {
    const int rpc = static_cast<int>(kSlotBytes) / rgb;
    for (int g = r.g0; g < r.g1; g += rpc)
      if (!f(g, min(rpc, r.g1 - g), 0, r.kc, true)) return false;
  } else {
    for (int g = r.g0; g < r.g1; ++g)
      for (int c0 = 0; c0 < r.kc; c0 += kPartCols)
        if (!f(g, 1, c0, min(kPartCols, r.kc - c0), c0 + kPartCols >= r.kc)) return false;
  }
  return true;
}

__device__ __forceinline__ int num_chunks(const MatRange &r) {
  int n = 0;
  for_each_chunk(r, [&](int, int, int, int, bool) {
    ++n;
    return true;
  });
  return n;
}

// Shared-memory ring of one CTA.  Slot index and phase parity advance
// incrementally (no divisions on the per-chunk path).
struct Ring {
  uint8_t *slots;
  uint64_t *full;
  uint64_t *empty;
  int nslots;
  int slot;          // consumer cursor (identical in every consumer thread)
  uint32_t parity;
};

struct RingPos {
  int slot;
  uint32_t parity;
};

__device__ __forceinline__ void ring_advance(RingPos &p, int by, int nslots) {
  p.slot += by;
  while (p.slot >= nslots) {
    p.slot -= nslots;
    p.parity ^= 1u;
  }
}

// Producer side: issue one chunk into the next slot.
struct Producer {
  Ring *ring;
  RingPos pos;
  uint32_t issued;
  Ctrl *ctrl;
  uint64_t limit_ns;
  uint64_t policy;

  __device__ __forceinline__ bool issue(const uint8_t *src, uint32_t bytes) {
    // reuse of a slot waits for the consumers to release its previous use
    if (issued >= static_cast<uint32_t>(ring->nslots) &&
        !mbar_wait(&ring->empty[pos.slot], pos.parity ^ 1u, ctrl, limit_ns, kWhereEmpty))
      return false;
    mbar_arrive_expect_tx(&ring->full[pos.slot], bytes);
    bulk_g2s_evict_first(ring->slots + static_cast<size_t>(pos.slot) * kSlotBytes, src, bytes,
                         &ring->full[pos.slot], policy);
    ++issued;
    ring_advance(pos, 1, ring->nslots);
    return true;
  }

  __device__ __forceinline__ bool issue_range(const MatRange &r) {
    const size_t rgb = static_cast<size_t>(r.kc) * 128;
    return for_each_chunk(r, [&](int g, int nrg, int c0, int ncols, bool) {
      const uint8_t *src = r.base + static_cast<size_t>(g) * rgb + static_cast<size_t>(c0) * 128;
      return issue(src, static_cast<uint32_t>(nrg) * ncols * 128);
    });
  }

  // Wait until every issued copy has landed, so no bulk copy still targets
  // this CTA's shared memory when it exits.
  __device__ __forceinline__ void drain() {
    const int n = issued < static_cast<uint32_t>(ring->nslots) ? static_cast<int>(issued) : ring->nslots;
    RingPos p = pos;
    for (int i = 0; i < n; ++i) {
      // step back one slot
      if (p.slot == 0) {
        p.slot = ring->nslots - 1;
        p.parity ^= 1u;
      } else {
        --p.slot;
      }
      const uint64_t start = globaltimer_ns();
      while (!mbar_try_wait(&ring->full[p.slot], p.parity)) {
        if (globaltimer_ns() - start > 2000000000ull) {
          raise_error(ctrl, kErrTimeout, kWhereDrain);
          return;
        }
      }
    }
  }
};

// Consumer: wait for the chunk at ring position p.
__device__ __forceinline__ bool ring_wait(Ring &ring, const RingPos &p, Ctrl *ctrl, uint64_t limit_ns) {
  return mbar_wait(&ring.full[p.slot], p.parity, ctrl, limit_ns, kWhereFull);
}

__device__ __forceinline__ const uint8_t *slot_ptr(const Ring &ring, int slot) {
  return ring.slots + static_cast<size_t>(slot) * kSlotBytes;
}

// Lanes c < n each wait (bounded) for the full barrier of the chunk c slots
// after p, so a warp waiting for several chunks pays about one wait.
__device__ __forceinline__ bool ring_wait_lanes(Ring &ring, const RingPos &p, int n, Ctrl *ctrl,
                                                uint64_t limit_ns) {
  const int lane = threadIdx.x & 31;
  bool ok = true;
  if (lane < n) {
    int s = p.slot + lane;
    uint32_t par = p.parity;
    while (s >= ring.nslots) {
      s -= ring.nslots;
      par ^= 1u;
    }
    ok = mbar_wait(&ring.full[s], par, ctrl, limit_ns, kWhereFull);
  }
  return __all_sync(0xffffffffu, ok);
}

// ---- tensor-core dot products (BF16) -------------------------------------------
// One row group (8 weight rows) is the B operand of mma.m16n8k16 (n = the 8
// rows, k = 16 columns); the activations are the A operand with batch row m
// in row m (rows >= MB are zero).  D[m][n] accumulates in FP32.  The packed
// weight layout is exactly ldmatrix's 8x8 tiles: chunk column j of the group
// holds 8 rows x 16 bytes at j * 128.
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

// Accumulate the dot products of one row group over chunk columns
// [jc_begin, jc_end) stepping by `stride` (multiples of 4): 4 chunk columns
// = 2 k16 steps per iteration.  `sg` = the group's bytes in shared memory,
// `xrow` = this lane's activation row (lane/4) or nullptr for zero rows,
// `col0` = chunk-column offset of sg within the full K.
__device__ __forceinline__ void mma_group(float (&d)[4], const uint8_t *sg, const __nv_bfloat16 *xrow,
                                          int col0, int jc_begin, int jc_end, int stride) {
  const int lane = threadIdx.x & 31;
  const uint32_t base = smem_u32(sg) + ((lane >> 3) * 128) + ((lane & 7) * 16);
  const int t2 = (lane & 3) * 2;
  for (int jc = jc_begin; jc < jc_end; jc += stride) {
    uint32_t b[4];
    ldsm_x4(b, base + jc * 128);
    uint32_t a0 = 0, a2 = 0, c0 = 0, c2 = 0;
    if (xrow != nullptr) {
      const __nv_bfloat16 *x = xrow + (col0 + jc) * 8 + t2;
      a0 = *reinterpret_cast<const uint32_t *>(x);
      a2 = *reinterpret_cast<const uint32_t *>(x + 8);
      c0 = *reinterpret_cast<const uint32_t *>(x + 16);
      c2 = *reinterpret_cast<const uint32_t *>(x + 24);
    }
    mma_16816(d, a0, a2, b[0], b[1]);
    mma_16816(d, c0, c2, b[2], b[3]);
  }
}

// CUDA-core dot products for W8 (int8 weights, chunk column = 16 weights).
__device__ __forceinline__ float dot_w8_cols(const uint8_t *sg, const __nv_bfloat16 *x, int col0, int j0,
                                             int jend, int stride) {
  const int rr = threadIdx.x & 7;
  float acc = 0.f;
  for (int j = j0; j < jend; j += stride) {
    const uint4 w = *reinterpret_cast<const uint4 *>(sg + j * 128 + rr * 16);
    const uint4 x0 = *reinterpret_cast<const uint4 *>(x + (col0 + j) * 16);
    const uint4 x1 = *reinterpret_cast<const uint4 *>(x + (col0 + j) * 16 + 8);
    acc = dot16_i8(w, x0, x1, acc);
  }
  return acc;
}

// One split-K step of a warp over up to kStepRows row groups that share
// their columns (whole row groups of several chunks, or the same K-slice of
// several row groups).  unit[i] = shared address of row group i's first
// chunk column of the slice + this lane's ldmatrix offset; the warp takes
// chunk columns warp*4 + kColGroups*u.  The row groups accumulate in
// independent chains d[i], so one activation fragment feeds nb MMAs and the
// MMA latency is hidden behind the other chains.
constexpr int kStepRows = 4;

template <int NR>
__device__ __forceinline__ void mma_step_rows(float (&d)[kStepRows][4], const uint32_t (&unit)[kStepRows],
                                              const __nv_bfloat16 *xrow, int col0, int ncols) {
  for (int jc = (threadIdx.x >> 5) * 4; jc < ncols; jc += kColGroups) {
    uint32_t b[NR][4];
#pragma unroll
    for (int i = 0; i < NR; ++i) ldsm_x4(b[i], unit[i] + jc * 128);
    uint32_t a0 = 0u, a2 = 0u, c0 = 0u, c2 = 0u;
    if (xrow != nullptr) {
      const __nv_bfloat16 *x = xrow + (col0 + jc) * 8;
      a0 = *reinterpret_cast<const uint32_t *>(x);
      a2 = *reinterpret_cast<const uint32_t *>(x + 8);
      c0 = *reinterpret_cast<const uint32_t *>(x + 16);
      c2 = *reinterpret_cast<const uint32_t *>(x + 24);
    }
#pragma unroll
    for (int i = 0; i < NR; ++i) mma_16816(d[i], a0, a2, b[i][0], b[i][1]);
#pragma unroll
    for (int i = 0; i < NR; ++i) mma_16816(d[i], c0, c2, b[i][2], b[i][3]);
  }
}

__device__ __forceinline__ void mma_step(float (&d)[kStepRows][4], const uint32_t (&unit)[kStepRows], int nb,
                                         const __nv_bfloat16 *xrow, int col0, int ncols) {
  switch (nb) {
    case 4: mma_step_rows<4>(d, unit, xrow, col0, ncols); break;
    case 3: mma_step_rows<3>(d, unit, xrow, col0, ncols); break;
    case 2: mma_step_rows<2>(d, unit, xrow, col0, ncols); break;
    default: mma_step_rows<1>(d, unit, xrow, col0, ncols); break;
  }
}

// Split-K consumption of a row-group range by all consumer warps (latency
// mode): every warp sees every chunk and takes 1/kWarps of its columns.  The
// per-warp partial of (batch row m, local row) goes to
// red[(warp * MB + m) * red_rows + local_row]; the caller sums the warps
// after a consumer_sync.  xs: BF16 activations [MB][K] in shared memory.
template <int MB, bool W8>
__device__ __forceinline__ bool consume_splitk(Ring &ring, const MatRange &r, const __nv_bfloat16 *xs, int K,
                                               int mrows, float *red, int red_rows, Ctrl *ctrl,
                                               uint64_t limit_ns) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (r.base == nullptr || r.g1 <= r.g0) return true;
  if constexpr (!W8) {
    const int am = lane >> 2, n = (lane & 3) * 2;
    const __nv_bfloat16 *xrow = am < mrows ? xs + static_cast<size_t>(am) * K + n : nullptr;
    const uint32_t lane_off = ((lane >> 3) * 128) + ((lane & 7) * 16);
    const int rgb = r.kc * 128;
    float d[kStepRows][4];
    uint32_t unit[kStepRows];
    RingPos pos{ring.slot, ring.parity};
#pragma unroll
    for (int i = 0; i < kStepRows; ++i) d[i][0] = d[i][1] = d[i][2] = d[i][3] = 0.f;
    // wait for the n (<= kStepRows) chunks from the cursor on, one lane per
    // chunk (the warp pays one wait latency, not n)
    auto wait_chunks = [&](int n) {
      const bool ok = ring_wait_lanes(ring, pos, n, ctrl, limit_ns);
#pragma unroll
      for (int c = 0; c < kStepRows; ++c) {
        int sl = pos.slot + c;
        if (sl >= ring.nslots) sl -= ring.nslots;
        unit[c] = smem_u32(slot_ptr(ring, sl)) + lane_off;
      }
      return ok;
    };
    // hand the n chunks at the cursor back to the producer, one lane each
    auto release_chunks = [&](int n) {
      __syncwarp();
      if (lane < n) {
        int sl = pos.slot + lane;
        if (sl >= ring.nslots) sl -= ring.nslots;
        mbar_arrive_count(&ring.empty[sl], 1);
      }
      ring_advance(pos, n, ring.nslots);
    };
    // row groups g..g+nb-1 are complete
    auto flush = [&](int g, int nb) {
#pragma unroll
      for (int i = 0; i < kStepRows; ++i) {
        if (i < nb && am < mrows) {
          float *o = red + (warp * MB + am) * red_rows + (g + i - r.g0) * 8 + n;
          o[0] = d[i][0];
          o[1] = d[i][1];
        }
        d[i][0] = d[i][1] = d[i][2] = d[i][3] = 0.f;
      }
    };
    if (rgb > static_cast<int>(kSlotBytes) || r.g1 - r.g0 == 1) {
      // one row group (or K-slices of row groups): chunk by chunk, one
      // accumulator chain per warp
      const __nv_bfloat16 *xr = am < mrows ? xs + static_cast<size_t>(am) * K : nullptr;
      const bool ok = for_each_chunk(r, [&](int g, int nrg, int col0, int ncols, bool last) {
        if (!ring_wait(ring, pos, ctrl, limit_ns)) return false;
        const uint8_t *sc = slot_ptr(ring, pos.slot);
        for (int q = 0; q < nrg; ++q) {
          mma_group(d[0], sc + static_cast<size_t>(q) * ncols * 128, xr, col0, warp * 4, ncols, kColGroups);
          if (last) flush(g + q, 1);
        }
        release_chunks(1);
        return true;
      });
      if (!ok) return false;
    } else if (2 * rgb > static_cast<int>(kSlotBytes)) {
      // one row group per chunk: up to kStepRows chunks per step
      // a step waits for at most nslots chunks: the producer must be able
      // to have them all in flight at once
      const int maxn = min(kStepRows, ring.nslots);
      for (int g = r.g0; g < r.g1; g += maxn) {
        const int nb = min(maxn, r.g1 - g);
        if (!wait_chunks(nb)) return false;
        mma_step(d, unit, nb, xrow, 0, r.kc);
        flush(g, nb);
        release_chunks(nb);
      }
    } else {
      // several row groups per chunk, kStepRows at a time
      const int rpc = static_cast<int>(kSlotBytes) / rgb;
      for (int g = r.g0; g < r.g1;) {
        if (!wait_chunks(1)) return false;
        const uint32_t cbase = unit[0];
        const int take = min(rpc, r.g1 - g);
        for (int t0 = 0; t0 < take; t0 += kStepRows) {
#pragma unroll
          for (int i = 0; i < kStepRows; ++i) unit[i] = cbase + (t0 + i) * rgb;
          const int nb = min(kStepRows, take - t0);
          mma_step(d, unit, nb, xrow, 0, r.kc);
          flush(g + t0, nb);
        }
        release_chunks(1);
        g += take;
      }
    }
    ring.slot = pos.slot;
    ring.parity = pos.parity;
    return true;
  } else {
    float acc[MB];
#pragma unroll
    for (int m = 0; m < MB; ++m) acc[m] = 0.f;
    RingPos pos{ring.slot, ring.parity};
    const bool ok = for_each_chunk(r, [&](int g, int nrg, int col0, int ncols, bool last) {
      if (!ring_wait(ring, pos, ctrl, limit_ns)) return false;
      const uint8_t *s = slot_ptr(ring, pos.slot);
      for (int q = 0; q < nrg; ++q) {
        const uint8_t *sg = s + static_cast<size_t>(q) * ncols * 128;
        const int cg = warp * 4 + (lane >> 3);
#pragma unroll
        for (int m = 0; m < MB; ++m)
          if (m < mrows) acc[m] += dot_w8_cols(sg, xs + static_cast<size_t>(m) * K, col0, cg, ncols, kColGroups);
        if (last) {
          const int local = (g + q - r.g0) * 8;
#pragma unroll
          for (int m = 0; m < MB; ++m) {
            float v = acc[m];
            v += __shfl_xor_sync(0xffffffffu, v, 8);
            v += __shfl_xor_sync(0xffffffffu, v, 16);
            if (lane < 8 && m < mrows) red[(warp * MB + m) * red_rows + local + lane] = v;
            acc[m] = 0.f;
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive_count(&ring.empty[pos.slot], 1);
      ring_advance(pos, 1, ring.nslots);
      return true;
    });
    ring.slot = pos.slot;
    ring.parity = pos.parity;
    return ok;
  }
}

// Chunk-per-warp consumption (throughput mode, whole row groups per chunk):
// chunk t is computed by warp t % 8.  Every warp still waits for and
// releases every chunk in order (empty-barrier count 8), so no warp ever
// waits more than one phase ahead on a slot.
template <int MB, bool W8, class F>
__device__ __forceinline__ bool consume_chunk_per_warp(Ring &ring, const MatRange &r, const __nv_bfloat16 *xs,
                                                       int K, int mrows, Ctrl *ctrl, uint64_t limit_ns,
                                                       F &&on_row) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  RingPos pos{ring.slot, ring.parity};
  int owner = 0;
  const bool ok = for_each_chunk(r, [&](int g, int nrg, int col0, int ncols, bool) {
    if (!ring_wait(ring, pos, ctrl, limit_ns)) return false;
    if (owner == warp) {
      const uint8_t *s = slot_ptr(ring, pos.slot);
      for (int q = 0; q < nrg; ++q) {
        const uint8_t *sg = s + static_cast<size_t>(q) * ncols * 128;
        if (!W8) {
          float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
          const int m = lane >> 2;
          const __nv_bfloat16 *xrow = m < mrows ? xs + static_cast<size_t>(m) * K : nullptr;
          mma_group(d0, sg, xrow, col0, 0, ncols, 8);
          mma_group(d1, sg, xrow, col0, 4, ncols, 8);
          const float v0 = d0[0] + d1[0];
          const float v1 = d0[1] + d1[1];
#pragma unroll
          for (int mm = 0; mm < MB; ++mm) {
            if (mm == m && m < mrows) {  // compile-time batch index for the callback
              on_row(mm, (g + q) * 8 + (lane & 3) * 2, v0);
              on_row(mm, (g + q) * 8 + (lane & 3) * 2 + 1, v1);
            }
          }
        } else {
#pragma unroll
          for (int m = 0; m < MB; ++m) {
            if (m < mrows) {
              float v = dot_w8_cols(sg, xs + static_cast<size_t>(m) * K, col0, lane >> 3, ncols, 4);
              v += __shfl_xor_sync(0xffffffffu, v, 8);
              v += __shfl_xor_sync(0xffffffffu, v, 16);
              if (lane < 8) on_row(m, (g + q) * 8 + lane, v);
            }
          }
        }
      }
    }
    owner = owner + 1 == kWarps ? 0 : owner + 1;
    __syncwarp();
    if (lane == 0) mbar_arrive_count(&ring.empty[pos.slot], 1);
    ring_advance(pos, 1, ring.nslots);
    return true;
  });
  ring.slot = pos.slot;
  ring.parity = pos.parity;
  return ok;
}

}  // namespace hb
