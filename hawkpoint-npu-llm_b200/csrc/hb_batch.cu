// hb_batch.cu -- the batched tensor-core path of libhawkb200.so.
//
// The persistent decoder kernel (hb_decoder.cuh) streams every weight once
// per launch for at most 8 rows on mma.sync.  Prefill (many positions of one
// sequence) and multi-stream decode (one position of many sequences) are
// dense contractions over many rows, so they run here instead as a short
// sequence of kernels per layer around tcgen05 GEMMs (hb_tc.cuh): the
// weights stream once per step for up to 128 rows, accumulate in TMEM, and
// the epilogues apply the reference's BF16 rounding points.
#include <unordered_map>

#include "hb_engine_impl.h"
#include "hb_tc.cuh"

using namespace hbi;

namespace {

// K slices per tile (one cluster) so that tiles x slices fills at most one
// wave (a second, partial wave doubles the time), each slice at least two K
// stages, at most a portable cluster's 8 CTAs.
int choose_ksplit(int tiles, int kst, int sms) {
  int ks = sms / tiles;
  ks = std::min(ks, kst >= 2 ? kst / 2 : 1);
  ks = std::min(ks, hb::tc::kMaxSlices);
  return std::max(ks, 1);
}

// Ring stages: at most 6, no more than a slice has K stages, within about
// 200 KB of shared memory.
int choose_stages(int npad, int ksplit, int kst) {
  const size_t per = hb::tc::kAStageBytes + static_cast<size_t>(npad) * 128;
  const size_t budget = 200u * 1024u - 64u;
  const int s = static_cast<int>(budget / (per + 16));
  return std::max(1, std::min({6, s, (kst + ksplit - 1) / ksplit}));
}

// Ring stages of the persistent LM head: at most 6 within about 200 KB.
int head_stages(int npad) {
  const size_t per = hb::tc::kAStageBytes + static_cast<size_t>(npad) * 128;
  const size_t fixed = hb::tc::head_smem_bytes(0, npad);
  return std::max(2, std::min(6, static_cast<int>((200u * 1024u - fixed) / per)));
}

struct GemmShape {
  int tiles, ksplit, kst, npad, stages;
};

GemmShape gemm_shape(int rows, int k, int n, int sms) {
  GemmShape g{};
  g.tiles = (rows + hb::tc::kTileRows - 1) / hb::tc::kTileRows;
  g.kst = k / hb::tc::kStageK;
  g.npad = hb::tc::pad_n(n);
  g.ksplit = choose_ksplit(g.tiles, g.kst, sms);
  g.stages = choose_stages(g.npad, g.ksplit, g.kst);
  return g;
}

constexpr size_t kCtrlBytes = 256;

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled from the driver the runtime loaded (no link to
// libcuda); NULL when the driver has none.
EncodeTiled encode_tiled() {
  static const EncodeTiled fn = [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    cudaGetLastError();
    return reinterpret_cast<EncodeTiled>(p);
  }();
  return fn;
}

// The GEMM's 3-D view of a packed matrix of `groups` row groups x K columns:
// 32-bit words {256 (a row group's 1 KB per 64-column stage), K / 64 stages,
// row groups}, box {256, 1, box_groups}; boxes past the last row group read
// zeros.  base is 16-byte aligned, K a multiple of 64.
bool packed_map(CUtensorMap *m, const void *base, int K, int groups, int box_groups) {
  const EncodeTiled fn = encode_tiled();
  if (!fn) return false;
  const cuuint64_t dims[3] = {256, static_cast<cuuint64_t>(K / hb::tc::kStageK), static_cast<cuuint64_t>(groups)};
  const cuuint64_t strides[2] = {hb::tc::kGroupStageBytes, static_cast<cuuint64_t>(K) * 16};
  const cuuint32_t box[3] = {256, 1, static_cast<cuuint32_t>(box_groups)};
  const cuuint32_t estride[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<void *>(base), dims, strides, box, estride,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// A launch of `kernel` that may start before the previous kernel on the
// stream completes (programmatic dependent launch: the kernel waits for it
// with griddepcontrol.wait before reading its results), the K slices of a
// GEMM tile one cluster of `cluster` CTAs.
template <typename... KArgs, typename... Args>
cudaError_t launch_early(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, int cluster,
                         Args &&...args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = static_cast<unsigned>(cluster);
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = cluster > 1 ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// One GEMM launch: tiles x ksplit CTAs, the K slices of a tile one cluster.
template <int EPI>
cudaError_t launch_gemm(const GemmShape &g, const hb::tc::GemmParams &P, cudaStream_t st) {
  return launch_early(hb::tc::gemm_kernel<EPI>, dim3(g.tiles * g.ksplit), dim3(hb::tc::kThreads),
                      hb::tc::gemm_smem_bytes(g.stages, g.npad, g.ksplit), st, g.ksplit, P);
}

// Fills P's shape fields and tensor maps for W (rows x K) times n rows of x.
bool gemm_params(hb::tc::GemmParams &P, const GemmShape &g, const void *w, int rows, int K, const void *x, int n) {
  P.rows = rows;
  P.K = K;
  P.N = n;
  P.npad = g.npad;
  P.tiles = g.tiles;
  P.ksplit = g.ksplit;
  P.kst = g.kst;
  P.stages = g.stages;
  return packed_map(&P.map_w, w, K, (rows + 7) / 8, hb::tc::kTileRows / 8) &&
         packed_map(&P.map_x, x, K, (n + 7) / 8, g.npad / 8);
}

}  // namespace

// Device buffers of the batched path, sized for kMaxRows rows and
// allocated on an engine's first batched step.
constexpr int kMaxRows = 256;
// the persistent LM head takes up to 128 output rows a launch (its
// transposed tile, 129 floats per row, must fit beside its ring)
constexpr int kHeadRows = 128;

struct hb_batch {
  int *d_meta = nullptr;            // slot [kMaxRows] | pos | tok | output rows
  int *d_argmax = nullptr;          // [kMaxRows]
  __nv_bfloat16 *h = nullptr, *h1 = nullptr, *qkv = nullptr;  // row-major [kMaxRows][*]
  uint8_t *xn = nullptr, *att = nullptr, *act = nullptr;      // packed GEMM inputs
  uint8_t *scratch = nullptr;       // Ctrl (cleared every step)
  float *part_val = nullptr;
  int *part_idx = nullptr;
  int lm_tiles = 0;
  float *logits = nullptr;          // [kMaxRows][vocab], allocated when first asked for
  int *h_meta = nullptr;            // pinned staging
  int *h_argmax = nullptr;
  hb::Ctrl *h_ctrl = nullptr;
  int sms = 0;
  // the step's launch sequence, captured once per (rows, output rows,
  // logits wanted); at most kMaxGraphs kept (all dropped when full)
  std::unordered_map<uint32_t, cudaGraphExec_t> graphs;
};

constexpr size_t kMaxGraphs = 512;
constexpr int kMetaWords = 4 * kMaxRows;

namespace {

hb::Ctrl *batch_ctrl(hb_batch *b) { return reinterpret_cast<hb::Ctrl *>(b->scratch); }

int batch_setup(hb_engine *e) {
  if (e->batch) return HB_OK;
  const hb_model_desc &d = e->desc;
  auto *b = new hb_batch();
  e->batch = b;
  cudaDeviceGetAttribute(&b->sms, cudaDevAttrMultiProcessorCount, e->device);
  const int H = d.hidden, I = d.intermediate, QKV = (d.q_heads + 2 * d.kv_heads) * d.head_dim;
  b->lm_tiles = (d.vocab + hb::tc::kTileRows - 1) / hb::tc::kTileRows;
  const size_t scratch = kCtrlBytes;
  int rc;
  if ((rc = dev_alloc(e, &b->d_meta, kMetaWords)) || (rc = dev_alloc(e, &b->d_argmax, kMaxRows)) ||
      (rc = dev_alloc(e, &b->h, static_cast<size_t>(kMaxRows) * H)) ||
      (rc = dev_alloc(e, &b->h1, static_cast<size_t>(kMaxRows) * H)) ||
      (rc = dev_alloc(e, &b->qkv, static_cast<size_t>(kMaxRows) * QKV)) ||
      (rc = dev_alloc(e, &b->xn, static_cast<size_t>(kMaxRows) * H * 2)) ||
      (rc = dev_alloc(e, &b->att, static_cast<size_t>(kMaxRows) * H * 2)) ||
      (rc = dev_alloc(e, &b->act, static_cast<size_t>(kMaxRows) * I * 2)) ||
      (rc = dev_alloc(e, &b->scratch, scratch)) ||
      (rc = dev_alloc(e, &b->part_val, static_cast<size_t>(b->lm_tiles) * kMaxRows)) ||
      (rc = dev_alloc(e, &b->part_idx, static_cast<size_t>(b->lm_tiles) * kMaxRows)))
    return rc;
  HB_CUDA(e, cudaMallocHost(reinterpret_cast<void **>(&b->h_meta), sizeof(int) * kMetaWords));
  HB_CUDA(e, cudaMallocHost(reinterpret_cast<void **>(&b->h_argmax), sizeof(int) * kMaxRows));
  HB_CUDA(e, cudaMallocHost(reinterpret_cast<void **>(&b->h_ctrl), sizeof(hb::Ctrl)));
  // opt every GEMM variant into the most shared memory any row count needs
  // (outside any stream capture)
  size_t smem = 0;
  const int shapes[5][2] = {{QKV, H}, {H, H}, {2 * I, H}, {H, I}, {d.vocab, H}};
  for (const auto &sh : shapes)
    for (int n = 16; n <= kMaxRows; n += 16) {
      const GemmShape g = gemm_shape(sh[0], sh[1], n, b->sms);
      smem = std::max(smem, hb::tc::gemm_smem_bytes(g.stages, g.npad, g.ksplit));
    }
  const void *fns[5] = {reinterpret_cast<const void *>(hb::tc::gemm_kernel<0>),
                        reinterpret_cast<const void *>(hb::tc::gemm_kernel<1>),
                        reinterpret_cast<const void *>(hb::tc::gemm_kernel<2>),
                        reinterpret_cast<const void *>(hb::tc::gemm_kernel<3>),
                        reinterpret_cast<const void *>(hb::tc::gemm_kernel<4>)};
  for (const void *fn : fns)
    HB_CUDA(e, cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  size_t head_smem = 0;
  for (int n = 16; n <= kHeadRows; n += 16) head_smem = std::max(head_smem, hb::tc::head_smem_bytes(head_stages(n), n));
  HB_CUDA(e, cudaFuncSetAttribute(hb::tc::lm_head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(head_smem)));
  return HB_OK;
}

// One tensor-core GEMM of the step: W (packed, rows x K) times the packed
// rows `x`, epilogue EPI.
template <int EPI>
int gemm(hb_engine *e, const uint8_t *w, int rows, int K, const uint8_t *x, int n, hb::tc::GemmParams P) {
  hb_batch *b = e->batch;
  const GemmShape g = gemm_shape(rows, K, n, b->sms);
  if (!gemm_params(P, g, w, rows, K, x, n)) return fail(e, HB_ERR_CUDA, "batched step: tensor map encoding failed");
  P.ctrl = batch_ctrl(b);
  P.limit_ns = e->limit_ns;
  HB_CUDA(e, launch_gemm<EPI>(g, P, e->stream));
  return HB_OK;
}

// The LM head over every vocabulary tile (persistent lm_head_kernel, one CTA
// per SM at most): FP32 logits when P.y is set, per-tile column maxima.
int lm_head(hb_engine *e, const uint8_t *w, int rows, int K, const uint8_t *x, int n, hb::tc::GemmParams P) {
  hb_batch *b = e->batch;
  GemmShape g{};
  g.tiles = (rows + hb::tc::kTileRows - 1) / hb::tc::kTileRows;
  g.kst = K / hb::tc::kStageK;
  g.npad = hb::tc::pad_n(n);
  g.ksplit = 1;
  g.stages = head_stages(g.npad);
  if (!gemm_params(P, g, w, rows, K, x, n)) return fail(e, HB_ERR_CUDA, "batched step: tensor map encoding failed");
  P.ctrl = batch_ctrl(b);
  P.limit_ns = e->limit_ns;
  HB_CUDA(e, launch_early(hb::tc::lm_head_kernel, dim3(std::min(g.tiles, b->sms)), dim3(hb::tc::kHeadThreads),
                          hb::tc::head_smem_bytes(g.stages, g.npad), e->stream, 1, P));
  return HB_OK;
}

// Enqueues the whole model over n rows on the engine's stream: row i is
// token tok[i] at position pos[i] of KV slot slot[i] (uploaded from the
// pinned h_meta; the host has checked them).  The final norm and LM head run
// over the n_out rows listed in h_meta's output-row region only (a prefill
// chunk needs one), leaving their argmax in the pinned h_argmax and the
// control block in h_ctrl.
int batch_record(hb_engine *e, int n, int n_out, bool want_logits) {
  hb_batch *b = e->batch;
  const hb_model_desc &d = e->desc;
  const int H = d.hidden, I = d.intermediate, QKV = (d.q_heads + 2 * d.kv_heads) * d.head_dim;
  const int group = d.q_heads / d.kv_heads;
  cudaStream_t st = e->stream;
  HB_CUDA(e, cudaMemsetAsync(b->scratch, 0, kCtrlBytes, st));
  HB_CUDA(e, cudaMemcpyAsync(b->d_meta, b->h_meta, sizeof(int) * kMetaWords, cudaMemcpyHostToDevice, st));
  hb::tc::Rows R{b->d_meta, b->d_meta + kMaxRows, b->d_meta + 2 * kMaxRows};
  const auto *embed = reinterpret_cast<const __nv_bfloat16 *>(e->d_blob + d.embedding);
  hb::tc::embed_norm_kernel<<<(n + 3) / 4, hb::tc::kThreads, 0, st>>>(embed, R.tok, n, e->layer_ptrs[0].gamma_in,
                                                                     d.rms_eps, H, b->h, b->xn);
  hb::tc::KvArgs A{};
  A.qkv = b->qkv;
  A.QKV = QKV;
  A.QH = d.q_heads;
  A.KVH = d.kv_heads;
  A.group = group;
  A.H = H;
  A.cos = e->d_rope_cos;
  A.sin = e->d_rope_sin;
  A.kv = e->d_kv;
  A.L = d.layers;
  A.ctx = d.context;
  const size_t att_smem = static_cast<size_t>(2) * d.context * 128 + static_cast<size_t>(group) * 512;
  // per layer: qkv (+ RoPE and K / V append), attention, o (+ residual),
  // norm, gate / up (+ SwiGLU), down (+ residual), the next layer's norm --
  // each launched early, its weights prefetched while its predecessor ends
  const dim3 norm_grid((n + 3) / 4);
  int rc;
  for (int l = 0; l < d.layers; ++l) {
    const hb::LayerPtrs &lp = e->layer_ptrs[l];
    hb::tc::GemmParams P{};
    P.bias = d.has_qkv_bias ? lp.bias : nullptr;
    P.out = b->qkv;
    A.layer = l;
    P.kv = A;
    P.R = R;
    if ((rc = gemm<hb::tc::kEpiQkv>(e, lp.w_qkv, QKV, H, b->xn, n, P))) return rc;
    HB_CUDA(e, launch_early(hb::tc::attention_kernel, dim3(n, d.kv_heads), dim3(32 * group), att_smem, st, 1, A, R,
                            b->att));
    P = hb::tc::GemmParams{};
    P.resid = b->h;
    P.out = b->h1;
    if ((rc = gemm<hb::tc::kEpiResid>(e, lp.w_o, H, H, b->att, n, P))) return rc;
    HB_CUDA(e, launch_early(hb::tc::norm_pack_kernel, norm_grid, dim3(hb::tc::kThreads), 0, st, 1,
                            static_cast<const __nv_bfloat16 *>(b->h1), static_cast<const int *>(nullptr), n,
                            lp.gamma_post, d.rms_eps, H, b->xn));
    P = hb::tc::GemmParams{};
    P.out = reinterpret_cast<__nv_bfloat16 *>(b->act);
    if ((rc = gemm<hb::tc::kEpiSwiglu>(e, lp.w_gu, 2 * I, H, b->xn, n, P))) return rc;
    P = hb::tc::GemmParams{};
    P.resid = b->h1;
    P.out = b->h;
    if ((rc = gemm<hb::tc::kEpiResid>(e, lp.w_down, H, I, b->act, n, P))) return rc;
    if (l + 1 < d.layers)
      HB_CUDA(e, launch_early(hb::tc::norm_pack_kernel, norm_grid, dim3(hb::tc::kThreads), 0, st, 1,
                              static_cast<const __nv_bfloat16 *>(b->h), static_cast<const int *>(nullptr), n,
                              e->layer_ptrs[l + 1].gamma_in, d.rms_eps, H, b->xn));
  }
  HB_CUDA(e, launch_early(hb::tc::norm_pack_kernel, dim3((n_out + 3) / 4), dim3(hb::tc::kThreads), 0, st, 1,
                          static_cast<const __nv_bfloat16 *>(b->h), static_cast<const int *>(b->d_meta + 3 * kMaxRows),
                          n_out, reinterpret_cast<const float *>(e->d_blob + d.gamma_final), d.rms_eps, H, b->xn));
  // the LM head in launches of up to 128 output rows (packed rows c0.. start
  // at row group c0 / 8 of xn)
  for (int c0 = 0; c0 < n_out; c0 += kHeadRows) {
    hb::tc::GemmParams P{};
    P.y = want_logits ? b->logits + static_cast<size_t>(c0) * d.vocab : nullptr;
    P.part_val = b->part_val + c0;
    P.part_idx = b->part_idx + c0;
    P.pstride = kMaxRows;
    const uint8_t *x = b->xn + static_cast<size_t>(c0 / 8) * H * 16;
    if ((rc = lm_head(e, e->d_blob + d.w_lm, d.vocab, H, x, std::min(kHeadRows, n_out - c0), P))) return rc;
  }
  HB_CUDA(e, launch_early(hb::tc::argmax_reduce_kernel, dim3(n_out), dim3(256), 0, st, 1,
                          static_cast<const float *>(b->part_val), static_cast<const int *>(b->part_idx), b->lm_tiles,
                          kMaxRows, b->d_argmax));
  HB_CUDA(e, cudaGetLastError());
  HB_CUDA(e, cudaMemcpyAsync(b->h_argmax, b->d_argmax, sizeof(int) * n_out, cudaMemcpyDeviceToHost, st));
  HB_CUDA(e, cudaMemcpyAsync(b->h_ctrl, b->scratch, sizeof(hb::Ctrl), cudaMemcpyDeviceToHost, st));
  return HB_OK;
}

void drop_graphs(hb_batch *b) {
  for (auto &kv : b->graphs) cudaGraphExecDestroy(kv.second);
  b->graphs.clear();
}

// One batched step: replays the captured launch sequence for (n, n_out,
// logits) -- capturing it on first use -- then waits and checks the control
// block.  A stream that cannot be captured runs the sequence directly.
int batch_forward(hb_engine *e, int n, int n_out, bool want_logits) {
  hb_batch *b = e->batch;
  cudaStream_t st = e->stream;
  const uint32_t key = static_cast<uint32_t>(n) | static_cast<uint32_t>(n_out) << 9 | (want_logits ? 1u << 18 : 0u);
  if (!b->graphs.count(key) && b->graphs.size() >= kMaxGraphs) drop_graphs(b);
  cudaGraphExec_t &exec = b->graphs[key];
  int rc = HB_OK;
  if (!exec && st != nullptr && cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
    rc = batch_record(e, n, n_out, want_logits);
    cudaGraph_t graph = nullptr;
    const cudaError_t end = cudaStreamEndCapture(st, &graph);
    if (rc == HB_OK && end == cudaSuccess && graph != nullptr &&
        cudaGraphInstantiate(&exec, graph, 0) != cudaSuccess)
      exec = nullptr;
    if (graph) cudaGraphDestroy(graph);
    cudaGetLastError();
    if (rc) return rc;
    if (end != cudaSuccess || !exec) return fail(e, HB_ERR_CUDA, "batched step: graph capture failed");
  } else if (!exec) {
    cudaGetLastError();
    if ((rc = batch_record(e, n, n_out, want_logits))) return rc;
  }
  if (exec) HB_CUDA(e, cudaGraphLaunch(exec, st));
  HB_CUDA(e, cudaStreamSynchronize(st));
  if (b->h_ctrl->err == hb::kErrTimeout)
    return fail(e, HB_ERR_DEVICE_TIMEOUT, "batched step: a device wait gave up (where %d)", b->h_ctrl->err_where);
  if (b->h_ctrl->err) return fail(e, HB_ERR_STATE, "batched step: device error %d", b->h_ctrl->err);
  return HB_OK;
}

// Checks shared by the batched entry points; makes the engine's device current.
int batch_check(hb_engine *e, int n) {
  if (!e) return fail(nullptr, HB_ERR_INVALID_ARG, "engine is NULL");
  if (!e->loaded) return fail(e, HB_ERR_STATE, "weights not loaded");
  if (e->desc.weight_format != HB_WEIGHTS_BF16)
    return fail(e, HB_ERR_UNSUPPORTED, "the batched tensor-core step needs BF16 weights");
  if (e->paged) return fail(e, HB_ERR_UNSUPPORTED, "the batched tensor-core step needs the 64-position cache");
  if (n < 1 || n > kMaxRows) return fail(e, HB_ERR_INVALID_ARG, "n must be in [1, %d]", kMaxRows);
  const hb_model_desc &d = e->desc;
  if (d.hidden % hb::tc::kStageK || d.intermediate % hb::tc::kStageK)
    return fail(e, HB_ERR_UNSUPPORTED, "hidden and intermediate must be multiples of 64");
  if (d.head_dim != hb::tc::kHeadDimTc)
    return fail(e, HB_ERR_UNSUPPORTED, "the batched step needs 64-dimension heads");
  return HB_OK;
}

}  // namespace

namespace hbi {
void batch_release(hb_engine *e) {
  hb_batch *b = e->batch;
  if (!b) return;
  void *dev[] = {b->d_meta, b->d_argmax, b->h, b->h1, b->qkv, b->xn, b->att, b->act, b->scratch,
                 b->part_val, b->part_idx, b->logits};
  for (void *p : dev)
    if (p) cudaFree(p);
  void *host[] = {b->h_meta, b->h_argmax, b->h_ctrl};
  for (void *p : host)
    if (p) cudaFreeHost(p);
  drop_graphs(b);
  delete b;
  e->batch = nullptr;
}
}  // namespace hbi

extern "C" {

size_t hb_tc_gemm_scratch_bytes(int rows, int k, int n) {
  if (rows <= 0 || k <= 0 || n <= 0) return 0;
  return kCtrlBytes;  // the control block (partial sums stay on chip)
}

int hb_tc_gemm(const void *w_dev, int rows, int k, const void *x_dev, int n, float *y_dev, void *scratch_dev,
               size_t scratch_bytes, void *stream) {
  if (!w_dev || !x_dev || !y_dev || !scratch_dev)
    return fail(nullptr, HB_ERR_INVALID_ARG, "hb_tc_gemm: null pointer");
  if (rows <= 0 || rows % 8 || k <= 0 || k % hb::tc::kStageK || n < 1 || n > hb::tc::kMaxN)
    return fail(nullptr, HB_ERR_INVALID_ARG,
                "hb_tc_gemm: rows must be a positive multiple of 8, k of 64, and 1 <= n <= 256");
  if ((reinterpret_cast<uintptr_t>(w_dev) | reinterpret_cast<uintptr_t>(x_dev) |
       reinterpret_cast<uintptr_t>(scratch_dev)) & 15)
    return fail(nullptr, HB_ERR_INVALID_ARG, "hb_tc_gemm: operands must be 16-byte aligned");
  int dev = 0, sms = 0, major = 0;
  HB_CUDA(nullptr, cudaGetDevice(&dev));
  HB_CUDA(nullptr, cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  HB_CUDA(nullptr, cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
  if (major != 10) return fail(nullptr, HB_ERR_UNSUPPORTED, "hb_tc_gemm: needs an sm_100 GPU");
  const GemmShape g = gemm_shape(rows, k, n, sms);
  if (scratch_bytes < kCtrlBytes)
    return fail(nullptr, HB_ERR_INVALID_ARG, "hb_tc_gemm: scratch needs %zu bytes", kCtrlBytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t *scr = static_cast<uint8_t *>(scratch_dev);
  HB_CUDA(nullptr, cudaMemsetAsync(scr, 0, kCtrlBytes, st));  // the control block starts clear on every call
  hb::tc::GemmParams P{};
  if (!gemm_params(P, g, w_dev, rows, k, x_dev, n))
    return fail(nullptr, HB_ERR_CUDA, "hb_tc_gemm: tensor map encoding failed");
  P.y = y_dev;
  P.ctrl = reinterpret_cast<hb::Ctrl *>(scr);
  P.limit_ns = kDefaultLimitNs;
  const size_t smem = hb::tc::gemm_smem_bytes(g.stages, g.npad, g.ksplit);
  HB_CUDA(nullptr, cudaFuncSetAttribute(hb::tc::gemm_kernel<hb::tc::kEpiF32>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  HB_CUDA(nullptr, launch_gemm<hb::tc::kEpiF32>(g, P, st));
  return HB_OK;
}

int hb_step_rows(hb_engine *e, int n, const int32_t *slots, const int32_t *token_ids, const int32_t *positions,
                 int n_out, const int32_t *out_rows, int32_t *argmax_out, float *logits_out) {
  int rc = batch_check(e, n);
  if (rc) return rc;
  DeviceScope device_scope_(e->device);
  if (!device_scope_.ok) return fail(e, HB_ERR_CUDA, "cudaSetDevice(%d) failed", e->device);
  if (!slots || !token_ids || !positions) return fail(e, HB_ERR_INVALID_ARG, "rows are NULL");
  if (out_rows ? (n_out < 1 || n_out > n) : n_out != n)
    return fail(e, HB_ERR_INVALID_ARG, "n_out must be in [1, n] with out_rows, n without");
  const hb_model_desc &d = e->desc;
  for (int i = 0; i < n; ++i) {
    if (slots[i] < 0 || slots[i] >= d.max_slots)
      return fail(e, HB_ERR_INVALID_ARG, "row %d: slot %d outside [0, %d)", i, slots[i], d.max_slots);
    if (token_ids[i] < 0 || token_ids[i] >= d.vocab)
      return fail(e, HB_ERR_INVALID_ARG, "row %d: token id %d outside the vocabulary", i, token_ids[i]);
    if (positions[i] < 0 || positions[i] >= d.context)
      return fail(e, HB_ERR_INVALID_ARG, "row %d: position outside the %d-token context", i, d.context);
    for (int k = 0; k < i; ++k)
      if (slots[k] == slots[i] && positions[k] == positions[i])
        return fail(e, HB_ERR_INVALID_ARG, "rows %d and %d write the same slot position", k, i);
  }
  for (int i = 0; out_rows && i < n_out; ++i)
    if (out_rows[i] < 0 || out_rows[i] >= n)
      return fail(e, HB_ERR_INVALID_ARG, "output row %d: %d outside [0, %d)", i, out_rows[i], n);
  if ((rc = batch_setup(e))) return rc;
  hb_batch *b = e->batch;
  if (logits_out && !b->logits && (rc = dev_alloc(e, &b->logits, static_cast<size_t>(kMaxRows) * d.vocab)))
    return rc;
  for (int i = 0; i < n; ++i) {
    b->h_meta[i] = slots[i];
    b->h_meta[kMaxRows + i] = positions[i];
    b->h_meta[2 * kMaxRows + i] = token_ids[i];
  }
  for (int i = 0; i < n_out; ++i) b->h_meta[3 * kMaxRows + i] = out_rows ? out_rows[i] : i;
  if ((rc = batch_forward(e, n, n_out, logits_out != nullptr))) return rc;
  if (argmax_out)
    for (int i = 0; i < n_out; ++i) argmax_out[i] = b->h_argmax[i];
  if (logits_out)
    HB_CUDA(e, cudaMemcpy(logits_out, b->logits, sizeof(float) * n_out * d.vocab, cudaMemcpyDeviceToHost));
  return HB_OK;
}

int hb_prefill_tc(hb_engine *e, int slot, const int32_t *ids, int n, int start_pos, float *last_logits,
                  int32_t *argmax_out) {
  if (!ids || n < 1) return fail(e, HB_ERR_INVALID_ARG, "ids must hold at least one token");
  std::vector<int32_t> slots(kMaxRows, slot), pos(kMaxRows);
  int rc = HB_OK;
  for (int done = 0; done < n && rc == HB_OK;) {
    const int m = std::min(kMaxRows, n - done);
    for (int i = 0; i < m; ++i) pos[i] = start_pos + done + i;
    const bool last = done + m == n;
    const int32_t out_row = m - 1;  // only the chunk's last position reaches the LM head
    int32_t am = 0;
    rc = hb_step_rows(e, m, slots.data(), ids + done, pos.data(), 1, &out_row, &am,
                      last ? last_logits : nullptr);
    if (rc == HB_OK && last && argmax_out) *argmax_out = am;
    done += m;
  }
  return rc;
}

int hb_tc_gemm_status(const void *scratch_dev, void *stream) {
  if (!scratch_dev) return fail(nullptr, HB_ERR_INVALID_ARG, "hb_tc_gemm_status: null scratch");
  hb::Ctrl c{};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  HB_CUDA(nullptr, cudaMemcpyAsync(&c, scratch_dev, sizeof(c), cudaMemcpyDeviceToHost, st));
  HB_CUDA(nullptr, cudaStreamSynchronize(st));
  if (c.err == hb::kErrTimeout)
    return fail(nullptr, HB_ERR_DEVICE_TIMEOUT, "hb_tc_gemm: a device wait gave up (where %d)", c.err_where);
  return c.err ? fail(nullptr, HB_ERR_STATE, "hb_tc_gemm: device error %d", c.err) : HB_OK;
}

}  // extern "C"
