// spt_internal.cuh -- device data layout and kernel launchers shared by the
// C ABI (spt_api.cu) and the kernels (spt_kernels.cu).
//
// HBM layout of one expert matrix in the GEMV arena ("G8" layout)
// --------------------------------------------------------------
// A GGUF MXFP4 expert tensor is E experts x R rows x nb 17-byte blocks
// (ggufindex/index.go:550, forward/mxfp4.go:56-59: byte 0 = E8M0 scale,
// byte 1+i holds element i in its low nibble and element i+16 in its high
// nibble).  17-byte blocks are not 16-byte aligned, so the arena repacks them
// once into two planes:
//
//   nibbles: uint4 nib[E][G][NQ][32]  G = ceil(R/8) row groups, NQ = ceil(nb/4)
//            lane l = 4*i + q of a warp owns row 8g+i and "chain quarter" q;
//            the 16 bytes are four 32-bit words, word t = block 4*Q+t, and
//            nibble j of a word is element 8q+j of that block.
//   scales:  uint32 scl[E][G][NQ][8]  byte t of word i = E8M0 byte of block
//            4*Q+t of row 8g+i.
//
// One warp-wide 16-byte load reads 512 contiguous bytes = 4 blocks of 8 rows.
// Thread (i,q) then holds exactly the 8 FMA chains 8q..8q+7 of the
// reference's AVX2 dot (forward/mxfp4_amd64.go:11-26): accumulator register
// a_q of that kernel, lane by lane.
#pragma once
#include <atomic>
#include <utility>
#include <cuda_runtime.h>
#include <stdint.h>

#include "spt_gemv16.cuh"
#include "spt_mma.cuh"

namespace spt {

constexpr int kDispatchMaxExperts = 256;  // shared-memory tables of the dispatch kernel
constexpr int kSelectMaxK = 32;

struct MatrixG8 {
  const uint4 *nib = nullptr;     // [E][G][NQ][32]
  const uint32_t *scl = nullptr;  // [E][G][NQ][8]
  int rows = 0;                   // R
  int blocks = 0;                 // nb = K/32
  int groups = 0;                 // G
  int quads = 0;                  // NQ
};

inline size_t g8_nib_count(int64_t experts, int rows, int blocks) {
  return (size_t)experts * (size_t)((rows + 7) / 8) * (size_t)((blocks + 3) / 4) * 32;
}
inline size_t g8_scl_count(int64_t experts, int rows, int blocks) {
  return (size_t)experts * (size_t)((rows + 7) / 8) * (size_t)((blocks + 3) / 4) * 8;
}

// Device pointers of one layer in the arena.
struct LayerDev {
  const float *router = nullptr;       // [E][H] fp32
  const float *router_bias = nullptr;  // [E]
  MatrixG8 gate, up, down;             // gate/up: R = D, K = H; down: R = H, K = D
  const float *gate_bias = nullptr;    // [E][D]
  const float *up_bias = nullptr;      // [E][D]
  const float *down_bias = nullptr;    // [E][H]
  bool has_g8 = false;                 // CUDA-core GEMV planes present
  bool has_mma = false;                // tcgen05 planes present
  MmaMatrix gu_mma, dn_mma;            // gate/up interleaved [E][2D][KP/2]; down [E][H][KPd/2]
  bool gemv16_ok = false;              // every scale byte in [kF16ScaleLo, kF16ScaleHi] (decode GEMV usable)
  const float *norm = nullptr;         // post-attention RMSNorm weight [H] (layer stack), or null
};

// Per-call device scratch (owned by the context, grown on demand).
struct ScratchDev {
  float *logits = nullptr;      // [T][E]
  int32_t *sel_idx = nullptr;   // [T*K]
  float *sel_w = nullptr;       // [T*K]
  int32_t *offsets = nullptr;   // [E+1] expert segment starts in dispatch order
  int32_t *perm = nullptr;      // [T*K] dispatch position -> slot
  int32_t *slot_pos = nullptr;  // [T*K] slot -> dispatch position, -1 if not dispatched
  int32_t *act_list = nullptr;  // [E] active experts ascending
  int32_t *meta = nullptr;      // [0] active experts, [1] dispatched slots
  float *act = nullptr;         // [T*K][D] SwiGLU activations in dispatch order
  float *res = nullptr;         // [T*K][H] down + bias in dispatch order
};

struct Dims {
  int H, D, E, K;
};

// ---- launchers (spt_kernels.cu); all enqueue on `stream` ----------------

// Optional output of the router launch: the decode GEMV's split operand of
// the T input rows (token order, [T][2][kp] halves) and their exponents,
// made from the rows the shared-memory router stages anyway.  *split_done
// tells whether this launch wrote them (else the caller runs
// launch_split_rows).
struct RouterSplit {
  __half *xq = nullptr;
  int32_t *xe = nullptr;
  int kp = 0;
};
// normBatch (8 lanes) applied to the router's input first: out = rows of
// (x * w) * f, f = 1/float32(sqrt(float64(sum(x^2)/dim + eps))).  Folded into
// the router's prologue when it stages its rows in shared memory (and then
// written out by the router's CTAs for the expert kernels), else a separate
// k_rmsnorm launch before the router; either way the router reads the
// normalised rows and `out` holds them afterwards.
struct RouterNorm {
  const float *w = nullptr;
  float eps = 0.0f;
  float *out = nullptr;
};
cudaError_t launch_select(const float *logits, int T, int E, int K, int32_t *sel_idx,
                          float *sel_w, cudaStream_t stream);
// Tensor-core tile layout computed by the dispatch kernel (bn = 0: none).
struct DispatchPlan {
  int bn = 0, mt_gu = 0, mt_dn = 0;  // tokens per tile, row tiles per expert
  int32_t *pad_off = nullptr;        // [E] first 128-row activation slot
  int32_t *tile_gu = nullptr;        // [E+1] gate/up tile prefix over active experts
  int32_t *tile_dn = nullptr;        // [E+1] down tile prefix
  int32_t *pos_expert = nullptr;     // [S] expert of each dispatch position
  // [E+1] first dispatch position of each active expert (act_off[i] =
  // offsets[act_list[i]]; the entry after the last active expert is the
  // dispatched count), written whenever non-null (bn may be 0)
  int32_t *act_off = nullptr;
};
cudaError_t launch_dispatch(const int32_t *sel_idx, const float *sel_w, int S, int E,
                            int32_t *offsets, int32_t *perm, int32_t *slot_pos,
                            int32_t *act_list, int32_t *meta, cudaStream_t stream,
                            const DispatchPlan *plan = nullptr, int key_div = 1);
// Top-k selection fused into the dispatch CTA (one device, T <= the limit):
// writes sel_idx / sel_w as launch_select does, then dispatches as above, one
// launch fewer.  Measured on B200 (GPT-OSS layer): T=1 0.8 us faster per
// block; T=32 and T=64 about 1% slower (the selection then sits serially in
// the one dispatch CTA), hence the small limit.
constexpr int kSelectDispatchMaxTokens = 8;
// The context option SPT_OPT_FUSED_SELECT = 0 keeps the separate selection
// launch (same results).
cudaError_t launch_select_dispatch(const float *logits, int T, int E, int K, int32_t *sel_idx, float *sel_w,
                                   int32_t *offsets, int32_t *perm, int32_t *slot_pos, int32_t *act_list,
                                   int32_t *meta, cudaStream_t stream, const DispatchPlan *plan = nullptr);
// Top-k selection and dispatch run by the shared-memory router's last CTA
// (T <= kRouterDispatchMaxTokens, one device): every CTA
// counts itself in *count after writing its logits, and the one that brings
// it to the grid size resets it to 0 and does what launch_select_dispatch
// does, reading the logits through L2.  One launch fewer again.
// Measured on B200 (GPT-OSS layer, c1 T = 32): 234.4 us per block with the
// 32 selections serial in the router's last CTA against 229.8 us with the
// separate selection and dispatch launches, hence decode batches only.
constexpr int kRouterDispatchMaxTokens = 8;
struct RouterDispatch {
  int32_t *sel_idx = nullptr;
  float *sel_w = nullptr;
  int32_t *offsets = nullptr, *perm = nullptr, *slot_pos = nullptr, *act_list = nullptr, *meta = nullptr;
  DispatchPlan plan;
  int topk = 0;
  unsigned *count = nullptr;  // zero between launches
};
// *dispatch_done (optional) tells whether the launch also selected and
// dispatched (only the shared-memory router can).  With err (the context's
// device error flag) the shared-memory router stages its rows with bulk
// copies on an mbarrier whose bounded wait records code 9 there; without it,
// with cp.async.
cudaError_t launch_router(const float *W, const float *x, const float *bias, int T, int H, int E,
                          float *logits, int portable_lanes, cudaStream_t stream,
                          const RouterSplit *split = nullptr, bool *split_done = nullptr,
                          const RouterNorm *norm = nullptr, int *launches = nullptr,
                          const RouterDispatch *dispatch = nullptr, bool *dispatch_done = nullptr,
                          int32_t *err = nullptr, int wait_shift = 31, int fault_stage = -1);
// SPT_OPT_FAULT_STAGE value that makes the shared-memory router's bounded
// wait run out (test hook; the tcgen05 stages are small numbers).
constexpr int kRouterFault = 1000;
// Expert-parallel helpers: gather the send rows (token of slot perm[p], local
// expert id sel_idx % experts_per_rank) for the meta[1] dispatched slots;
// per-rank row counts from the rank offsets; fill a float array.
cudaError_t launch_ep_gather(const float *x, const int32_t *sel_idx, const int32_t *perm, const int32_t *meta,
                             int K, int experts_per_rank, int H, int S, float *xs, int32_t *ms,
                             cudaStream_t stream);
cudaError_t launch_ep_counts(const int32_t *offsets, int world, int32_t *counts, cudaStream_t stream);
// Fixed-capacity exchange layout: rows for rank r at [r*cap, r*cap + count).
cudaError_t launch_ep_gather_cap(const float *x, const int32_t *sel_idx, const int32_t *perm, const int32_t *offsets,
                                 const int32_t *meta, int K, int experts_per_rank, int H, int S, int world, int cap,
                                 float *xs, int32_t *ms, int32_t *counts, int32_t *slot_pos, cudaStream_t stream);
cudaError_t launch_ep_recv_weights(const int32_t *counts, int cap, int world, float *w, cudaStream_t stream);

// Peer-memory exchange of the fixed-capacity layout (one GPU per rank).  The
// window of every rank, at the same byte offsets (base[r] = rank r's window as
// mapped in this process):
//   rows [2][world][cap][hidden] f32  token rows sent here, [call parity][sender][j]
//   ret  [2][world][cap][hidden] f32  result rows of this rank's slots, [parity][owner][j]
//   ids  [2][world][cap] i32          local expert id of each row in `rows`
//   cnt  [2][world] i32               rows each sender sent here
//   ffwd [world] u64, fret [world] u64  last call (sequence number) whose rows /
//                                     results from each rank have landed
constexpr int kEpMaxPeers = 32;
struct EpPeerLayout {
  uint8_t *base[kEpMaxPeers];
  int64_t rows_off = 0, ret_off = 0, ids_off = 0, cnt_off = 0, ffwd_off = 0, fret_off = 0, bytes = 0;
  int world = 1, rank = 0, cap = 0, hidden = 0;
};
cudaError_t launch_ep_send_peer(const float *x, const int32_t *sel_idx, const int32_t *perm, const int32_t *offsets,
                                const int32_t *meta, int K, int experts_per_rank, int S, const EpPeerLayout &L, int par,
                                uint64_t seq, int32_t *slot_pos, int32_t *arrive, cudaStream_t stream);
cudaError_t launch_ep_return_peer(const float *rows_out, const EpPeerLayout &L, int par, uint64_t seq, int32_t *arrive,
                                  cudaStream_t stream);
// bounded wait (about 2^shift clocks) for every rank's flag at flag_off to reach
// seq; on timeout *err = code
cudaError_t launch_ep_wait(const EpPeerLayout &L, int64_t flag_off, uint64_t seq, int shift, int32_t *err, int code,
                           cudaStream_t stream);
cudaError_t launch_ep_recv_weights_peer(const EpPeerLayout &L, int par, float *w, cudaStream_t stream);
cudaError_t launch_fill(float *p, int64_t n, float v, cudaStream_t stream);

// Addressing of the token rows a GEMV launch reads and writes, per
// dispatch position p of an expert segment:
//   kRowsMoEGateUp: x row = perm[p] / K (token), y row = p
//   kRowsMoEDown:   x row = p,                    y row = p
//   kRowsOffsets:   x at xoff[p], y at yoff[p] (element offsets)
enum RowMode : int { kRowsMoEGateUp = 0, kRowsMoEDown = 1, kRowsOffsets = 2 };

struct GemvLaunch {
  MatrixG8 m0, m1;             // m1 used only when gate_up
  const float *bias0 = nullptr;  // [E][R] or null
  const float *bias1 = nullptr;
  const float *x = nullptr;
  float *y = nullptr;
  int64_t x_stride = 0;         // elements per x row (modes 0, 1)
  int64_t y_stride = 0;         // elements per y row (modes 0, 1)
  const int32_t *perm = nullptr;
  const int64_t *xoff = nullptr;  // mode 2
  const int64_t *yoff = nullptr;
  const int32_t *offsets = nullptr;   // [E+1]
  const int32_t *act_list = nullptr;  // [E]
  const int32_t *meta = nullptr;      // meta[0] = active experts
  int top_k = 1;
  int mode = kRowsMoEGateUp;
  bool gate_up = false;         // fused gate+up+SwiGLU (writes SwiGLU(act))
  int max_active = 1;           // host upper bound of active experts (grid sizing)
  int mt = 1;                   // tokens per pass (1, 2, 4, 8)
};
cudaError_t launch_gemv(const GemvLaunch &a, int sm_count, cudaStream_t stream);

// out[t] = sum over ranks of fma(res[slot], w, .) (+ resid[t] when given;
// out may alias resid).
cudaError_t launch_combine(const float *res, const float *sel_w, const int32_t *slot_pos, int T,
                           int K, int H, float *out, cudaStream_t stream, const float *resid = nullptr);
cudaError_t launch_swiglu(const float *g, const float *u, float *act, int64_t n,
                          cudaStream_t stream);
cudaError_t launch_rmsnorm(const float *x, const float *w, int T, int dim, float eps, float *y,
                           int lanes, cudaStream_t stream);
cudaError_t launch_add(float *dst, const float *src, int64_t n, cudaStream_t stream);

// Repack `experts` x `rows` x `blocks` GGUF MXFP4 blocks (device bytes) into
// the G8 planes (which must be zeroed beforehand).
cudaError_t launch_repack_g8(const uint8_t *gguf, int64_t experts, int rows, int blocks,
                             uint4 *nib, uint32_t *scl, cudaStream_t stream);
// Generate synthetic MXFP4 blocks of experts [first_expert, first_expert +
// experts) straight into the G8 planes (expert 0 of the planes = first_expert).
cudaError_t launch_synth_g8(uint64_t seed, uint32_t tag, int64_t first_expert, int64_t experts, int rows,
                            int blocks, uint8_t scale_lo, uint8_t scale_hi, uint4 *nib, uint32_t *scl,
                            cudaStream_t stream);

// Raise a kernel's dynamic shared-memory limit once per device (the setting
// belongs to the device context that is current when it is made).  The
// record is keyed by the kernel's address: template instances share one C++
// type, and each needs its own attribute.
cudaError_t opt_in_smem_raw(const void *kernel, int bytes);
template <typename Kernel>
cudaError_t opt_in_smem(Kernel kernel, int bytes) {
  return opt_in_smem_raw(reinterpret_cast<const void *>(kernel), bytes);
}

// Launch a kernel that begins with pdl_wait(); pdl_launches_enabled() (the
// SPT_PDL environment variable, default on) decides whether it may overlap
// the tail of the previous kernel on the stream.
bool pdl_launches_enabled();
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_launches_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Q8_0 GEMV + argmax (spt_q80.cu): y[r] = dot(row r, x) for `rows` rows of
// input/32 34-byte blocks, w in the packed four-row-group layout that
// launch_q80_repack writes (q80_packed_bytes long, zeroed before the repack);
// best = packed argmax key, decoded into argmax/logit (either may be null).
cudaError_t launch_q80(const uint8_t *w, int64_t rows, int input, const float *x, float *y,
                       unsigned long long *best, int64_t *argmax, float *logit, int32_t *err, int sm_count,
                       cudaStream_t stream);
cudaError_t launch_q80_repack(const uint8_t *raw, int64_t rows, int input, uint8_t *packed, cudaStream_t stream);
uint64_t q80_packed_bytes(int64_t rows, int input);
int q80_rows_per_chunk(int input);

// Q4_0 products (spt_q40.cu): y[item][r] = dot(row r, x[item]) for `rows`
// rows of input/32 18-byte blocks (w padded by >= 16 bytes), batch 1 in the
// reference's one-input order, larger batches in its batched order.
cudaError_t launch_q40(const uint8_t *w, int64_t rows, int input, const float *x, int64_t batch, float *y,
                       int32_t *err, int sm_count, cudaStream_t stream);
bool q40_supported(int input);
size_t q40_smem_bytes(int input);

}  // namespace spt
