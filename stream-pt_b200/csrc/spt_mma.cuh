// spt_mma.cuh -- tcgen05 block-scaled grouped GEMM for the MoE experts.
//
// D[rows, tokens] = W[rows, K] x X[tokens, K]^T per (expert, 128-row tile,
// token tile), accumulated in fp32 in TMEM.  A = the GGUF MXFP4 weights (e2m1
// with the GGUF E8M0 block scales, fed to the tensor core unchanged); B = the
// activations written as a sum of block-scaled terms (see k_quantize_act), so
// that block outputs stay well inside the 1e-3 relative tolerance:
//   token tiles of 8 or 16 (decode):  kind::mxf4, kFp4Terms e2m1 terms
//     stacked along N (N = kFp4Terms*BN), both operands packed 4-bit in
//     shared memory;
//   128-token tiles (prefill):      kind::mxf4, kFp4Terms e2m1 terms, one
//     N = 128 MMA per term into the same accumulator, both operands packed
//     (ActFmt::kFp4Planes, the default); or kind::mxf8f6f4 with kActTerms
//     e4m3 terms, the weights unpacked to one byte per element by the TMA
//     (16U4_ALIGN16B) (ActFmt::kFp8Planes, the context option
//     SPT_OPT_PREFILL_FP8).
// Decode-sized tiles are bound by the weight stream: packed 4-bit weights need
// half the shared memory per K tile, so the ring keeps twice as many bytes in
// flight from HBM.
//
// HBM layout of the MMA arena (one layer):
//   gu_w   uint8 [E][2D/128][KP/128][128][64]  tile-major packed e2m1: one
//                                128-row x 128-element box is one contiguous
//                                8 KB block (row r of the box at r*64, element
//                                k of the row at byte k/2, low nibble for even
//                                k); gate/up rows interleaved (row 2d = gate
//                                d, row 2d+1 = up d); KP = K rounded up to 128
//                                (4-bit TMA boxes are 128 wide), pads zero
//   gu_sf  uint8 [E][2D/128][KP/128][512]  E8M0 scales in the tensor core's
//                                scale-factor atom: row m of the tile, block
//                                kb of the K tile at (m%32)*16 + (m/32)*4 + kb
//   dn_w   uint8 [E][ceil(H/128)][KPd/128][128][64], dn_sf [E][ceil(H/128)][KPd/128][512]
// Activations (per call), K-tile-major plus scale atoms.  Every BN-token tile
// owns one 128-row slot starting at pad_off[e] + (j/BN)*128 for token j of
// expert e, so its scale atom starts at slot row 0.
//   kFp4Stack:  term t, token j at slot row t*BN + j%BN; q [KP/128][RB][64],
//               sf [RB/128][KP/128][512].
//   kFp4Planes: q [KP/128][kFp4Terms][RB][64], sf [RB/128][KP/128][kFp4Terms][512].
//   kFp8Planes: q [KP/128][kActTerms][RB][128], sf [RB/128][KP/128][kActTerms][512].
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace spt {

constexpr int kMmaM = 128;       // rows per tile (tcgen05 M for cta_group::1)
constexpr int kMmaKT = 128;      // K elements per pipeline stage (one TMA box)
constexpr int kActTerms = 3;     // e4m3 terms of the activations (128-token tiles)
// e2m1 terms of the activations (tiles of <= 16 tokens).  Four keep the
// GPT-OSS block within max-rel 4.5e-4 and 1 - cos 5e-8 of the fp32 oracle
// (the tolerance is 1e-3 and 1e-5); six (about 1e-5) cost 2.5-7% more time,
// every stage carrying 12 KB of activation terms instead of 8 KB.
constexpr int kFp4Terms = 4;
constexpr int kMmaStageTilesFp4 = 4;  // K tiles per pipeline stage, FP4 mode
// 8-token tiles with at least two row tiles per SM: six K tiles per stage
// (three stages in the ring, fewer copy operations per byte); measured on
// B200: c1 +2 %, c4 +2.6 %, but c0 (one or two tiles per SM) -4 %.
constexpr int kMmaStageTilesWide = 6;
// 128-token tiles: each CTA unit covers this many 128-row weight tiles of
// one expert against one token tile, so every activation K tile it loads
// (all terms: 32 KB of e2m1 or 48 KB of e4m3) feeds three row tiles' MMAs
// instead of one; the shared-memory and TMEM copy traffic per output falls
// by about half.
constexpr int kPrefillRowTiles = 3;
// Units of one token tile: row tiles, or groups of kPrefillRowTiles of them.
inline int mma_row_units(int bn, int mtiles) {
  return bn == 128 ? (mtiles + kPrefillRowTiles - 1) / kPrefillRowTiles : mtiles;
}

struct MmaMatrix {
  uint8_t *w = nullptr;      // packed e2m1 rows
  uint8_t *sf = nullptr;     // scale-factor atoms
  int rows = 0;              // rows per expert (2D for gate/up, H for down)
  int k = 0;                 // logical K
  int kp = 0;                // K padded to 128
  int mtiles = 0;            // ceil(rows/128)
  int64_t experts = 0;
  alignas(64) CUtensorMap tmap;    // 2D [128 elements, boxes*128 rows] 16U4_ALIGN16B, box 128x128, SW128 (unpacked)
  alignas(64) CUtensorMap tmap_p;  // 3D [64 B, 128 rows, boxes] UINT8, box 64x128xkMmaStageTilesFp4, SW64 (packed)
  alignas(64) CUtensorMap tmap_p1; // same, one box
  alignas(64) CUtensorMap tmap_pw; // same, kMmaStageTilesWide boxes
  // 128-token tiles: one K tile of kPrefillRowTiles consecutive row tiles in
  // one copy each -- 4D [128 elements, 128 rows, K tiles, row tiles]
  // 16U4_ALIGN16B (unpacked, SW128; kFp8Planes) or 4D [64 B, 128 rows, K
  // tiles, row tiles] UINT8 (packed, SW64; kFp4Planes), and their scale
  // atoms, 3D [128 words, K tiles, row tiles] UINT32
  alignas(64) CUtensorMap tmap_g;
  alignas(64) CUtensorMap tmap_gp;
  alignas(64) CUtensorMap tmap_sfg;
};

// Per-call operands of one grouped GEMM launch.  Every copy operation costs
// the SM's copy engine about the same time whatever its size, so a pipeline
// stage moves `ks` K tiles of weights, activations (all terms) and scales in
// four operations; the `*1` maps move the single K tile left at the end of a
// tile when K/128 is odd.
struct MmaLaunch {
  alignas(64) CUtensorMap tmap_a;   // weights, ks boxes
  alignas(64) CUtensorMap tmap_a1;  // weights, 1 box
  alignas(64) CUtensorMap tmap_b;   // activations, ks K tiles x all terms
  alignas(64) CUtensorMap tmap_b1;  // activations, 1 K tile x all terms
  alignas(64) CUtensorMap tmap_sfa; // scale atoms of a row-tile group (MmaMatrix::tmap_sfg), 128-token tiles
  int ks = 1;                       // K tiles per pipeline stage
  const uint8_t *w = nullptr;        // packed weights (tile-major), for L2 prefetch
  const uint8_t *sfa = nullptr;
  const uint8_t *sfb = nullptr;
  int rows = 0, kp = 0, mtiles = 0, ktiles = 0;
  int rb = 0;                        // activation rows per term (multiple of 128)
  const int32_t *offsets = nullptr;  // [E+1] dispatch segment starts
  const int32_t *pad_off = nullptr;  // [E] padded activation row of each segment
  const int32_t *act_list = nullptr; // [E] active experts
  const int32_t *tile_off = nullptr; // [E+1] tile prefix over active experts
  const int32_t *meta = nullptr;     // [0] active experts
  int max_tiles = 0;                 // host upper bound of tiles (grid sizing)
  // epilogue
  int mode = 0;                      // 0: gate/up + SwiGLU -> act[pos][D]; 1: down -> y[pos][H]
  const float *bias0 = nullptr;      // gate bias [E][D] or down bias [E][H]
  const float *bias1 = nullptr;      // up bias [E][D]
  float *y = nullptr;
  int y_stride = 0;                  // D (mode 0) or H (mode 1)
  int out_rows = 0;                  // D (mode 0) or H (mode 1)
  int32_t *err = nullptr;            // set nonzero when a bounded wait gives up
  int prefetch = 0;                  // whole weight tiles prefetched into L2 ahead (0: off)
  int wait_shift = 31;               // bounded waits give up after ~2^wait_shift clocks
  int fault_stage = -1;              // failure injection (tests): CTA 0's producer skips this stage
};

// Activation operand formats.  Token tiles of 8 or 16 tokens: kFp4Stack
// (kFp4Terms e2m1 terms stacked along N, kMmaStageTilesFp4 K tiles per
// stage); 128-token tiles: kFp4Planes (kFp4Terms e2m1 terms, one plane and
// one N = 128 MMA each) or kFp8Planes (kActTerms e4m3 terms), one K tile per
// stage.  launch_mma_gemm takes bn 8, 16 or 128.
enum class ActFmt { kFp4Stack, kFp4Planes, kFp8Planes };
inline ActFmt mma_act_fmt(int bn, bool fp8_prefill) {
  return bn <= 16 ? ActFmt::kFp4Stack : fp8_prefill ? ActFmt::kFp8Planes : ActFmt::kFp4Planes;
}
inline bool mma_fp4(ActFmt f) { return f != ActFmt::kFp8Planes; }
inline int mma_terms(ActFmt f) { return f == ActFmt::kFp8Planes ? kActTerms : kFp4Terms; }
// K tiles per stage for bn-token tiles when a launch has up to max_tiles row
// tiles on sm_count SMs.
inline int mma_stage_tiles(int bn, int64_t max_tiles = 0, int sm_count = 148) {
  if (bn > 16) return 1;
  return (bn == 8 && max_tiles >= 2 * (int64_t)sm_count) ? kMmaStageTilesWide : kMmaStageTilesFp4;
}
// Activation rows of one TMA box (per term plane for the plane formats).
inline int mma_box_rows(ActFmt f, int bn) { return f == ActFmt::kFp4Stack ? kFp4Terms * bn : bn; }
// Bytes of the activation buffers for rb rows per term and kp padded K.
inline size_t mma_act_bytes(ActFmt f, int rb, int kp) {
  return f == ActFmt::kFp4Stack    ? (size_t)rb * (kp / 2)
         : f == ActFmt::kFp4Planes ? (size_t)kFp4Terms * rb * (kp / 2)
                                   : (size_t)kActTerms * rb * kp;
}
inline size_t mma_act_sf_bytes(ActFmt f, int rb, int kp) {
  return (size_t)(f == ActFmt::kFp4Stack ? 1 : mma_terms(f)) * (rb / kMmaM) * (kp / kMmaKT) * 512;
}

size_t mma_w_bytes(int64_t experts, int rows, int k);
size_t mma_sf_bytes(int64_t experts, int rows, int k);

// Encode the TMA map of a packed e2m1 matrix (returns false on failure).
bool mma_encode_weights(MmaMatrix *m);
// TMA map of the activations in format f: kFp4Stack [kt][rb][64 B] with box
// 64 B x kFp4Terms*bn rows x ktiles (SW64); kFp4Planes [kt][kFp4Terms][rb][64 B]
// with box 64 B x bn rows x kFp4Terms x ktiles (SW64); kFp8Planes
// [kt][kActTerms][rb][128 B] with box 128 B x bn rows x kActTerms x ktiles (SW128).
bool mma_encode_acts(CUtensorMap *map, uint8_t *q, int kp, int rb, int bn, ActFmt f, int ktiles);

cudaError_t launch_repack_mma_gu(const uint8_t *gate_gguf, const uint8_t *up_gguf, int64_t experts,
                                 int D, int K, MmaMatrix *m, cudaStream_t s);
cudaError_t launch_repack_mma(const uint8_t *gguf, int64_t experts, int rows, int K, MmaMatrix *m,
                              cudaStream_t s);
// Synthetic weights of experts [first_expert, first_expert + experts) (the
// Philox counters continue from first_expert, so a shard holds the same bytes
// as the same experts of a full arena).
cudaError_t launch_synth_mma_gu(uint64_t seed, uint32_t tag_gate, uint32_t tag_up, int64_t first_expert,
                                int64_t experts, int D, int K, uint8_t lo, uint8_t hi, MmaMatrix *m,
                                cudaStream_t s);
cudaError_t launch_synth_mma(uint64_t seed, uint32_t tag, int64_t first_expert, int64_t experts, int rows,
                             int K, uint8_t lo, uint8_t hi, MmaMatrix *m, cudaStream_t s);

// Quantize T token rows to the activation terms of format f, each row once,
// stored at every dispatch position of the token (slot_pos[t*top_k + r], -1:
// not dispatched).
cudaError_t launch_quantize_tokens(const float *x, int64_t stride, int T, int top_k, const int32_t *slot_pos,
                                   const int32_t *offsets, const int32_t *pad_off, const int32_t *pos_expert, int K,
                                   int kp, int rb, int bn, ActFmt f, uint8_t *q, uint8_t *sf, cudaStream_t s);
// The same per dispatch position p, source row src[(gather ? perm[p]/top_k :
// p) * src_stride + k].
cudaError_t launch_quantize_act(const float *src, int64_t src_stride, const int32_t *perm, int top_k,
                                bool gather, const int32_t *offsets, const int32_t *pad_off,
                                const int32_t *pos_expert, const int32_t *meta, int S_max, int K,
                                int kp, int rb, int bn, ActFmt f, uint8_t *q, uint8_t *sf, cudaStream_t s);

cudaError_t launch_mma_gemm(const MmaLaunch &a, int bn, ActFmt f, int sm_count, cudaStream_t s);

}  // namespace spt
