// Shared declarations between the kernel translation unit and the C ABI.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

namespace fav {

constexpr int kTileM = 128;       // GEMM rows (time steps) per CTA tile
constexpr int kKBlock = 64;       // K elements (channels) per pipeline stage
constexpr int kLatentChannels = 64;
constexpr int kStemChannels = 2048;
constexpr int kFinalChannels = 32;
constexpr int kStages = 6;
constexpr int kRates[kStages] = {8, 6, 5, 2, 2, 2};
constexpr int kDilations[3] = {1, 3, 9};
constexpr int kHop = 1920;
constexpr int kNumHistories = 26;

// Causal history of one stream ("slot"), the reference's 26 histories
// (647,424 bytes of window) kept as rings: history L (H_L rows x C_L channels)
// owns 2*H_L rows at ring offset 2*off_L floats; its window is the H_L rows
// starting at ring row head_L (mod 2*H_L). A step reads heads from one head
// table (the slot code's read parity), writes its new rows only into ring rows
// outside the current window and writes the advanced heads to the other table,
// so an unsuccessful step leaves the committed window untouched.
constexpr int kSlotFloats = 161856;                       // window floats (reference state size)
constexpr int kRingFloats = 2 * kSlotFloats;              // ring rows of all histories
constexpr int kHeadInts = 32;                             // per head table (26 used)
constexpr int kSlotStride = kRingFloats + 2 * kHeadInts;  // floats per slot

// kResidualPre: a residual unit whose A operand (depthwise + Snake_post, f16
// [rows][C]) was written by launch_depthwise; the engine TMA-loads it.
// kTconvPre: an int8 transposed conv whose two s8 taps were written by
// launch_quantize; the engine TMA-loads them.
enum LayerKind : int { kStem = 0, kTconv = 1, kResidual = 2, kTestGemm = 3, kResidualPre = 4, kTconvPre = 5 };

// Operand precision of a GEMM layer.
enum GemmMode : int {
  kModeF16 = 0,    // one f16 x f16 MMA, fp32 accumulate
  kModeSplit = 1,  // three bf16 MMAs (hi*hi + hi*lo + lo*hi), fp32 accumulate
  kModeI8 = 2,     // W8A8: s8 x s8 MMAs (kind::i8), s32 accumulate, per-row weight and activation scales
  kModeSplit4 = 3, // four bf16 MMAs (adds lo*lo): the fp32 product to ~2^-24 relative
};

// K elements of one int8 pipeline stage (128 bytes per operand row).
constexpr int kKBlockI8 = 128;

// Stream slot codes passed to a step: (slot << 2) | (fresh << 1) | read_parity.
// ``fresh`` starts the stream from an all-zero history.
struct StateRef {
  float* pool;            // history pool, kSlotStride floats per slot; nullptr = zero history, not advanced
  const int* slot_codes;  // device array, one code per stream of the call; nullptr = uniform
  int num_slots;
  int uniform_code;       // with slot_codes == nullptr: stream s uses (s << 2) | uniform_code
};

// One history of the current layer.
struct HistRef {
  int index;   // 0..25 (reference order)
  int ring;    // float offset of the ring inside a slot
  int rows;    // H (window rows)
  int width;   // C (channels per row)
};

// Epilogue outputs (bit mask). y = accumulator + bias (+ the layer input x for
// a residual unit). The epilogue also applies the next layer's pointwise
// prologue, so the next producer only does the work that needs neighbouring rows.
enum EpilogueFlags : int {
  kEpiX = 2,       // y (fp32) to out_x
  kEpiS = 4,       // Snake(y) with next_alpha/next_recip (fp32) to out_s
  kEpiPlanes = 8,  // split-bf16 hi/lo planes of Snake(y * next_scale + next_offset) to out_planes, the
                   // same planes one row later per stream to out_planes_prev (row t holds t - 1; a
                   // stream's first row holds the next layer's history), and the next layer's history
  kEpiAct = 16,    // int8 path: Snake(y * next_scale + next_offset) fp32 to out_s, per row the max of its
                   // magnitude over each column group of each N tile to rowmax_out[row * rowmax_parts + part],
                   // and the next layer's history
  kEpiS16 = 32,    // Snake(y) with next_alpha/next_recip rounded to f16, to out_s read as f16 (same layout
                   // as kEpiS at half the bytes)
};

struct LayerArgs {
  CUtensorMap tmap;   // producer input. Residual: s [rows][k] fp32, boxes of min(k, 64) channels x
                      // box_rows rows. Transposed conv: tap-0 planes [2][rows][k] bf16, boxes of
                      // 64 x 128 x 2 in the 128-byte swizzle (the MMA's A layout, hi tile then lo tile).
  CUtensorMap tmap2;  // transposed conv: tap-1 planes (each row holds the previous time step)
  // Epilogue outputs: y and Snake(y) as [rows][c] fp32 ([rows][stride][c] for a transposed conv);
  // planes as [2][rows][c] bf16 (hi, then lo).
  float* out_x;
  float* out_s;
  uint16_t* out_planes;
  uint16_t* out_planes_prev;
  HistRef hist_next;  // history of the layer that reads out_planes (its previous activated input)
  // int8 path (kModeI8 and kEpiAct):
  float* rowmax_out;         // [rows][rowmax_parts] partial row maxima of |out_s|
  int rowmax_parts;
  const float* rowmax_in;    // the same, written by the previous layer, for this layer's input rows
  int rowmax_in_parts;
  const float* w_scale;      // per-GEMM-column weight scale (transposed conv: current tap)
  const float* w_scale2;     // transposed conv: previous tap
  const float* row_scale;    // int8 kResidualPre: activation scale of each input row (quantize_residual)
  int hist_max_slot;         // transposed conv: head-table entry holding the history row's max |x|
  const float* dense_w;      // int8 plan's stem on CUDA cores: 1x1 weights [n_total][k] fp32
  int kind;
  int mode;
  int epi;              // EpilogueFlags
  int rows;             // GEMM rows: all streams' time steps at this layer's input
  int rows_per_stream;  // time steps per stream at this layer's input
  int k_channels;       // input channels (K of one tap)
  int num_kblocks;      // K blocks of the whole reduction (both taps for a transposed conv)
  int n_total;          // GEMM N
  int n_tile;           // GEMM N per CTA
  int n_major;          // tile order: 0 = M tiles fastest (share weights), 1 = N tiles fastest (share A)
  int c_out;            // output channels
  int stride;           // transposed-conv rate
  int dilation;         // residual depthwise dilation
  int box_rows;         // rows of one TMA input box (tile + causal halo)
  int raw_pitch;        // floats per staged input row (min(k, 64))
  const float* x;       // stem: latents [streams][64][z_stride]; residual: layer input x [rows][k] (skip)
  int z_stride;         // stem: frames per stream in the latent buffer
  int z_offset;         // stem: first frame of this step in the latent buffer
  const float* bias;
  const float* dw_w;    // stem depthwise taps [64][7]
  const float* dw_b;
  // Residual: per-64-channel-block coefficients packed for one bulk copy per K
  // block, [block][w0..w6, bias, alpha2, recip2][64] (zero padded).
  const float* coef;
  // Residual: the staged input is s = Snake_pre(y) in f16 (written by the
  // previous epilogue with kEpiS16; boxes of 64 channels x box_rows rows, 128
  // bytes per row); the producers read the box as is.
  int s16;
  const float* next_scale;  // coefficients of the pointwise prologue the epilogue applies
  const float* next_offset;
  const float* next_alpha;
  const float* next_recip;
  const uint8_t* wimg;  // packed weight tiles [N / img_nt][kblock][term][img_nt rows][128 B]
  // N tile the weight image was packed for (0: n_tile). A launch with a
  // smaller n_tile (more CTAs for a step of few rows) reads its NT rows of
  // each packed block: a contiguous run with the same 128-byte swizzle.
  int img_nt;
  StateRef state;
  HistRef hist;
  uint32_t* status;
  // Diagnostics (zero in every ordinary launch): polls after which a wait of
  // this launch gives up (0 = kWaitLimit), and a device flag the MMA issuer
  // waits for before its first MMA (nullptr = none). A flag that nothing sets
  // makes every role's wait run out, which tests the timeout path.
  uint32_t wait_limit;
  const uint32_t* gate;
};

struct FinalArgs {
  int rows;
  int rows_per_stream;
  const float* x;       // Snake_final(y) [rows][32]
  float* audio;         // [streams][audio_stride]
  int audio_stride;     // samples per stream in the audio buffer
  int audio_offset;     // first sample of this step in the audio buffer
  const float* w;       // [32][7]
  const float* b;       // [1]
  StateRef state;
  HistRef hist;
  uint32_t* status;
};

// Launches ``kernel`` so that it may start while the previous kernel in the
// stream drains (programmatic dependent launch); the kernel must call
// grid_dependency_sync() before its first access to memory earlier kernels use.
template <typename Args>
inline cudaError_t launch_overlapped(void (*kernel)(Args), unsigned grid, unsigned block, size_t smem,
                                     cudaStream_t stream, const Args& a) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, a);
}

// Fused stage-5 tail (fav_tail.cu): the three residual units and the final conv.
constexpr int kTailC = 32;  // stage-5 channels
struct TailUnitArgs {
  const float* pre_a;    // Snake before the depthwise conv [32]
  const float* pre_r;
  const float* coef;     // depthwise block [w0..w6, bias, alpha2, recip2][64] (zero padded)
  const float* bias;     // 1x1 bias [32]
  const uint8_t* wimg;   // 1x1 weights, 32 rows x 128 B (f16, K-major, 128-byte swizzle)
  HistRef hist;          // window of Snake_pre(input), 6 * dilation rows
};
// Rows of the fused tail's x boxes: one 128-row tile.
constexpr int kTailBoxRows = 128;
struct TailArgs {
  CUtensorMap xmap;      // stage input y [rows][32] fp32: boxes of 32 x kTailBoxRows, 128-byte swizzle
  int rows;              // all streams' rows (multiple of 128)
  int rows_per_stream;   // multiple of 128
  TailUnitArgs unit[3];
  const float* fin_a;    // final Snake [32]
  const float* fin_r;
  const float* fin_w;    // final conv [32][7]
  const float* fin_b;    // [1]
  HistRef fin_hist;      // window of Snake_final(y3), 6 rows
  float* audio;
  int audio_stride;
  int audio_offset;
  StateRef state;
  uint32_t* status;
};
cudaError_t launch_tail(const TailArgs& a, cudaStream_t stream);

// Fused residual stage (fav_stage.cu): the three residual units of a stage with
// 64 or 128 channels (stages 4 and 3) and the next transposed conv's planes.
struct StageUnitArgs {
  const float* pre_a;    // Snake before the depthwise conv [C]
  const float* pre_r;
  const float* coef;     // depthwise blocks [C / 64][w0..w6, bias, alpha2, recip2][64]
  const float* bias;     // 1x1 bias [C]
  const uint8_t* wimg;   // 1x1 weights [C / 64][C rows][128 B] (f16, K-major, 128-byte swizzle)
  HistRef hist;          // window of Snake_pre(input) (f16 values), 6 * dilation rows
};
struct StageArgs {
  CUtensorMap xmap;      // stage input y [rows][C] fp32: boxes of 32 channels x 128 rows, 128-byte swizzle
  // out_planes / out_planes_prev as [2 planes][streams][rows_per_stream][C]
  // bf16: store boxes of 64 channels x 128 rows, 128-byte swizzle.
  CUtensorMap planes_map;
  CUtensorMap prev_map;
  const float* x;        // the stage input (L2 prefetch of the next tile)
  int channels;          // C: 64 or 128
  int rows;              // all streams' rows
  int rows_per_stream;
  StageUnitArgs unit[3];
  const float* next_scale;   // next stage's affine and Snake [C]
  const float* next_offset;
  const float* next_alpha;
  const float* next_recip;
  uint16_t* out_planes;      // [2][rows][C] bf16 (hi, then lo)
  uint16_t* out_planes_prev; // the same one row later per stream (a stream's first row: hist_next's row)
  HistRef hist_next;         // next transposed conv's one-row history, packed (hi << 16) | lo per channel
  StateRef state;
  uint32_t* status;
  // Diagnostics, as in LayerArgs: polls after which a wait gives up (0 =
  // kWaitLimit), and a device flag the first MMA waits for (nullptr = none).
  uint32_t wait_limit;
  const uint32_t* gate;
};
cudaError_t launch_stage(const StageArgs& a, cudaStream_t stream);
cudaError_t prepare_stage();
int stage_sm_count();  // SMs of the device prepare_stage ran on

// Depthwise pre-pass of a residual unit (fav_prepass.cu): A = Snake_post(
// depthwise_k7(s)) as f16 [rows][channels] for a kResidualPre GEMM, plus the
// layer's new history window.
struct DepthwiseArgs {
  const float* s;        // Snake_pre(x) [rows][channels] fp32
  uint16_t* a;           // A operand [rows][channels] f16
  const float* coef;     // [channels / 64][w0..w6, bias, alpha2, recip2][64]
  int rows;
  int rows_per_stream;
  int channels;          // multiple of 4, at most 1024
  int dilation;
  StateRef state;
  HistRef hist;
};
cudaError_t launch_depthwise(const DepthwiseArgs& a, cudaStream_t stream);

// Quantise-once pre-pass of an int8 transposed conv (fav_prepass.cu): the
// conv's two s8 taps, each row quantised with its time step's scale (the
// reference's per-time-step activation scale over all input channels).
struct QuantizeArgs {
  const float* act;      // [rows][channels] fp32 activation written by the previous epilogue
  const float* rowmax;   // [rows][parts] partial maxima of |act| (one per N tile of that epilogue)
  int parts;
  uint8_t* q0;           // [rows][channels] s8: row t
  uint8_t* q1;           // [rows][channels] s8: row t - 1 (a stream's first row: its history row)
  int rows;
  int rows_per_stream;
  int channels;          // multiple of 4
  StateRef state;
  HistRef hist;          // the conv's one-row fp32 history
  int hist_max_slot;     // head-table entry holding the history row's max |x|
};
cudaError_t launch_quantize(const QuantizeArgs& a, cudaStream_t stream);

// Pre-pass of an int8 residual unit (fav_prepass.cu): the unit's A operand,
// Snake_post(depthwise_k7(s)) in the int8 path's fixed operation order,
// quantised per row with the recipe's per-time-step scale over all channels
// (s8 [rows][channels]) plus that scale per row, and the layer's new history
// window.
struct QuantResidualArgs {
  const float* s;        // Snake_pre(x) [rows][channels] fp32
  uint8_t* q;            // A operand [rows][channels] s8
  float* scale;          // [rows]
  const float* coef;     // [channels / 64][w0..w6, bias, alpha2, recip2][64]
  int rows;
  int rows_per_stream;
  int channels;          // 128, 256, 512 or 1024
  int dilation;
  StateRef state;
  HistRef hist;
};
cudaError_t launch_quantize_residual(const QuantResidualArgs& a, cudaStream_t stream);
cudaError_t prepare_tail();

// Kernel launchers (fav_kernels.cu). Return cudaError_t of the launch.
cudaError_t launch_gemm_layer(const LayerArgs& a, cudaStream_t stream);
// Epilogue warps per TMEM lane quarter of the engine instance that runs a
// layer of this N tile and kind (3 for TMA-fed A operands, else 1); a kEpiAct
// epilogue writes rowmax_parts = (n_total / n_tile) * that partial maxima per row.
int epilogue_column_groups(int n_tile, int kind);
constexpr int kMaxRowmaxParts = 12;
// The int8 plan's stem (depthwise k=7 -> 1x1 -> stage 0's affine + Snake, row
// maxima and history) on CUDA cores, every sum in the int8 oracle's order.
cudaError_t launch_stem_exact(const LayerArgs& a, cudaStream_t stream);
// Diagnostic: out[i] = the int8 path's fixed-order sine of x[i] (device arrays).
cudaError_t launch_sine_test(const float* x, int n, float* out, cudaStream_t stream);
cudaError_t launch_final(const FinalArgs& a, cudaStream_t stream);
cudaError_t prepare_kernels();

// Coefficient vectors per 64-channel block of a residual unit: depthwise taps
// w0..w6, depthwise bias, the second Snake's alpha and reciprocal, then the
// first Snake's alpha and reciprocal (used when the unit reads y itself).
constexpr int kCoefResidual = 10;

// Rows of the TMA input box of a residual unit: the 128-row tile plus the
// causal halo of 6*dilation rows.
inline int box_rows_for(int kind, int dilation) {
  return kind == kResidual ? kTileM + 6 * dilation : 0;
}

}  // namespace fav
