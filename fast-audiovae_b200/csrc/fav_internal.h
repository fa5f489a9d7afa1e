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

enum LayerKind : int { kStem = 0, kTconv = 1, kResidual = 2, kTestGemm = 3 };

// Operand precision of a GEMM layer.
enum GemmMode : int {
  kModeF16 = 0,    // one f16 x f16 MMA, fp32 accumulate
  kModeSplit = 1,  // three bf16 MMAs (hi*hi + hi*lo + lo*hi), fp32 accumulate
};

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

struct LayerArgs {
  CUtensorMap tmap;       // TMA map of the layer input x [rows][k] fp32 (transposed conv, residual)
  CUtensorMap tmap_out;   // TMA map of the output, 32 x 32 fp32 boxes, 128-byte swizzle
                          // (transposed conv: 3-D view [rows][rate][c_out], boxes 32 x 1 x 32)
  CUtensorMap tmap_skip;  // residual: TMA map of x for the skip add, 32 x 32 boxes, 128-byte swizzle
  int kind;
  int mode;
  int rows;             // GEMM rows: all streams' time steps at this layer's input
  int rows_per_stream;  // time steps per stream at this layer's input
  int k_channels;       // input channels (K of one tap)
  int num_kblocks;      // K blocks of the whole reduction (both taps for a transposed conv)
  int n_total;          // GEMM N
  int n_tile;           // GEMM N per CTA
  int c_out;            // output channels
  int stride;           // transposed-conv rate
  int dilation;         // residual depthwise dilation
  int box_rows;         // rows of one TMA input box (tile + causal halo)
  int raw_pitch;        // floats per staged input row (min(k, 64))
  const float* x;       // input activations [rows][k] fp32 (stem: latents [streams][64][z_stride])
  int z_stride;         // stem: frames per stream in the latent buffer
  int z_offset;         // stem: first frame of this step in the latent buffer
  float* out;           // output activations fp32
  const float* bias;
  const float* scale;   // stage affine
  const float* offset;
  const float* alpha1;  // Snake before the projection (stage) / before the depthwise conv (residual)
  const float* recip1;
  const float* alpha2;  // Snake after the depthwise conv (residual)
  const float* recip2;
  const float* dw_w;    // depthwise taps: stem [64][7], residual [7][C]
  const float* dw_b;
  // Per-64-channel-block coefficients, packed for one bulk copy per K block:
  // transposed conv [block][scale, offset, alpha, recip][64]; residual
  // [block][alpha1, recip1, w0..w6, bias, alpha2, recip2][64] (zero padded).
  const float* coef;
  const uint8_t* wimg;  // packed weight tiles [n_tile][kblock][term][n_tile rows][128 B]
  StateRef state;
  HistRef hist;
  uint32_t* status;
};

struct FinalArgs {
  int rows;
  int rows_per_stream;
  const float* x;       // [rows][32]
  float* audio;         // [streams][audio_stride]
  int audio_stride;     // samples per stream in the audio buffer
  int audio_offset;     // first sample of this step in the audio buffer
  const float* alpha;
  const float* recip;
  const float* w;       // [32][7]
  const float* b;       // [1]
  StateRef state;
  HistRef hist;
  uint32_t* status;
};

// Kernel launchers (fav_kernels.cu). Return cudaError_t of the launch.
cudaError_t launch_gemm_layer(const LayerArgs& a, cudaStream_t stream);
cudaError_t launch_final(const FinalArgs& a, cudaStream_t stream);
cudaError_t prepare_kernels();

constexpr int kCoefTconv = 4;      // coefficient vectors per channel block
constexpr int kCoefResidual = 12;

// Rows of the TMA input box for a layer kind: the 128-row tile plus the
// causal halo (one row for a transposed conv, 6*dilation for a residual unit).
inline int box_rows_for(int kind, int dilation) {
  return kind == kTconv ? kTileM + 1 : kind == kResidual ? kTileM + 6 * dilation : 0;
}

}  // namespace fav
