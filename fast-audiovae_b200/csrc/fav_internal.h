// Shared declarations between the kernel translation unit and the C ABI.
#pragma once
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
// floats of causal history per stream (the reference's 647,424 bytes)
constexpr int kSlotFloats = 161856;

enum LayerKind : int { kStem = 0, kTconv = 1, kResidual = 2, kTestGemm = 3 };

// Operand precision of a GEMM layer.
enum GemmMode : int {
  kModeF16 = 0,    // one f16 x f16 MMA, fp32 accumulate
  kModeSplit = 1,  // three bf16 MMAs (hi*hi + hi*lo + lo*hi), fp32 accumulate
};

// Stream slot codes passed to a step: (slot << 2) | (fresh << 1) | read_parity.
// The history of ``slot`` is read from pool half ``read_parity`` (or taken as
// zero when ``fresh``) and the advanced history is written to the other half.
struct StateRef {
  const float* pool_in;   // state pool (both halves); nullptr = all histories zero
  float* pool_out;        // state pool written; nullptr = histories not advanced
  const int* slot_codes;  // device array, one code per stream of the call; nullptr = uniform
  int num_slots;          // slots per pool half
  int uniform_code;       // with slot_codes == nullptr: stream s uses (s << 2) | uniform_code
};

struct LayerArgs {
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
  const float* dw_w;    // depthwise taps [C][7]
  const float* dw_b;
  const uint8_t* wimg;  // packed weight tiles [n_tile][kblock][term][n_tile rows][128 B]
  StateRef state;
  int state_off;        // offset of this layer's history inside a slot (floats)
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
  int state_off;
  uint32_t* status;
};

// Kernel launchers (fav_kernels.cu). Return cudaError_t of the launch.
cudaError_t launch_gemm_layer(const LayerArgs& a, cudaStream_t stream);
cudaError_t launch_final(const FinalArgs& a, cudaStream_t stream);
cudaError_t prepare_kernels();

// Bytes of one packed weight tile set (all terms) for ``n_tile`` rows.
inline size_t weight_tile_bytes(int n_tile, int mode) {
  return (size_t)n_tile * 128 * (mode == kModeSplit ? 2 : 1);
}

}  // namespace fav
