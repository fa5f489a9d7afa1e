// Pre-passes that write a GEMM's A operand once to HBM for the engine to
// TMA-load.
//
// Depthwise pre-pass of a residual unit (stages 0 and 1): the A operand of the
// unit's 1x1 projection, Snake_post(depthwise_k7(s)) in f16, written once to
// HBM so the GEMM engine TMA-loads it (LayerKind kResidualPre) instead of
// rebuilding it in every N tile's producers. The reference computes the unit
// as snake -> causal depthwise conv (with the stream's history) -> snake ->
// 1x1 conv (mps_decoder.py residual blocks, restated at oracle/decoder.py:165-171).
//
// At these stages a stream has 8 or 48 rows per frame, fewer than the 6d rows
// of history a dilated tap reaches back, so most taps come from the history
// ring. One thread per (row, channel quad) gives the gathers the whole GPU's
// memory-level parallelism; the arithmetic (fused multiply-add chain, Snake)
// is the producers' own, so the result is the same bit for bit.
//
// Each thread also writes its row of the layer's new history window (the
// input rows s that the next step's taps reach), zero rows for a fresh stream
// whose window is longer than the chunk, and the stream's advanced head.
#include "fav_common.cuh"

namespace fav {
namespace {

constexpr int kDwThreads = 256;

// Four blocks per SM (64 registers) keep more gathers in flight than the
// unconstrained 80-register build; measured faster at stages 0-1.
__global__ void __launch_bounds__(kDwThreads, 4) depthwise_kernel(const __grid_constant__ DepthwiseArgs a) {
  grid_dependency_sync();
  const int C = a.channels, quads = C / 4;
  const long long idx = (long long)blockIdx.x * kDwThreads + threadIdx.x;
  if (idx >= (long long)a.rows * quads) return;
  const int g = (int)(idx / quads), q = (int)(idx - (long long)g * quads);
  const int N = a.rows_per_stream, d = a.dilation, H = 6 * d;
  const int s = g / N, t = g - s * N;
  const int n_new = N < H ? N : H;
  const bool pool = a.state.pool != nullptr;
  int code = 0, head = 0;
  float* slot = nullptr;
  if (pool) {
    code = a.state.slot_codes ? a.state.slot_codes[s] : ((s << 2) | a.state.uniform_code);
    slot = slot_base(a.state, code);
    if (!(code & 2)) head = head_table(slot, code & 1)[a.hist.index];
  }
  const int kl = (4 * q) & (kKBlock - 1);
  const float* cf = a.coef + (size_t)(4 * q / kKBlock) * kCoefResidual * 64 + kl;
  float4 w[7], win[7];
#pragma unroll
  for (int j = 0; j < 7; ++j) w[j] = ldg4(cf + j * 64);
  const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int j = 0; j < 7; ++j) {
    const int back = (6 - j) * d;
    const int tp = t - back;
    if (tp >= 0) {
      win[j] = ldg4(a.s + (size_t)(g - back) * C + 4 * q);
    } else if (pool && !(code & 2)) {
      int row = head + H + tp;  // window [head, head + H)
      if (row >= 2 * H) row -= 2 * H;
      win[j] = ldg4(slot + a.hist.ring + row * a.hist.width + 4 * q);
    } else {
      win[j] = zero4;
    }
  }
  const float4 y =
      snake4<false, false>(dw7<false, false>(w, win, ldg4(cf + 7 * 64)), ldg4(cf + 8 * 64), ldg4(cf + 9 * 64));
  *reinterpret_cast<uint2*>(a.a + (size_t)g * C + 4 * q) = make_uint2(pack_f16(y.x, y.y), pack_f16(y.z, y.w));
  if (!pool) return;
  if (t >= N - n_new)
    *reinterpret_cast<float4*>(hist_new_row(a.state, a.hist, code, head, t, N) + 4 * q) = win[6];
  if ((code & 2) && N < H) {
    // A fresh stream's window starts as H - N zero rows before its N new ones.
    for (int r = N + t; r < H; r += N)
      *reinterpret_cast<float4*>(slot + a.hist.ring + r * a.hist.width + 4 * q) = zero4;
  }
  if (t == 0 && q == 0) hist_commit_head(a.state, a.hist, code, head, N);
}

// Quantise-once pre-pass of an int8 transposed conv (int8 plans): the recipe
// quantises each time step of the conv's input with its own scale, max|x|/127
// over all input channels (precision.cpp ip_prepare, restated in
// oracle/int8_recipe.py). Each row is quantised once here into both taps:
// tap 0 at its own row, tap 1 one row later in the same stream; a stream's
// first tap-1 row is its history row (the previous step's last input row,
// kept in fp32 with its max in a spare head-table entry), zero for a fresh
// stream. The scale and rounding are the engine's producers' own, so the s8
// operands are the same bit for bit; one thread per (row, channel quad).
__global__ void __launch_bounds__(kDwThreads) quantize_kernel(const __grid_constant__ QuantizeArgs a) {
  grid_dependency_sync();
  const int C = a.channels, quads = C / 4;
  const long long idx = (long long)blockIdx.x * kDwThreads + threadIdx.x;
  if (idx >= (long long)a.rows * quads) return;
  const int g = (int)(idx / quads), q = (int)(idx - (long long)g * quads);
  const int N = a.rows_per_stream;
  const int s = g / N, t = g - s * N;
  float m = 0.f;
  for (int p = 0; p < a.parts; ++p) m = fmaxf(m, __ldg(a.rowmax + (size_t)g * a.parts + p));
  const uint32_t v = quant4(ldg4(a.act + (size_t)g * C + 4 * q), quant_scale(m));
  *reinterpret_cast<uint32_t*>(a.q0 + (size_t)g * C + 4 * q) = v;
  if (t + 1 < N) *reinterpret_cast<uint32_t*>(a.q1 + (size_t)(g + 1) * C + 4 * q) = v;
  if (t == 0) {
    float4 hv = make_float4(0.f, 0.f, 0.f, 0.f);
    float hm = 0.f;
    if (a.state.pool) {
      const int code = a.state.slot_codes ? a.state.slot_codes[s] : ((s << 2) | a.state.uniform_code);
      if (!(code & 2)) {
        float* slot = slot_base(a.state, code);
        const int* heads = head_table(slot, code & 1);
        int row = heads[a.hist.index] + a.hist.rows - 1;  // window row of time -1
        if (row >= 2 * a.hist.rows) row -= 2 * a.hist.rows;
        hv = ldg4(slot + a.hist.ring + row * a.hist.width + 4 * q);
        hm = __int_as_float(heads[a.hist_max_slot]);
      }
    }
    *reinterpret_cast<uint32_t*>(a.q1 + (size_t)g * C + 4 * q) = quant4(hv, quant_scale(hm));
  }
}

// Pre-pass of an int8 residual unit: one thread per (row, channel quad), a
// block of 256 threads covering 1024 / C whole rows, so each row's maximum
// |h| over all C channels (the recipe's per-time-step activation scale,
// precision.cpp ip_prepare) is reduced inside the block. h = Snake_post(
// depthwise_k7(s)) runs in the int8 oracle's fixed operation order (every
// product and sum rounded, the fixed-order sine), as the engine's producers
// did; the s8 values and scales are the recipe's round-half-to-even
// quantisation. History taps, the new window rows and the heads as in
// depthwise_kernel. Four blocks per SM (64 registers, a few spilled): the
// fixed-order arithmetic is a long dependent chain per element, and twice
// the resident warps of the unconstrained build hide more of its latency
// (int8 step 4.93 -> 4.35 ms).
__global__ void __launch_bounds__(kDwThreads, 4) quantize_residual_kernel(const __grid_constant__ QuantResidualArgs a) {
  __shared__ float part[kDwThreads / 32];
  grid_dependency_sync();
  const int C = a.channels, quads = C / 4;
  const int g = blockIdx.x * (kDwThreads / quads) + threadIdx.x / quads;
  const int q = threadIdx.x % quads;
  const bool valid = g < a.rows;
  const int N = a.rows_per_stream, d = a.dilation, H = 6 * d;
  const int s = valid ? g / N : 0, t = valid ? g - s * N : 0;
  const int n_new = N < H ? N : H;
  const bool pool = a.state.pool != nullptr;
  int code = 0, head = 0;
  float* slot = nullptr;
  if (pool && valid) {
    code = a.state.slot_codes ? a.state.slot_codes[s] : ((s << 2) | a.state.uniform_code);
    slot = slot_base(a.state, code);
    if (!(code & 2)) head = head_table(slot, code & 1)[a.hist.index];
  }
  const int kl = (4 * q) & (kKBlock - 1);
  const float* cf = a.coef + (size_t)(4 * q / kKBlock) * kCoefResidual * 64 + kl;
  const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 y = zero4, win[7];
  if (valid) {
    float4 w[7];
#pragma unroll
    for (int j = 0; j < 7; ++j) w[j] = ldg4(cf + j * 64);
#pragma unroll
    for (int j = 0; j < 7; ++j) {
      const int back = (6 - j) * d;
      const int tp = t - back;
      if (tp >= 0) {
        win[j] = ldg4(a.s + (size_t)(g - back) * C + 4 * q);
      } else if (pool && !(code & 2)) {
        int row = head + H + tp;  // window [head, head + H)
        if (row >= 2 * H) row -= 2 * H;
        win[j] = ldg4(slot + a.hist.ring + row * a.hist.width + 4 * q);
      } else {
        win[j] = zero4;
      }
    }
    y = snake4<true>(dw7<true>(w, win, ldg4(cf + 7 * 64)), ldg4(cf + 8 * 64), ldg4(cf + 9 * 64));
  }
  // Row maximum of |y| over the row's C / 4 threads (whole warps for C >= 128).
  float m = fmaxf(fmaxf(fabsf(y.x), fabsf(y.y)), fmaxf(fabsf(y.z), fabsf(y.w)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = m;
  __syncthreads();
  const int w0 = (threadIdx.x / quads) * (quads / 32), nw = quads / 32;
  m = part[w0];
  for (int k = 1; k < nw; ++k) m = fmaxf(m, part[w0 + k]);
  if (!valid) return;
  const float sc = quant_scale(m);
  *reinterpret_cast<uint32_t*>(a.q + (size_t)g * C + 4 * q) = quant4(y, sc);
  if (q == 0) a.scale[g] = sc;
  if (!pool) return;
  if (t >= N - n_new)
    *reinterpret_cast<float4*>(hist_new_row(a.state, a.hist, code, head, t, N) + 4 * q) = win[6];
  if ((code & 2) && N < H) {
    // A fresh stream's window starts as H - N zero rows before its N new ones.
    for (int r = N + t; r < H; r += N)
      *reinterpret_cast<float4*>(slot + a.hist.ring + r * a.hist.width + 4 * q) = zero4;
  }
  if (t == 0 && q == 0) hist_commit_head(a.state, a.hist, code, head, N);
}

}  // namespace

cudaError_t launch_quantize_residual(const QuantResidualArgs& a, cudaStream_t stream) {
  if (a.rows <= 0) return cudaSuccess;
  if (a.channels < 128 || a.channels > 1024 || (a.channels & (a.channels - 1))) return cudaErrorInvalidValue;
  const int rows_per_block = kDwThreads / (a.channels / 4);
  return launch_overlapped(quantize_residual_kernel, (unsigned)((a.rows + rows_per_block - 1) / rows_per_block),
                           kDwThreads, 0, stream, a);
}

cudaError_t launch_quantize(const QuantizeArgs& a, cudaStream_t stream) {
  if (a.rows <= 0) return cudaSuccess;
  if (a.channels % 4) return cudaErrorInvalidValue;
  const long long items = (long long)a.rows * (a.channels / 4);
  return launch_overlapped(quantize_kernel, (unsigned)((items + kDwThreads - 1) / kDwThreads), kDwThreads, 0,
                           stream, a);
}

cudaError_t launch_depthwise(const DepthwiseArgs& a, cudaStream_t stream) {
  if (a.rows <= 0) return cudaSuccess;
  if (a.channels % 4 || a.channels > 1024) return cudaErrorInvalidValue;
  const long long items = (long long)a.rows * (a.channels / 4);
  return launch_overlapped(depthwise_kernel, (unsigned)((items + kDwThreads - 1) / kDwThreads), kDwThreads, 0,
                           stream, a);
}

}  // namespace fav
