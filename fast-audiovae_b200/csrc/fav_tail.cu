// Fused tail of the decoder step: stage 5's three residual units and the final
// conv (Snake_final -> causal conv 32 -> 1, k = 7 -> tanh) in one persistent
// kernel (the reference's mps_decoder.py stage loop and final conv, restated in
// the fp32 oracle at oracle/decoder.py:160-175).
//
// Stage 5 has 32 channels and 1920 rows per frame, so its per-layer kernels
// move whole [rows][32] activations through HBM four times per unit for a
// 32 x 32 projection. Here each CTA takes 128 output rows (audio samples) at a
// time and keeps every intermediate in shared memory:
//
//   x              rows [-84, 128)   TMA box, 128-byte swizzle
//   Snake_pre1(x)  rows [-84, 128) -> depthwise d=1 -> Snake -> f16 A -> MMA
//   y1             rows [-78, 128)   = x + (A W1 + b1)
//   Snake_pre2(y1) rows [-78, 128) -> depthwise d=3 -> ...
//   y2             rows [-60, 128)
//   Snake_pre3(y2) rows [-60, 128) -> depthwise d=9 -> ...
//   Snake_f(y3)    rows [-6, 128)  -> final conv -> audio rows [0, 128)
//
// (row 0 = the tile's first output row). The halo rows before the tile are
// recomputed from x, except where a stream starts at the tile: rows before a
// stream's first row come from the layers' history rings instead (the rows of
// the previous stream, or of no stream, only feed rows that are discarded).
// Stage 5 has 1920 rows per frame, a multiple of 128, so a tile never straddles
// two streams. The tile holding a stream's last row writes the new windows.
// Every row is computed by the same instructions wherever it falls in a tile,
// so halo rows equal the rows the neighbouring tile keeps, and a stream decoded
// in chunks equals the same stream decoded at once, bit for bit.
//
// The 32 x 32 projections run on the tensor cores (tcgen05.mma kind::f16, M =
// 128 x 2 tiles, N = 32, K = 32, fp32 accumulators in TMEM); depthwise convs,
// Snake, skip adds and the final conv run on the CUDA cores, 512 threads per
// CTA, in the operation order of the per-layer kernels.
#include "fav_common.cuh"

namespace fav {
namespace {

constexpr int kTailThreads = 512;
constexpr int kTailRows = 128;   // output rows per tile
constexpr int kTailHalo = 84;    // x rows before the tile: 6 + 18 + 54 + 6
constexpr int kTailIn = kTailRows + kTailHalo;
constexpr int kTailBuf = ((kTailIn * 128 + 1023) / 1024) * 1024;  // one row buffer (fp32 rows of 128 B)
constexpr int kTailA = 256 * 128;                                 // f16 A operand: 2 M tiles
constexpr int kTailW = kTailC * 128;                              // one unit's B operand
constexpr int kTailCoef = kCoefResidual * 64;                     // floats of one unit's depthwise block

struct TailSmem {
  // byte offsets from the 1024-aligned base
  static constexpr int kX0 = 0;
  static constexpr int kX1 = kTailBuf;
  static constexpr int kP = 2 * kTailBuf;
  static constexpr int kQ = 3 * kTailBuf;
  static constexpr int kA = 4 * kTailBuf;
  static constexpr int kW = kA + kTailA;
  static constexpr int kCoefs = kW + 3 * kTailW;                 // floats from here on
  static constexpr int kUnitCoef = 0;                            // [3][kTailCoef]
  static constexpr int kPwBias = 3 * kTailCoef;                  // [3][32]
  static constexpr int kPreA = kPwBias + 3 * kTailC;             // [3][32]
  static constexpr int kPreR = kPreA + 3 * kTailC;               // [3][32]
  static constexpr int kFinA = kPreR + 3 * kTailC;               // [32]
  static constexpr int kFinR = kFinA + kTailC;                   // [32]
  static constexpr int kFinW = kFinR + kTailC;                   // [7][32] (tap-major)
  static constexpr int kFinB = kFinW + kTailC * 7;               // [4]
  static constexpr int kCoefFloats = kFinB + 4;
  static constexpr int kMisc = kCoefs + kCoefFloats * 4;         // ints: heads[4], code, pad
  static constexpr int kBars = ((kMisc + 8 * 4 + 7) / 8) * 8;    // xfull[2], mma_done, tmem slot
  static constexpr int kOut = ((kBars + 4 * 8 + 15) / 16) * 16;   // float[128]: one tile's audio
  static constexpr int kBytes = kOut + kTailRows * 4;
  static constexpr int kAlloc = kBytes + 1024;
};
static_assert(TailSmem::kAlloc <= 227 * 1024, "tail kernel shared memory");

// fp32 row buffers: row r, channel quad q (channels 4q .. 4q+3) in the 128-byte
// swizzle (16-byte chunk q of row r at chunk q ^ (r & 7)), the layout a TMA
// box with CU_TENSOR_MAP_SWIZZLE_128B writes. Both access patterns used here
// (a lane per row, and eight lanes per row) are then free of bank conflicts.
__device__ __forceinline__ int swq(int r, int q) { return r * 32 + ((q ^ (r & 7)) << 2); }

__device__ __forceinline__ int stream_code(const StateRef& st, int s) {
  return st.slot_codes ? st.slot_codes[s] : ((s << 2) | st.uniform_code);
}

// Window row of time tp (-H <= tp < 0) of a history whose window starts at head.
__device__ __forceinline__ float4 hist_quad(const StateRef& st, const HistRef& h, int code, int head, int tp, int q) {
  if (!st.pool || (code & 2)) return make_float4(0.f, 0.f, 0.f, 0.f);
  int row = head + h.rows + tp;
  if (row >= 2 * h.rows) row -= 2 * h.rows;
  return ldg4(slot_base(st, code) + h.ring + row * h.width + 4 * q);
}

// Depthwise k=7 (dilation d) + Snake_post of rows [0, n_out) into the f16 A
// operand, for this thread's chain of L rows in channel quad q.
template <int L>
__device__ __forceinline__ void depthwise_chains(const float* uc, const float* pbuf, uint8_t* aop, int rg, int q, int d,
                                                 int n_out) {
  const int i0 = (rg / d) * L * d + rg % d;
  if (i0 >= n_out) return;
  float4 w[7], win[7];
#pragma unroll
  for (int j = 0; j < 7; ++j) w[j] = lds4(uc + j * 64 + 4 * q);
  const float4 bias = lds4(uc + 7 * 64 + 4 * q), al2 = lds4(uc + 8 * 64 + 4 * q), rc2 = lds4(uc + 9 * 64 + 4 * q);
#pragma unroll
  for (int j = 0; j < 6; ++j) win[j] = lds4(pbuf + swq(i0 + j * d, q));
#pragma unroll
  for (int c = 0; c < L; ++c) {
    const int i = i0 + c * d;
    if (i >= n_out) break;
    win[6] = lds4(pbuf + swq(i + 6 * d, q));
    const float4 y = snake4(dw7<false>(w, win, bias), al2, rc2);
    *reinterpret_cast<uint2*>(aop + sw128_offset(i, 4 * q)) = make_uint2(pack_f16(y.x, y.y), pack_f16(y.z, y.w));
#pragma unroll
    for (int j = 0; j < 6; ++j) win[j] = win[j + 1];
  }
}

__global__ void __launch_bounds__(kTailThreads, 1) tail_kernel(const __grid_constant__ TailArgs a) {
  extern __shared__ uint8_t tail_smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tail_smem_raw) + 1023) & ~uintptr_t(1023));
  float* xbuf[2] = {reinterpret_cast<float*>(sm + TailSmem::kX0), reinterpret_cast<float*>(sm + TailSmem::kX1)};
  float* pbuf = reinterpret_cast<float*>(sm + TailSmem::kP);
  float* qbuf = reinterpret_cast<float*>(sm + TailSmem::kQ);
  uint8_t* aop = sm + TailSmem::kA;
  uint8_t* wop = sm + TailSmem::kW;
  float* cf = reinterpret_cast<float*>(sm + TailSmem::kCoefs);
  int* misc = reinterpret_cast<int*>(sm + TailSmem::kMisc);
  float* obuf = reinterpret_cast<float*>(sm + TailSmem::kOut);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + TailSmem::kBars);
  uint64_t* xfull = bars;         // [2]
  uint64_t* mma_done = bars + 2;  // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int N = a.rows_per_stream;
  const int num_tiles = a.rows / kTailRows;
  constexpr uint32_t kBoxBytes = kTailIn * 128;

  // ---- one-time setup: barriers, TMEM, coefficients and weights
  if (tid == 0) {
    mbar_init(&xfull[0], 1);
    mbar_init(&xfull[1], 1);
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 64);
    tmem_relinquish();
  }
  for (int u = 0; u < 3; ++u) {
    const TailUnitArgs& un = a.unit[u];
    for (int i = tid; i < kTailCoef; i += kTailThreads) cf[TailSmem::kUnitCoef + u * kTailCoef + i] = __ldg(un.coef + i);
    for (int i = tid; i < kTailC; i += kTailThreads) {
      cf[TailSmem::kPwBias + u * kTailC + i] = __ldg(un.bias + i);
      cf[TailSmem::kPreA + u * kTailC + i] = __ldg(un.pre_a + i);
      cf[TailSmem::kPreR + u * kTailC + i] = __ldg(un.pre_r + i);
    }
    for (int i = tid; i < kTailW / 16; i += kTailThreads)
      reinterpret_cast<uint4*>(wop + u * kTailW)[i] = __ldg(reinterpret_cast<const uint4*>(un.wimg) + i);
  }
  for (int i = tid; i < kTailC; i += kTailThreads) {
    cf[TailSmem::kFinA + i] = __ldg(a.fin_a + i);
    cf[TailSmem::kFinR + i] = __ldg(a.fin_r + i);
  }
  for (int i = tid; i < kTailC * 7; i += kTailThreads) cf[TailSmem::kFinW + (i % 7) * kTailC + i / 7] = __ldg(a.fin_w + i);
  if (tid == 0) cf[TailSmem::kFinB] = __ldg(a.fin_b);
  fence_async_smem();  // weights written by the generic proxy, read by the tensor core
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dependency_sync();  // plan constants above; the stage input and histories below

  if (tid == 0 && blockIdx.x < num_tiles) {
    mbar_arrive_expect_tx(&xfull[0], kBoxBytes);
    tma_load_2d(xbuf[0], &a.xmap, 0, (int)blockIdx.x * kTailRows - kTailHalo, &xfull[0]);
  }

  bool ok = true;
  bool issued_next = false;  // this iteration started the next tile's x load
  uint32_t n_mma = 0;
  int k = 0;
  for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++k) {
    const int buf = k & 1;
    const int m0 = t * kTailRows;
    const int s = m0 / N, t0 = m0 - s * N;  // stream and its first time step in this tile
    const bool first = t0 == 0, last = t0 + kTailRows == N;
    // Next tile's x into the other buffer (free: the previous tile has ended).
    issued_next = t + (int)gridDim.x < num_tiles;
    if (tid == 0 && issued_next) {
      mbar_arrive_expect_tx(&xfull[buf ^ 1], kBoxBytes);
      tma_load_2d(xbuf[buf ^ 1], &a.xmap, 0, (t + (int)gridDim.x) * kTailRows - kTailHalo, &xfull[buf ^ 1]);
    }
    // Stream slot and window heads (units 0-2, final), when the tile reads or writes a window.
    if (tid < 4 && (first || last)) {
      const int code = stream_code(a.state, s);
      const HistRef& h = tid < 3 ? a.unit[tid].hist : a.fin_hist;
      misc[tid] = (a.state.pool && !(code & 2)) ? head_table(slot_base(a.state, code), code & 1)[h.index] : 0;
      if (tid == 0) misc[4] = code;
    }
    ok = __syncthreads_and(mbar_wait(&xfull[buf], (k >> 1) & 1, a.status, kDevTimeoutLoader));
    if (!ok) break;
    const int code = misc[4];
    float* xb = xbuf[buf];

#pragma unroll
    for (int u = 0; u < 3; ++u) {
      const int d = u == 0 ? 1 : u == 1 ? 3 : 9, H = 6 * d;
      const int in_off = u == 0 ? 84 : u == 1 ? 78 : 60;  // input buffer row of relative row 0
      const int n_in = kTailRows + in_off;      // input rows
      const int n_out = n_in - H;               // depthwise / projection rows
      const float* in = u == 1 ? qbuf : xb;     // unit input y (x for unit 0)
      float* out = u == 0 ? qbuf : u == 1 ? xb : qbuf;  // y1 -> q, y2 -> x buffer, Snake_f(y3) -> q
      const HistRef& hist = a.unit[u].hist;
      const float* uc = cf + TailSmem::kUnitCoef + u * kTailCoef;
      // (a) p = Snake_pre(input) (units 1 and 2: written by the previous
      // unit's epilogue); a stream's first tile takes the rows before the
      // stream from the history window.
      // Each thread keeps one channel quad (q = tid % 8) in (a) and (b).
      const int q = tid & 7, rg = tid >> 3;
      if (u == 0) {
        const float4 pa = lds4(cf + TailSmem::kPreA + 4 * q);
        const float4 pr = lds4(cf + TailSmem::kPreR + 4 * q);
        for (int i = rg; i < n_in; i += kTailThreads / 8)
          *reinterpret_cast<float4*>(pbuf + swq(i, q)) = snake4(lds4(in + swq(i, q)), pa, pr);
      }
      if (first) {
        if (u == 0) __syncthreads();
        for (int i = in_off - H + rg; i < in_off; i += kTailThreads / 8)
          *reinterpret_cast<float4*>(pbuf + swq(i, q)) = hist_quad(a.state, hist, code, misc[u], i - in_off, q);
      }
      if (u == 0 || first) __syncthreads();
      // (b) A = Snake_post(depthwise(p)) in f16; the stream's last tile also
      // writes the new window (the last H rows of p).
      // A thread's rows form a chain i0, i0 + d, ... (blocks of L*d rows split
      // into d chains of L), so the seven taps slide through registers: L = 4
      // covers unit 0's 206 rows with 64 row groups, L = 3 the others'.
      if (u == 0) {
        depthwise_chains<4>(uc, pbuf, aop, rg, q, 1, n_out);
      } else {
        depthwise_chains<3>(uc, pbuf, aop, rg, q, d, n_out);
      }
      if (last && a.state.pool && tid < H * 8) {
        const int m = tid >> 3, q = tid & 7;  // window row m = time N - H + m
        *reinterpret_cast<float4*>(hist_new_row(a.state, hist, code, misc[u], N - H + m, N) + 4 * q) =
            lds4(pbuf + swq(in_off + kTailRows - H + m, q));
      }
      fence_async_smem();
      tc_fence_before();
      __syncthreads();
      // (c) D[mt] = A[mt] W^T for the two 128-row M tiles, K = 32 (two K = 16 steps).
      if (tid == 0) {
        tc_fence_after();
        const uint32_t a0 = smem_u32(aop), b0 = smem_u32(wop + u * kTailW);
        constexpr uint32_t idesc = instr_desc_f16(0u, kTailC);
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
          for (int ks = 0; ks < 2; ++ks)
            mma_f16(tmem + mt * kTailC, smem_desc_sw128(a0 + mt * kTileM * 128 + ks * 32),
                    smem_desc_sw128(b0 + ks * 32), idesc, ks ? 1u : 0u);
        mma_commit(mma_done);
      }
      ok = __syncthreads_and(mbar_wait(mma_done, n_mma & 1, a.status, kDevTimeoutMma));
      ++n_mma;
      tc_fence_after();
      if (!ok) break;
      // (d) y = input + (D + b) for rows [0, n_out), with Snake_pre of the next
      // unit into p (the next unit's input rows); unit 2 keeps Snake_final(y).
      {
        const int lq = warp & 3, mt = (warp >> 2) & 1, half = warp >> 3;
        const int i = mt * kTileM + lq * 32 + lane;
        uint32_t r[16];
        tmem_ld16_async(tmem + ((uint32_t)(lq * 32) << 16) + (uint32_t)(mt * kTailC + half * 16), r);
        tmem_wait_ld(r);
        if (i < n_out) {
          const float* pb = cf + TailSmem::kPwBias + u * kTailC;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int q = half * 4 + j;
            const float4 b = lds4(pb + 4 * q);
            const float4 x = lds4(in + swq(i + H, q));
            float4 y = make_float4(x.x + (__uint_as_float(r[4 * j]) + b.x), x.y + (__uint_as_float(r[4 * j + 1]) + b.y),
                                   x.z + (__uint_as_float(r[4 * j + 2]) + b.z), x.w + (__uint_as_float(r[4 * j + 3]) + b.w));
            if (u == 2) {
              y = snake4(y, lds4(cf + TailSmem::kFinA + 4 * q), lds4(cf + TailSmem::kFinR + 4 * q));
            } else {
              *reinterpret_cast<float4*>(pbuf + swq(i, q)) =
                  snake4(y, lds4(cf + TailSmem::kPreA + (u + 1) * kTailC + 4 * q),
                         lds4(cf + TailSmem::kPreR + (u + 1) * kTailC + 4 * q));
            }
            *reinterpret_cast<float4*>(out + swq(i, q)) = y;
          }
        }
      }
      tc_fence_before();
      __syncthreads();
    }
    if (!ok) break;
    // Final conv over q = Snake_final(y3), rows [0, 134) = relative [-6, 128):
    // a stream's first tile takes rows [0, 6) from the final history; its last
    // tile writes the new window (relative rows [122, 128)).
    if (first && tid < 48) {
      const int m = tid >> 3, q = tid & 7;
      *reinterpret_cast<float4*>(qbuf + swq(m, q)) = hist_quad(a.state, a.fin_hist, code, misc[3], m - 6, q);
    }
    if (last && a.state.pool && tid >= 64 && tid < 64 + 48) {
      const int m = (tid - 64) >> 3, q = (tid - 64) & 7;
      *reinterpret_cast<float4*>(hist_new_row(a.state, a.fin_hist, code, misc[3], N - 6 + m, N) + 4 * q) =
          lds4(qbuf + swq(kTailRows + m, q));
    }
    if (last && a.state.pool && tid == 128) {
      for (int u = 0; u < 3; ++u) hist_commit_head(a.state, a.unit[u].hist, code, misc[u], N);
      hist_commit_head(a.state, a.fin_hist, code, misc[3], N);
    }
    __syncthreads();
    {
      // Four lanes per output row, eight channels each: one accumulator per
      // channel of a quad (taps oldest first), summed in a fixed tree.
      const int o = tid >> 2, grp = tid & 3;
      const float* fw = cf + TailSmem::kFinW;
      float4 acc4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int j = 0; j < 7; ++j) {
#pragma unroll
        for (int qq = 0; qq < 2; ++qq) {
          const int q = 2 * grp + qq;
          const float4 v = lds4(qbuf + swq(o + j, q));
          const float4 wj = lds4(fw + j * kTailC + 4 * q);
          acc4.x = fmaf(wj.x, v.x, acc4.x);
          acc4.y = fmaf(wj.y, v.y, acc4.y);
          acc4.z = fmaf(wj.z, v.z, acc4.z);
          acc4.w = fmaf(wj.w, v.w, acc4.w);
        }
      }
      float acc = (acc4.x + acc4.y) + (acc4.z + acc4.w);
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      if (grp == 0) {
        const float y = tanhf(acc + cf[TailSmem::kFinB]);
        // The reference checks the audio is finite (gpu.py:182-184).
        if (!(fabsf(y) <= 1.f)) record_error(a.status, kDevNonFinite);
        obuf[o] = y;
      }
    }
    fence_async_smem();  // this tile's generic writes to the x buffer precede the next TMA into it
    __syncthreads();
    if (tid < 32) {
      // One warp stores the tile's 128 samples as 512 contiguous bytes, whole
      // 128-byte lines whether the audio is device memory or mapped host
      // memory. (obuf is rewritten only after the next tile's barriers.)
      float* dst = a.audio + (size_t)s * a.audio_stride + a.audio_offset + t0;
      if ((reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
        reinterpret_cast<float4*>(dst)[tid] = lds4(obuf + 4 * tid);
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) dst[tid + 32 * k] = obuf[tid + 32 * k];
      }
    }
  }
  // After a timeout: let x loads still in flight land before the CTA exits
  // (a wait on a load that has landed returns at once).
  if (!ok && tid == 0) {
    mbar_wait(&xfull[k & 1], (k >> 1) & 1, a.status, kDevTimeoutLoader);
    if (issued_next) mbar_wait(&xfull[(k + 1) & 1], ((k + 1) >> 1) & 1, a.status, kDevTimeoutLoader);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 64);
}

int g_tail_sms = 0;

}  // namespace

cudaError_t prepare_tail() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&g_tail_sms, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(tail_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TailSmem::kAlloc);
  return e;
}

cudaError_t launch_tail(const TailArgs& a, cudaStream_t stream) {
  if (a.rows <= 0) return cudaSuccess;
  if (a.rows % kTailRows || a.rows_per_stream % kTailRows) return cudaErrorInvalidValue;
  const int tiles = a.rows / kTailRows;
  const int grid = tiles < g_tail_sms ? tiles : g_tail_sms;
  return launch_overlapped(tail_kernel, grid, kTailThreads, TailSmem::kAlloc, stream, a);
}

}  // namespace fav
