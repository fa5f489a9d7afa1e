// Fused tail of the decoder step: stage 5's three residual units and the final
// conv (Snake_final -> causal conv 32 -> 1, k = 7 -> tanh) in one persistent
// kernel (the reference's mps_decoder.py stage loop and final conv, restated in
// the fp32 oracle at oracle/decoder.py:160-175).
//
// Stage 5 has 32 channels and 1920 rows per frame, so its per-layer kernels
// move whole [rows][32] activations through HBM four times per unit for a
// 32 x 32 projection. Here each CTA takes a contiguous range of 128-row tiles
// (audio samples) and keeps every intermediate in shared memory. Within a tile,
// with row 0 its first output row:
//
//   Snake_pre1(x)  rows [-6, 128)  -> depthwise d=1 -> Snake -> f16 A -> MMA
//   y1             rows [0, 128)   = x + (A W1 + b1)
//   Snake_pre2(y1) rows [-18, 128) -> depthwise d=3 -> ...
//   y2             rows [0, 128)   (over y1, in place)
//   Snake_pre3(y2) rows [-54, 128) -> depthwise d=9 -> ...
//   Snake_f(y3)    rows [-6, 128)  (over y2, in place) -> final conv -> audio
//
// The rows before row 0 of each Snake_pre input (6d of them) and of Snake_f(y3)
// are the previous tile's last rows, kept in shared memory from one tile to the
// next of the same stream. At a stream's first tile they come from the layers'
// history rings instead, and the stream's last tile writes the new windows. A
// range that starts inside a stream first runs the tile before it as a warm-up
// tile with zero carried rows and discards its output: the zeros reach its rows
// [0, 6) of y1, [0, 24) of y2 and [0, 78) of y3 only, so the rows it carries on
// (its last 6, 18, 54 and 6) are exact. Stage 5 has 1920 rows per frame, a
// multiple of 128, so a tile never straddles two streams. Every row is computed
// by the same instructions wherever it is computed, so a stream decoded in
// chunks equals the same stream decoded at once, bit for bit.
//
// The 32 x 32 projections run on the tensor cores (tcgen05.mma kind::f16, M =
// 128, N = 32, K = 32, fp32 accumulators in TMEM); depthwise convs, Snake, skip
// adds and the final conv run on the CUDA cores in the operation order of the
// per-layer kernels. The phases of a tile are separated by block barriers, so
// a CTA alone leaves the SM idle at each of them: large launches run two CTAs
// of 256 threads per SM, whose phases interleave; a launch of at most one tile
// per SM runs one CTA of 512 threads per tile, for the shortest tile.
#include "fav_common.cuh"

namespace fav {
namespace {

constexpr int kTailRows = 128;  // output rows per tile
static_assert(kTailBoxRows == kTailRows, "x box: one tile's rows");
constexpr uint32_t kXBytes = kTailBoxRows * 128;
constexpr int kPOff = 54;                    // P buffer row of relative row 0 (rows [-54, 128))
constexpr int kQOff = 6;                     // Q buffer row of relative row 0 (rows [-6, 128))
constexpr int kCarryRows = 6 + 18 + 54 + 6;  // carried input rows of units 0-2 and the final conv
constexpr int kTailW = kTailC * 128;         // one unit's B operand
constexpr int kTailCoef = kCoefResidual * 64;  // floats of one unit's depthwise block

constexpr int row_buffer_bytes(int rows) { return ((rows * 128 + 1023) / 1024) * 1024; }

struct TailSmem {
  // byte offsets from the 1024-aligned base; fp32 row buffers of 128 B rows
  static constexpr int kX = 0;                                         // x: rows [0, 128)
  static constexpr int kP = kX + row_buffer_bytes(kTailRows);          // Snake_pre of a unit's input
  static constexpr int kQ = kP + row_buffer_bytes(kPOff + kTailRows);  // y1, y2, Snake_f(y3)
  static constexpr int kA = kQ + row_buffer_bytes(kQOff + kTailRows);  // f16 A operand, 128 rows
  static constexpr int kW = kA + kTailRows * 128;
  static constexpr int kCarry = kW + 3 * kTailW;                 // float[kCarryRows][32], plain rows
  static constexpr int kCoefs = kCarry + kCarryRows * 128;       // floats from here on
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
  static constexpr int kBars = ((kMisc + 8 * 4 + 7) / 8) * 8;    // xfull, mma_done, tmem slot
  static constexpr int kOut = ((kBars + 3 * 8 + 15) / 16) * 16;  // float[128]: one tile's audio
  static constexpr int kBytes = kOut + kTailRows * 4;
  static constexpr int kAlloc = kBytes + 1024;
};
// Two CTAs per SM: 228 KB of shared memory per SM, 1 KB of it reserved per CTA.
static_assert(2 * (TailSmem::kAlloc + 1024) <= 228 * 1024, "two tail CTAs per SM");

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

// Depthwise k=7 (dilation d) + Snake_post of A rows [0, 128) into the f16 A
// operand, A row i from P rows kPOff - 6d + i + j*d (j = 0..6), for this
// thread's chain of L rows i0, i0 + d, ... in channel quad q: blocks of L*d
// rows split into d chains of L, so the seven taps slide through registers.
template <int L>
__device__ __forceinline__ void depthwise_chains(const float* uc, const float* pbuf, uint8_t* aop, int rg, int q,
                                                 int d) {
  const int i0 = (rg / d) * L * d + rg % d;
  if (i0 >= kTailRows) return;
  const int base = kPOff - 6 * d;
  float4 w[7], win[7];
#pragma unroll
  for (int j = 0; j < 7; ++j) w[j] = lds4(uc + j * 64 + 4 * q);
  const float4 bias = lds4(uc + 7 * 64 + 4 * q), al2 = lds4(uc + 8 * 64 + 4 * q), rc2 = lds4(uc + 9 * 64 + 4 * q);
#pragma unroll
  for (int j = 0; j < 6; ++j) win[j] = lds4(pbuf + swq(base + i0 + j * d, q));
#pragma unroll
  for (int c = 0; c < L; ++c) {
    const int i = i0 + c * d;
    if (i >= kTailRows) break;
    win[6] = lds4(pbuf + swq(base + i + 6 * d, q));
    const float4 y = snake4(dw7<false>(w, win, bias), al2, rc2);
    *reinterpret_cast<uint2*>(aop + sw128_offset(i, 4 * q)) = make_uint2(pack_f16(y.x, y.y), pack_f16(y.z, y.w));
#pragma unroll
    for (int j = 0; j < 6; ++j) win[j] = win[j + 1];
  }
}

// Chain length covering 128 rows with `groups` row groups at dilation d.
__host__ __device__ constexpr int chain_length(int groups, int d) {
  for (int L = 1; L <= kTailRows; ++L) {
    const int full = kTailRows / (L * d), rest = kTailRows - full * L * d;
    if (full * d + (rest < d ? rest : d) <= groups) return L;
  }
  return kTailRows;
}
static_assert(chain_length(64, 1) == 2 && chain_length(64, 3) == 3 && chain_length(64, 9) == 3, "512 threads");
static_assert(chain_length(32, 1) == 4 && chain_length(32, 3) == 5 && chain_length(32, 9) == 5, "256 threads");

// 32 lanes x 8 consecutive fp32 accumulator columns.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
      : "r"(taddr)
      : "memory");
}

// First carry-buffer row of unit u's carried rows (u = 3: the final conv's).
__device__ __forceinline__ constexpr int carry_off(int u) { return u == 0 ? 0 : u == 1 ? 6 : u == 2 ? 24 : 78; }

template <int kThreads>
__global__ void __launch_bounds__(kThreads, 512 / kThreads) tail_kernel(const __grid_constant__ TailArgs a) {
  constexpr int kGroups = kThreads / 8;  // row groups: eight lanes, one channel quad each
  extern __shared__ uint8_t tail_smem_raw[];
  // Aligned by an offset from the shared array (not through an integer), so
  // the compiler keeps every access through it in the shared state space.
  uint8_t* sm = tail_smem_raw + ((1024u - (smem_u32(tail_smem_raw) & 1023u)) & 1023u);
  float* xbuf = reinterpret_cast<float*>(sm + TailSmem::kX);
  float* pbuf = reinterpret_cast<float*>(sm + TailSmem::kP);
  float* qbuf = reinterpret_cast<float*>(sm + TailSmem::kQ);
  uint8_t* aop = sm + TailSmem::kA;
  uint8_t* wop = sm + TailSmem::kW;
  float* carry = reinterpret_cast<float*>(sm + TailSmem::kCarry);
  float* cf = reinterpret_cast<float*>(sm + TailSmem::kCoefs);
  int* misc = reinterpret_cast<int*>(sm + TailSmem::kMisc);
  float* obuf = reinterpret_cast<float*>(sm + TailSmem::kOut);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + TailSmem::kBars);
  uint64_t* xfull = bars;
  uint64_t* mma_done = bars + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q = tid & 7, rg = tid >> 3;  // channel quad and row group in the row-parallel phases
  const int N = a.rows_per_stream;
  const int num_tiles = a.rows / kTailRows;
  // This CTA's contiguous range of tiles, preceded by a discarded warm-up
  // tile when the range starts inside a stream.
  const int t_begin = (int)((long long)blockIdx.x * num_tiles / gridDim.x);
  const int t_end = (int)((long long)(blockIdx.x + 1) * num_tiles / gridDim.x);
  const int t_first = (t_begin < t_end && (t_begin * kTailRows) % N != 0) ? t_begin - 1 : t_begin;

  // ---- one-time setup: barriers, TMEM, coefficients, weights, zero carries
  if (tid == 0) {
    mbar_init(xfull, 1);
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 32);
    tmem_relinquish();
  }
  for (int u = 0; u < 3; ++u) {
    const TailUnitArgs& un = a.unit[u];
    for (int i = tid; i < kTailCoef; i += kThreads) cf[TailSmem::kUnitCoef + u * kTailCoef + i] = __ldg(un.coef + i);
    for (int i = tid; i < kTailC; i += kThreads) {
      cf[TailSmem::kPwBias + u * kTailC + i] = __ldg(un.bias + i);
      cf[TailSmem::kPreA + u * kTailC + i] = __ldg(un.pre_a + i);
      cf[TailSmem::kPreR + u * kTailC + i] = __ldg(un.pre_r + i);
    }
    for (int i = tid; i < kTailW / 16; i += kThreads)
      reinterpret_cast<uint4*>(wop + u * kTailW)[i] = __ldg(reinterpret_cast<const uint4*>(un.wimg) + i);
  }
  for (int i = tid; i < kTailC; i += kThreads) {
    cf[TailSmem::kFinA + i] = __ldg(a.fin_a + i);
    cf[TailSmem::kFinR + i] = __ldg(a.fin_r + i);
  }
  for (int i = tid; i < kTailC * 7; i += kThreads) cf[TailSmem::kFinW + (i % 7) * kTailC + i / 7] = __ldg(a.fin_w + i);
  if (tid == 0) cf[TailSmem::kFinB] = __ldg(a.fin_b);
  for (int i = tid; i < kCarryRows * kTailC; i += kThreads) carry[i] = 0.f;
  fence_async_smem();  // weights written by the generic proxy, read by the tensor core
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dependency_sync();  // plan constants above; the stage input and histories below

  // x of tile t: relative rows [0, 128) into X.
  auto load_x = [&](int t) {
    mbar_arrive_expect_tx(xfull, kXBytes);
    tma_load_2d(xbuf, &a.xmap, 0, t * kTailRows, xfull);
  };
  if (tid == 0 && t_first < t_end) load_x(t_first);
  int loads = t_first < t_end ? 1 : 0;  // x loads issued (counted alike by every thread)
  uint32_t n_mma = 0;                   // MMA groups issued (likewise)
  bool ok = true;
  int k = 0;
  for (int t = t_first; t < t_end && ok; ++t, ++k) {
    const bool discard = t < t_begin;  // the warm-up tile: only its carried rows are kept
    const int m0 = t * kTailRows;
    const int s = m0 / N, t0 = m0 - s * N;  // stream and its first time step in this tile
    const bool first = t0 == 0, last = !discard && t0 + kTailRows == N;
    // Stream slot and window heads (units 0-2, final), when the tile reads or writes a window.
    if (tid < 4 && (first || last)) {
      const int code = stream_code(a.state, s);
      const HistRef& h = tid < 3 ? a.unit[tid].hist : a.fin_hist;
      misc[tid] = (a.state.pool && !(code & 2)) ? head_table(slot_base(a.state, code), code & 1)[h.index] : 0;
      if (tid == 0) misc[4] = code;
    }
    ok = __syncthreads_and(mbar_wait(xfull, k & 1, a.status, kDevTimeoutLoader));
    if (!ok) break;
    const int code = misc[4];
    // Rows before relative row 0 of unit u's Snake_pre input in P (u = 3: of
    // Snake_final(y3) in Q): the history window at a stream's first tile, the
    // previous tile's carried rows inside a stream.
    auto fill_halo = [&](int u) {
      const int H = u == 0 ? 6 : u == 1 ? 18 : u == 2 ? 54 : 6;
      const HistRef& hist = u < 3 ? a.unit[u].hist : a.fin_hist;
      float* buf = u < 3 ? pbuf : qbuf;
      const int row0 = u < 3 ? kPOff - H : kQOff - 6;  // buffer row of relative row -H
      for (int j = rg; j < H; j += kGroups)
        *reinterpret_cast<float4*>(buf + swq(row0 + j, q)) =
            first ? hist_quad(a.state, hist, code, misc[u], j - H, q) : lds4(carry + (carry_off(u) + j) * 32 + 4 * q);
    };

#pragma unroll
    for (int u = 0; u < 3; ++u) {
      const int d = u == 0 ? 1 : u == 1 ? 3 : 9, H = 6 * d;
      // Unit input y: x in X for unit 0, y1 / y2 in Q for units 1 and 2. The
      // output y (Snake_final(y3) after unit 2) goes to Q, over the input.
      const float* in = u == 0 ? xbuf : qbuf;
      const int in_row0 = u == 0 ? 0 : kQOff;  // buffer row of relative row 0 of the input
      const HistRef& hist = a.unit[u].hist;
      const float* uc = cf + TailSmem::kUnitCoef + u * kTailCoef;
      // (a) P = Snake_pre(input) rows [0, 128) (units 1 and 2: written by the
      // previous unit's epilogue) and the H rows before them (fill_halo; for
      // units 1 and 2 in the previous unit's epilogue phase, whose rows are
      // disjoint from these).
      if (u == 0) {
        const float4 pa = lds4(cf + TailSmem::kPreA + 4 * q);
        const float4 pr = lds4(cf + TailSmem::kPreR + 4 * q);
        for (int i = rg; i < kTailRows; i += kGroups)
          *reinterpret_cast<float4*>(pbuf + swq(kPOff + i, q)) = snake4(lds4(xbuf + swq(i, q)), pa, pr);
        fill_halo(0);
        __syncthreads();
      }
      // (b) A = Snake_post(depthwise(P)) in f16.
      if (u == 0) {
        depthwise_chains<chain_length(kGroups, 1)>(uc, pbuf, aop, rg, q, 1);
      } else if (u == 1) {
        depthwise_chains<chain_length(kGroups, 3)>(uc, pbuf, aop, rg, q, 3);
      } else {
        depthwise_chains<chain_length(kGroups, 9)>(uc, pbuf, aop, rg, q, 9);
      }
      // The unit's last H input rows: carried to the next tile, and at the
      // stream's last tile the new history window.
      for (int j = rg; j < H; j += kGroups) {
        const float4 v = lds4(pbuf + swq(kPOff + kTailRows - H + j, q));
        *reinterpret_cast<float4*>(carry + (carry_off(u) + j) * 32 + 4 * q) = v;
        if (last && a.state.pool)
          *reinterpret_cast<float4*>(hist_new_row(a.state, hist, code, misc[u], N - H + j, N) + 4 * q) = v;
      }
      fence_async_smem();
      tc_fence_before();
      __syncthreads();
      // (c) D = A W^T, M = 128, N = 32, K = 32 (two K = 16 steps).
      if (tid == 0) {
        tc_fence_after();
        const uint32_t a0 = smem_u32(aop), b0 = smem_u32(wop + u * kTailW);
        constexpr uint32_t idesc = instr_desc_f16(0u, kTailC);
#pragma unroll
        for (int ks = 0; ks < 2; ++ks)
          mma_f16(tmem, smem_desc_sw128(a0 + ks * 32), smem_desc_sw128(b0 + ks * 32), idesc, ks ? 1u : 0u);
        mma_commit(mma_done);
      }
      ++n_mma;
      ok = __syncthreads_and(mbar_wait(mma_done, (n_mma - 1) & 1, a.status, kDevTimeoutMma));
      tc_fence_after();
      if (!ok) break;
      // (d) y = input + (D + b) into Q row kQOff + i, with Snake_pre of the
      // next unit into P row kPOff + i; unit 2 keeps Snake_final(y). A lane
      // reads TMEM lane i (its warp's lane quarter) and owns row i's columns
      // of its column group, so the in-place update reads and writes only the
      // thread's own elements.
      const float* pb = cf + TailSmem::kPwBias + u * kTailC;
      auto finish = [&](int i, int q4, const uint32_t* r) {
        const float4 b = lds4(pb + 4 * q4);
        const int ib = in_row0 + i;
        const float4 x = lds4(in + swq(ib, q4));
        float4 y = make_float4(x.x + (__uint_as_float(r[0]) + b.x), x.y + (__uint_as_float(r[1]) + b.y),
                               x.z + (__uint_as_float(r[2]) + b.z), x.w + (__uint_as_float(r[3]) + b.w));
        if (u == 2) {
          y = snake4(y, lds4(cf + TailSmem::kFinA + 4 * q4), lds4(cf + TailSmem::kFinR + 4 * q4));
        } else {
          *reinterpret_cast<float4*>(pbuf + swq(kPOff + i, q4)) =
              snake4(y, lds4(cf + TailSmem::kPreA + (u + 1) * kTailC + 4 * q4),
                     lds4(cf + TailSmem::kPreR + (u + 1) * kTailC + 4 * q4));
        }
        *reinterpret_cast<float4*>(qbuf + swq(kQOff + i, q4)) = y;
      };
      {
        const int lq = warp & 3, cg = warp >> 2;  // lane quarter, column group
        const int i = lq * 32 + lane;
        if constexpr (kThreads == 512) {
          uint32_t r[8];  // four groups of 8 columns
          tmem_ld8(tmem + ((uint32_t)(lq * 32) << 16) + (uint32_t)(cg * 8), r);
#pragma unroll
          for (int j = 0; j < 2; ++j) finish(i, cg * 2 + j, r + 4 * j);
        } else {
          uint32_t r[16];  // two groups of 16 columns
          tmem_ld16_async(tmem + ((uint32_t)(lq * 32) << 16) + (uint32_t)(cg * 16), r);
          tmem_wait_ld(r);
#pragma unroll
          for (int j = 0; j < 4; ++j) finish(i, cg * 4 + j, r + 4 * j);
        }
      }
      // The next unit's halo rows (after unit 2: the final conv's).
      fill_halo(u + 1);
      tc_fence_before();
      __syncthreads();
      // X has had its last reader (unit 0): the next tile's x box goes in now.
      if (u == 0 && t + 1 < t_end) {
        if (tid == 0) load_x(t + 1);
        ++loads;
      }
    }
    if (!ok) break;
    // Final conv over Q = Snake_final(y3), rows [0, 134) = relative [-6, 128).
    // Each row group of eight lanes (one channel quad each) walks a chain of
    // consecutive output rows with the seven taps sliding through registers:
    // one accumulator per channel (taps oldest first), then the quad's sum and
    // a butterfly over the eight lanes, which leaves every lane the same total.
    {
      constexpr int L = kTailRows / kGroups;
      const float* fw = cf + TailSmem::kFinW;
      float4 w[7], win[7];
#pragma unroll
      for (int j = 0; j < 7; ++j) w[j] = lds4(fw + j * kTailC + 4 * q);
#pragma unroll
      for (int j = 0; j < 6; ++j) win[j] = lds4(qbuf + swq(rg * L + j, q));
      const float fb = cf[TailSmem::kFinB];
#pragma unroll
      for (int c = 0; c < L; ++c) {
        const int o = rg * L + c;
        win[6] = lds4(qbuf + swq(o + 6, q));
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 7; ++j) {
          acc.x = fmaf(w[j].x, win[j].x, acc.x);
          acc.y = fmaf(w[j].y, win[j].y, acc.y);
          acc.z = fmaf(w[j].z, win[j].z, acc.z);
          acc.w = fmaf(w[j].w, win[j].w, acc.w);
        }
        float sum = (acc.x + acc.y) + (acc.z + acc.w);
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        sum += __shfl_xor_sync(0xffffffffu, sum, 4);
        if (q == 0) {
          const float y = tanhf(sum + fb);
          // The reference checks the audio is finite (gpu.py:182-184).
          if (!discard && !(fabsf(y) <= 1.f)) record_error(a.status, kDevNonFinite);
          obuf[o] = y;
        }
#pragma unroll
        for (int j = 0; j < 6; ++j) win[j] = win[j + 1];
      }
    }
    // The final conv's last six input rows (relative [122, 128)): carried on,
    // and at the stream's end the new window; then the new window heads.
    if (tid < 48) {
      const int m = tid >> 3, qd = tid & 7;
      const float4 v = lds4(qbuf + swq(kQOff + kTailRows - 6 + m, qd));
      *reinterpret_cast<float4*>(carry + (carry_off(3) + m) * 32 + 4 * qd) = v;
      if (last && a.state.pool)
        *reinterpret_cast<float4*>(hist_new_row(a.state, a.fin_hist, code, misc[3], N - 6 + m, N) + 4 * qd) = v;
    }
    if (last && a.state.pool && tid == 64) {
      for (int u = 0; u < 3; ++u) hist_commit_head(a.state, a.unit[u].hist, code, misc[u], N);
      hist_commit_head(a.state, a.fin_hist, code, misc[3], N);
    }
    __syncthreads();
    if (!discard && tid < 32) {
      // One warp stores the tile's 128 samples as 512 contiguous bytes, whole
      // 128-byte lines whether the audio is device memory or mapped host
      // memory. (obuf is rewritten only after the next tile's barriers.)
      float* dst = a.audio + (size_t)s * a.audio_stride + a.audio_offset + t0;
      if ((reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
        reinterpret_cast<float4*>(dst)[tid] = lds4(obuf + 4 * tid);
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) dst[tid + 32 * c] = obuf[tid + 32 * c];
      }
    }
  }
  // After a timeout: let the last x load and MMA group issued finish before the
  // CTA frees its TMEM and exits (a wait on a finished phase returns at once).
  if (!ok && tid == 0) {
    if (loads > 0) mbar_wait(xfull, (loads - 1) & 1, a.status, kDevTimeoutLoader);
    if (n_mma > 0) mbar_wait(mma_done, (n_mma - 1) & 1, a.status, kDevTimeoutMma);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 32);
}

int g_tail_sms = 0;

}  // namespace

cudaError_t prepare_tail() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&g_tail_sms, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(tail_kernel<512>, cudaFuncAttributeMaxDynamicSharedMemorySize, TailSmem::kAlloc);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(tail_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, TailSmem::kAlloc);
  return e;
}

cudaError_t launch_tail(const TailArgs& a, cudaStream_t stream) {
  if (a.rows <= 0) return cudaSuccess;
  if (a.rows % kTailRows || a.rows_per_stream % kTailRows) return cudaErrorInvalidValue;
  const int tiles = a.rows / kTailRows;
  // At most one tile per SM: one 512-thread CTA per tile. Otherwise two
  // 256-thread CTAs per SM, each over a contiguous range of tiles.
  if (tiles <= g_tail_sms) return launch_overlapped(tail_kernel<512>, tiles, 512, TailSmem::kAlloc, stream, a);
  const int grid = tiles < 2 * g_tail_sms ? tiles : 2 * g_tail_sms;
  return launch_overlapped(tail_kernel<256>, grid, 256, TailSmem::kAlloc, stream, a);
}

}  // namespace fav
