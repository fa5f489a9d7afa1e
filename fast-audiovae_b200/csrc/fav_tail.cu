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
//   y2             rows [0, 128)
//   Snake_pre3(y2) rows [-54, 128) -> depthwise d=9 -> ...
//   Snake_f(y3)    rows [-6, 128)  -> final conv -> audio rows [0, 128)
//
// The rows before row 0 of each Snake_pre input (6d of them) and of Snake_f(y3)
// are the previous tile's last rows, kept in shared memory from one tile to the
// next of the same stream. At a stream's first tile they come from the layers'
// history rings instead, and the stream's last tile writes the new windows.
// A range that starts inside a stream has no previous tile: its first tile
// recomputes the halo from x rows [-84, 128) (6 + 18 + 54 + 6 rows, two M
// tiles per unit). Stage 5 has 1920 rows per frame, a multiple of 128, so a
// tile never straddles two streams. Every row is computed by the same
// instructions wherever it is computed, so carried, recomputed and history
// rows agree, and a stream decoded in chunks equals the same stream decoded at
// once, bit for bit.
//
// The 32 x 32 projections run on the tensor cores (tcgen05.mma kind::f16, M =
// 128 (x 2 for a recomputed halo), N = 32, K = 32, fp32 accumulators in TMEM); depthwise convs,
// Snake, skip adds and the final conv run on the CUDA cores, 512 threads per
// CTA, in the operation order of the per-layer kernels.
#include "fav_common.cuh"

namespace fav {
namespace {

constexpr int kTailThreads = 512;
constexpr int kTailRows = 128;   // output rows per tile
constexpr int kTailHalo = 84;    // x rows before the tile: 6 + 18 + 54 + 6
constexpr int kTailIn = kTailRows + kTailHalo;
static_assert(kTailIn == kTailBoxRows, "x box of a tile with its halo");
constexpr int kCompactRow0 = kTailIn - kTailCompactBoxRows;  // buffer row of a carried tile's box
static_assert(kCompactRow0 % 8 == 0, "a box starts on a 1024-byte boundary of the swizzled buffer");
constexpr uint32_t kBoxBytes = kTailBoxRows * 128;
constexpr uint32_t kCompactBoxBytes = kTailCompactBoxRows * 128;
constexpr int kCarryRows = 6 + 18 + 54 + 6;  // carried input rows of units 0-2 and the final conv
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

// Depthwise k=7 (dilation d) + Snake_post of A rows [0, n_out) into the f16 A
// operand, A row i from p rows base + i + j*d (j = 0..6), for this thread's
// chain of L rows in channel quad q.
template <int L>
__device__ __forceinline__ void depthwise_chains(const float* uc, const float* pbuf, uint8_t* aop, int rg, int q, int d,
                                                 int n_out, int base) {
  const int i0 = (rg / d) * L * d + rg % d;
  if (i0 >= n_out) return;
  float4 w[7], win[7];
#pragma unroll
  for (int j = 0; j < 7; ++j) w[j] = lds4(uc + j * 64 + 4 * q);
  const float4 bias = lds4(uc + 7 * 64 + 4 * q), al2 = lds4(uc + 8 * 64 + 4 * q), rc2 = lds4(uc + 9 * 64 + 4 * q);
#pragma unroll
  for (int j = 0; j < 6; ++j) win[j] = lds4(pbuf + swq(base + i0 + j * d, q));
#pragma unroll
  for (int c = 0; c < L; ++c) {
    const int i = i0 + c * d;
    if (i >= n_out) break;
    win[6] = lds4(pbuf + swq(base + i + 6 * d, q));
    const float4 y = snake4(dw7<false>(w, win, bias), al2, rc2);
    *reinterpret_cast<uint2*>(aop + sw128_offset(i, 4 * q)) = make_uint2(pack_f16(y.x, y.y), pack_f16(y.z, y.w));
#pragma unroll
    for (int j = 0; j < 6; ++j) win[j] = win[j + 1];
  }
}

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

__global__ void __launch_bounds__(kTailThreads, 1) tail_kernel(const __grid_constant__ TailArgs a) {
  extern __shared__ uint8_t tail_smem_raw[];
  // Aligned by an offset from the shared array (not through an integer), so
  // the compiler keeps every access through it in the shared state space.
  uint8_t* sm = tail_smem_raw + ((1024u - (smem_u32(tail_smem_raw) & 1023u)) & 1023u);
  float* xbuf[2] = {reinterpret_cast<float*>(sm + TailSmem::kX0), reinterpret_cast<float*>(sm + TailSmem::kX1)};
  float* pbuf = reinterpret_cast<float*>(sm + TailSmem::kP);
  float* qbuf = reinterpret_cast<float*>(sm + TailSmem::kQ);
  uint8_t* aop = sm + TailSmem::kA;
  uint8_t* wop = sm + TailSmem::kW;
  float* carry = reinterpret_cast<float*>(sm + TailSmem::kCarry);
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
  // This CTA's contiguous range of tiles: consecutive tiles of one stream
  // carry each unit's last 6d input rows (and the final conv's last six) in
  // shared memory instead of recomputing them. Only a range that starts inside
  // a stream recomputes its first tile's 84-row halo from x.
  const int t_begin = (int)((long long)blockIdx.x * num_tiles / gridDim.x);
  const int t_end = (int)((long long)(blockIdx.x + 1) * num_tiles / gridDim.x);

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

  // x of tile t into buffer b: a warm tile (its 84-row halo recomputed) takes
  // relative rows [-84, 128) into buffer rows [0, 212); any other tile rows
  // [-4, 128) into buffer rows [80, 212) (row 80: a 1024-byte boundary of the
  // swizzled buffer).
  auto load_x = [&](int t, int b, bool warm) {
    if (warm) {
      mbar_arrive_expect_tx(&xfull[b], kBoxBytes);
      tma_load_2d(xbuf[b], &a.xmap, 0, t * kTailRows - kTailHalo, &xfull[b]);
    } else {
      mbar_arrive_expect_tx(&xfull[b], kCompactBoxBytes);
      tma_load_2d(xbuf[b] + kCompactRow0 * 32, &a.xmap_c, 0, t * kTailRows - (kTailHalo - kCompactRow0), &xfull[b]);
    }
  };
  if (tid == 0 && t_begin < t_end) load_x(t_begin, 0, (t_begin * kTailRows) % N != 0);

  bool ok = true;
  bool issued_next = false;  // this iteration started the next tile's x load
  uint32_t n_mma = 0;
  int k = 0;
  for (int t = t_begin; t < t_end && ok; ++t, ++k) {
    const int buf = k & 1;
    const int m0 = t * kTailRows;
    const int s = m0 / N, t0 = m0 - s * N;  // stream and its first time step in this tile
    const bool first = t0 == 0, last = t0 + kTailRows == N;
    const bool warm = k == 0 && !first;  // the range starts inside a stream: halo recomputed
    // Next tile's x into the other buffer (free: the previous tile has ended).
    issued_next = t + 1 < t_end;
    if (tid == 0 && issued_next) load_x(t + 1, buf ^ 1, false);
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
      const int hb = in_off - H;                          // buffer row of relative row -H
      const float* in = u == 1 ? qbuf : xb;     // unit input y (x for unit 0)
      float* out = u == 0 ? qbuf : u == 1 ? xb : qbuf;  // y1 -> q, y2 -> x buffer, Snake_f(y3) -> q
      const HistRef& hist = a.unit[u].hist;
      const float* uc = cf + TailSmem::kUnitCoef + u * kTailCoef;
      // A warm tile computes relative rows [H - in_off, 128) (its halo too:
      // two M tiles), A row i = relative row i + H - in_off; any other tile
      // relative rows [0, 128) (one M tile), A row i = relative row i.
      const int n_out = warm ? kTailRows + in_off - H : kTailRows;
      const int a_base = warm ? 0 : hb;  // p row of A row 0's oldest tap
      const int q = tid & 7, rg = tid >> 3;
      // (a) p = Snake_pre(input) over the rows this tile computes (units 1 and
      // 2: written by the previous unit's epilogue), and the H rows before
      // relative row 0: the history window at a stream's first tile, the
      // previous tile's carried rows inside a stream.
      if (u == 0) {
        const float4 pa = lds4(cf + TailSmem::kPreA + 4 * q);
        const float4 pr = lds4(cf + TailSmem::kPreR + 4 * q);
        for (int i = (warm ? 0 : in_off) + rg; i < kTailIn; i += kTailThreads / 8)
          *reinterpret_cast<float4*>(pbuf + swq(i, q)) = snake4(lds4(in + swq(i, q)), pa, pr);
      }
      if (first) {
        for (int j = rg; j < H; j += kTailThreads / 8)
          *reinterpret_cast<float4*>(pbuf + swq(hb + j, q)) = hist_quad(a.state, hist, code, misc[u], j - H, q);
      } else if (!warm) {
        for (int j = rg; j < H; j += kTailThreads / 8)
          *reinterpret_cast<float4*>(pbuf + swq(hb + j, q)) = lds4(carry + (carry_off(u) + j) * 32 + 4 * q);
      }
      __syncthreads();
      // (b) A = Snake_post(depthwise(p)) in f16. A thread's rows form a chain
      // i0, i0 + d, ... (blocks of L*d rows split into d chains of L), so the
      // seven taps slide through registers: L = 4 covers a warm unit 0's 206
      // rows with 64 row groups, L = 2 a carried unit 0's 128, L = 3 the others.
      if (warm && u == 0) {
        depthwise_chains<4>(uc, pbuf, aop, rg, q, 1, n_out, a_base);
      } else if (u == 0) {
        depthwise_chains<2>(uc, pbuf, aop, rg, q, 1, n_out, a_base);
      } else {
        depthwise_chains<3>(uc, pbuf, aop, rg, q, d, n_out, a_base);
      }
      // The unit's last H input rows: carried to the next tile, and at the
      // stream's last tile the new history window.
      for (int j = rg; j < H; j += kTailThreads / 8) {
        const float4 v = lds4(pbuf + swq(in_off + kTailRows - H + j, q));
        *reinterpret_cast<float4*>(carry + (carry_off(u) + j) * 32 + 4 * q) = v;
        if (last && a.state.pool) *reinterpret_cast<float4*>(hist_new_row(a.state, hist, code, misc[u], N - H + j, N) + 4 * q) = v;
      }
      fence_async_smem();
      tc_fence_before();
      __syncthreads();
      // (c) D[mt] = A[mt] W^T for the M tiles, K = 32 (two K = 16 steps).
      if (tid == 0) {
        tc_fence_after();
        const uint32_t a0 = smem_u32(aop), b0 = smem_u32(wop + u * kTailW);
        constexpr uint32_t idesc = instr_desc_f16(0u, kTailC);
        for (int mt = 0; mt < (warm ? 2 : 1); ++mt)
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
      // (d) y = input + (D + b), with Snake_pre of the next unit into p (the
      // next unit's input rows); unit 2 keeps Snake_final(y). A row i lands
      // in buffer row a_base + i of the output (whose relative row 0 is at
      // in_off - H) and reads its skip from input row a_base + i + H.
      const int lq = warp & 3;
      const float* pb = cf + TailSmem::kPwBias + u * kTailC;
      auto finish = [&](int i, int q4, const uint32_t* r) {
        const int ob = a_base + i;  // out / p buffer row of A row i
        const float4 b = lds4(pb + 4 * q4);
        const float4 x = lds4(in + swq(ob + H, q4));
        float4 y = make_float4(x.x + (__uint_as_float(r[0]) + b.x), x.y + (__uint_as_float(r[1]) + b.y),
                               x.z + (__uint_as_float(r[2]) + b.z), x.w + (__uint_as_float(r[3]) + b.w));
        if (u == 2) {
          y = snake4(y, lds4(cf + TailSmem::kFinA + 4 * q4), lds4(cf + TailSmem::kFinR + 4 * q4));
        } else {
          *reinterpret_cast<float4*>(pbuf + swq(ob, q4)) =
              snake4(y, lds4(cf + TailSmem::kPreA + (u + 1) * kTailC + 4 * q4),
                     lds4(cf + TailSmem::kPreR + (u + 1) * kTailC + 4 * q4));
        }
        *reinterpret_cast<float4*>(out + swq(ob, q4)) = y;
      };
      if (warm) {
        const int mt = (warp >> 2) & 1, half = warp >> 3;
        const int i = mt * kTileM + lq * 32 + lane;
        uint32_t r[16];
        tmem_ld16_async(tmem + ((uint32_t)(lq * 32) << 16) + (uint32_t)(mt * kTailC + half * 16), r);
        tmem_wait_ld(r);
        if (i < n_out) {
#pragma unroll
          for (int j = 0; j < 4; ++j) finish(i, half * 4 + j, r + 4 * j);
        }
      } else {
        // One M tile: 16 warps as 4 lane quarters x 4 groups of 8 columns.
        const int cg = warp >> 2;
        uint32_t r[8];
        tmem_ld8(tmem + ((uint32_t)(lq * 32) << 16) + (uint32_t)(cg * 8), r);
        const int i = lq * 32 + lane;
#pragma unroll
        for (int j = 0; j < 2; ++j) finish(i, cg * 2 + j, r + 4 * j);
      }
      tc_fence_before();
      __syncthreads();
    }
    if (!ok) break;
    // Final conv over q = Snake_final(y3), rows [0, 134) = relative [-6, 128):
    // rows [0, 6) from the final history at a stream's first tile, from the
    // previous tile inside a stream (computed by a warm tile); the last six
    // rows are carried on, and written as the new window at the stream's end.
    if (tid < 48 && !warm) {
      const int m = tid >> 3, q = tid & 7;
      *reinterpret_cast<float4*>(qbuf + swq(m, q)) =
          first ? hist_quad(a.state, a.fin_hist, code, misc[3], m - 6, q) : lds4(carry + (carry_off(3) + m) * 32 + 4 * q);
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
      // The final conv's last six rows, carried to the next tile.
      if (tid >= 128 && tid < 128 + 48) {
        const int m = (tid - 128) >> 3, q = (tid - 128) & 7;
        *reinterpret_cast<float4*>(carry + (carry_off(3) + m) * 32 + 4 * q) = lds4(qbuf + swq(kTailRows + m, q));
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
