// Fused residual stage: the three residual units of a stage with C = 64 or 128
// channels (stages 4 and 3) and the split-bf16 planes of the next transposed
// conv's activated input, in one persistent kernel (the reference's
// mps_decoder.py _Residual.decode loop and the next _Stage.decode prologue,
// restated in the fp32 oracle at oracle/decoder.py).
//
// As per-layer kernels each unit moves y, its f16 Snake_pre(y) and the skip
// input through HBM around a C x C projection. Here a CTA takes a contiguous
// range of 128-row tiles (time steps of one stream; a stream's last tile may
// be partial) and keeps every intermediate in shared memory. Within a tile,
// with row 0 its first row:
//
//   P = f16 Snake_pre1(x)  rows [-6, 128)  -> depthwise d=1 -> Snake -> f16 A -> MMA
//   y1 = x + (A W1 + b1)   rows [0, 128)   (over x in X)
//   P = f16 Snake_pre2(y1) rows [-18, 128) -> depthwise d=3 -> ...
//   y2                     (over y1)
//   P = f16 Snake_pre3(y2) rows [-54, 128) -> depthwise d=9 -> ...
//   y3 -> split-bf16 planes of Snake(y3 * scale + offset) for the next conv
//
// The rows before row 0 of each P come from the previous tile of the same
// stream (kept in a small carry buffer) or, at a stream's first tile, from
// the unit's history ring; a stream's last tile writes the new windows. A
// range that starts inside a stream first runs the tile before it as a
// warm-up tile with zero carried rows and discards its output (the zeros
// reach its rows [0, 6) of y1, [0, 24) of y2 and [0, 78) of y3; the rows it
// carries on are exact). Every value is computed with the same operations, in
// the same order and at the same roundings as the per-layer kernels (f16
// Snake_pre staging, fused multiply-add depthwise chains, f16 x f16 MMAs over
// the K blocks in order, the planes epilogue), so the fused stage equals them
// bit for bit and a chunked stream equals the same stream decoded at once.
//
// The C x C projections run on the tensor cores (tcgen05.mma kind::f16, M =
// 128, N = C, fp32 accumulators in TMEM); the unit's B operand is streamed
// into shared memory by a bulk copy while the previous unit finishes. The
// phases of a tile are separated by block barriers: C = 64 runs two CTAs of
// 256 threads per SM, whose phases interleave (one 512-thread CTA per tile
// when a launch has at most one tile per SM); C = 128 runs one 512-thread CTA
// per SM. Stage 2 (C = 256) keeps y in TMEM instead (stage256_kernel below).
#include "fav_common.cuh"

namespace fav {
namespace {

constexpr int kSR = 128;                 // rows per tile
constexpr int kSPOff = 54;               // P row of relative row 0 (rows [-54, 128))
constexpr int kSPRows = kSPOff + kSR;    // 182
constexpr int kSCarryRows = 6 + 18 + 54;  // carried P rows of units 0-2

template <int C>
struct StageSmem {
  static constexpr int kXBlocks = C / 32;  // fp32 column blocks (128-byte rows, TMA boxes)
  static constexpr int kKB = C / 64;       // f16 column blocks (128-byte rows): K blocks
  // byte offsets from the 1024-aligned base
  static constexpr int kX = 0;                               // y: [kXBlocks][128][32] fp32, 128-byte swizzle
  static constexpr int kA = kX + kXBlocks * kSR * 128;       // A: [kKB][128][64] f16 (MMA layout)
  static constexpr int kW = kA + kKB * kSR * 128;            // one unit's B: [kKB][C][64] f16 (MMA layout)
  static constexpr int kP = kW + kKB * C * 128;              // P: [kKB][182][64] f16, 16-byte chunks swizzled
  static constexpr int kCarry = kP + kKB * kSPRows * 128;    // [78][C] f16, plain rows
  static constexpr int kCoefs = kCarry + kSCarryRows * C * 2;  // floats from here on
  static constexpr int kUnitCoefFloats = kKB * kCoefResidual * 64;
  static constexpr int kUnitCoef = 0;                        // [3][kKB][w0..w6, bias, alpha2, recip2][64]
  static constexpr int kPwBias = 3 * kUnitCoefFloats;        // [3][C]
  static constexpr int kPreA = kPwBias + 3 * C;              // [3][C]
  static constexpr int kPreR = kPreA + 3 * C;                // [3][C]
  static constexpr int kNScale = kPreR + 3 * C;              // [C] next stage's affine and Snake
  static constexpr int kNOffset = kNScale + C;
  static constexpr int kNAlpha = kNOffset + C;
  static constexpr int kNRecip = kNAlpha + C;
  static constexpr int kCoefFloats = kNRecip + C;
  static constexpr int kMisc = kCoefs + kCoefFloats * 4;     // ints: heads[4], code, pad
  static constexpr int kBars = ((kMisc + 8 * 4 + 7) / 8) * 8;  // xfull, wfull, mma_done, tmem slot
  static constexpr int kBytes = kBars + 4 * 8;
  static constexpr int kAlloc = kBytes + 1024;
};
// C = 64: two CTAs per SM (228 KB of shared memory per SM, 1 KB of it reserved per CTA).
static_assert(2 * (StageSmem<64>::kAlloc + 1024) <= 228 * 1024, "two C=64 stage CTAs per SM");
static_assert(StageSmem<128>::kAlloc <= 227 * 1024, "one C=128 stage CTA per SM");

// fp32 row buffers (X): row r, channel quad q (< 8) of a 32-channel block in
// the 128-byte swizzle a TMA box with CU_TENSOR_MAP_SWIZZLE_128B writes.
__device__ __forceinline__ int xq_off(int r, int q) { return r * 32 + ((q ^ (r & 7)) << 2); }

// P: f16 row pr, channel quad q (4 channels, 8 bytes) of the whole row (block
// q / 16), with the 16-byte chunks of each 128-byte row swizzled by pr & 7 so
// a lane per row (epilogue writes) spreads over the banks.
__device__ __forceinline__ int p_off(int pr, int q) {
  const int kb = q >> 4, qb = q & 15;
  return kb * kSPRows * 128 + pr * 128 + ((((qb >> 1) ^ (pr & 7)) << 4) | ((qb & 1) << 3));
}
__device__ __forceinline__ float4 p_load(const uint8_t* p, int pr, int q) {
  const uint2 h = *reinterpret_cast<const uint2*>(p + p_off(pr, q));
  const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
  const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&h.y));
  return make_float4(lo.x, lo.y, hi.x, hi.y);
}
__device__ __forceinline__ uint2 f16x4(float4 v) { return make_uint2(pack_f16(v.x, v.y), pack_f16(v.z, v.w)); }
__device__ __forceinline__ float4 f16x4_to_float(uint2 h) {
  const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
  const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&h.y));
  return make_float4(lo.x, lo.y, hi.x, hi.y);
}

__device__ __forceinline__ int stage_code(const StateRef& st, int s) {
  return st.slot_codes ? st.slot_codes[s] : ((s << 2) | st.uniform_code);
}

// Window row of time tp (-H <= tp < 0) of a history whose window starts at head.
__device__ __forceinline__ float4 stage_hist_quad(const StateRef& st, const HistRef& h, int code, int head, int tp,
                                                  int q) {
  if (!st.pool || (code & 2)) return make_float4(0.f, 0.f, 0.f, 0.f);
  int row = head + h.rows + tp;
  if (row >= 2 * h.rows) row -= 2 * h.rows;
  return ldg4(slot_base(st, code) + h.ring + row * h.width + 4 * q);
}

// First carry row of unit u's carried P rows.
__device__ __forceinline__ constexpr int scarry_off(int u) { return u == 0 ? 0 : u == 1 ? 6 : 24; }

// Chain length covering 128 rows with `groups` row groups at dilation d.
__host__ __device__ constexpr int stage_chain(int groups, int d) {
  for (int L = 1; L <= kSR; ++L) {
    const int full = kSR / (L * d), rest = kSR - full * L * d;
    if (full * d + (rest < d ? rest : d) <= groups) return L;
  }
  return kSR;
}

// Depthwise k=7 (dilation d) + Snake_post of A rows [0, 128) into the f16 A
// operand, A row i from P rows kSPOff - 6d + i + j*d (j = 0..6), for this
// thread's chain of L rows i0, i0 + d, ... in channel quad q: blocks of L*d
// rows split into d chains of L, so the seven taps slide through registers.
template <int L>
__device__ __forceinline__ void stage_chains(const float* ucoef, const uint8_t* pbuf, uint8_t* aop, int rg, int q,
                                             int d) {
  const int i0 = (rg / d) * L * d + rg % d;
  if (i0 >= kSR) return;
  const int kb = q >> 4, qb = q & 15;
  const float* uc = ucoef + kb * kCoefResidual * 64 + 4 * qb;
  uint8_t* ab = aop + kb * kSR * 128;
  const int base = kSPOff - 6 * d;
  float4 w[7], win[7];
#pragma unroll
  for (int j = 0; j < 7; ++j) w[j] = lds4(uc + j * 64);
  const float4 bias = lds4(uc + 7 * 64), al2 = lds4(uc + 8 * 64), rc2 = lds4(uc + 9 * 64);
#pragma unroll
  for (int j = 0; j < 6; ++j) win[j] = p_load(pbuf, base + i0 + j * d, q);
#pragma unroll
  for (int c = 0; c < L; ++c) {
    const int i = i0 + c * d;
    if (i >= kSR) break;
    win[6] = p_load(pbuf, base + i + 6 * d, q);
    *reinterpret_cast<uint2*>(ab + sw128_offset(i, 4 * qb)) = f16x4(snake4(dw7<false>(w, win, bias), al2, rc2));
#pragma unroll
    for (int j = 0; j < 6; ++j) win[j] = win[j + 1];
  }
}

template <int C, int kThreads>
__global__ void __launch_bounds__(kThreads, 512 / kThreads) stage_kernel(const __grid_constant__ StageArgs a) {
  using L = StageSmem<C>;
  constexpr int kQuads = C / 4;                 // channel quads per row
  constexpr int kGroups = kThreads / kQuads;    // row groups of the row-parallel phases
  constexpr int kColGroups = kThreads / 128;    // warps per TMEM lane quarter
  constexpr int kCW = C / kColGroups;           // epilogue columns per thread (16 or 32)
  constexpr int kKB = L::kKB;
  constexpr uint32_t kXBytes = L::kXBlocks * kSR * 128;
  constexpr uint32_t kWBytes = kKB * C * 128;
  static_assert(kThreads % kQuads == 0 && kCW % 16 == 0, "thread mapping");
  extern __shared__ uint8_t stage_smem_raw[];
  // Aligned by an offset from the shared array (not through an integer), so
  // the compiler keeps every access through it in the shared state space.
  uint8_t* sm = stage_smem_raw + ((1024u - (smem_u32(stage_smem_raw) & 1023u)) & 1023u);
  float* xbuf = reinterpret_cast<float*>(sm + L::kX);
  uint8_t* aop = sm + L::kA;
  uint8_t* wop = sm + L::kW;
  uint8_t* pbuf = sm + L::kP;
  uint8_t* carry = sm + L::kCarry;
  float* cf = reinterpret_cast<float*>(sm + L::kCoefs);
  int* misc = reinterpret_cast<int*>(sm + L::kMisc);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::kBars);
  uint64_t* xfull = bars;
  uint64_t* wfull = bars + 1;
  uint64_t* mma_done = bars + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t wl = a.wait_limit ? a.wait_limit : kWaitLimit;  // polls before a wait gives up
  const int q = tid % kQuads, rg = tid / kQuads;  // channel quad and row group in the row-parallel phases
  const int N = a.rows_per_stream;
  const int tps = (N + kSR - 1) / kSR;  // tiles per stream (the last one may be partial)
  const int num_tiles = (a.rows / N) * tps;
  // This CTA's contiguous range of tiles, preceded by a discarded warm-up
  // tile when the range starts inside a stream.
  const int t_begin = (int)((long long)blockIdx.x * num_tiles / gridDim.x);
  const int t_end = (int)((long long)(blockIdx.x + 1) * num_tiles / gridDim.x);
  const int t_first = (t_begin < t_end && t_begin % tps != 0) ? t_begin - 1 : t_begin;

  // ---- one-time setup: barriers, TMEM, coefficients, zero carries
  if (tid == 0) {
    mbar_init(xfull, 1);
    mbar_init(wfull, 1);
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, C);
    tmem_relinquish();
  }
  for (int u = 0; u < 3; ++u) {
    const StageUnitArgs& un = a.unit[u];
    for (int i = tid; i < L::kUnitCoefFloats; i += kThreads) cf[L::kUnitCoef + u * L::kUnitCoefFloats + i] = __ldg(un.coef + i);
    for (int i = tid; i < C; i += kThreads) {
      cf[L::kPwBias + u * C + i] = __ldg(un.bias + i);
      cf[L::kPreA + u * C + i] = __ldg(un.pre_a + i);
      cf[L::kPreR + u * C + i] = __ldg(un.pre_r + i);
    }
  }
  for (int i = tid; i < C; i += kThreads) {
    cf[L::kNScale + i] = __ldg(a.next_scale + i);
    cf[L::kNOffset + i] = __ldg(a.next_offset + i);
    cf[L::kNAlpha + i] = __ldg(a.next_alpha + i);
    cf[L::kNRecip + i] = __ldg(a.next_recip + i);
  }
  for (int i = tid; i < kSCarryRows * C / 2; i += kThreads) reinterpret_cast<uint32_t*>(carry)[i] = 0u;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dependency_sync();  // plan constants above; the stage input and histories below

  // y of the tile at global row m0: C / 32 boxes of 32 channels x 128 rows.
  auto load_x = [&](int m0) {
    mbar_arrive_expect_tx(xfull, kXBytes);
#pragma unroll
    for (int b = 0; b < L::kXBlocks; ++b) tma_load_2d(sm + L::kX + b * kSR * 128, &a.xmap, 32 * b, m0, xfull);
  };
  auto load_w = [&](int u) {
    mbar_arrive_expect_tx(wfull, kWBytes);
    bulk_g2s(wop, a.unit[u].wimg, kWBytes, wfull);
  };
  auto tile_m0 = [&](int t) { return (t / tps) * N + (t % tps) * kSR; };
  if (tid == 0 && t_first < t_end) {
    load_x(tile_m0(t_first));
    load_w(0);
  }
  int loads = t_first < t_end ? 1 : 0;   // x loads issued (counted alike by every thread)
  uint32_t n_w = t_first < t_end ? 1 : 0;  // weight loads issued
  uint32_t n_mma = 0;                       // MMA groups issued
  bool ok = true;
  int k = 0;
  for (int t = t_first; t < t_end && ok; ++t, ++k) {
    const bool discard = t < t_begin;  // the warm-up tile: only its carried rows are kept
    const int s = t / tps, j = t - s * tps;
    const int m0 = s * N + j * kSR;
    const int v = min(kSR, N - j * kSR);  // valid rows of the tile
    const bool first = j == 0, last = !discard && j == tps - 1;
    // Stream slot and window heads (units 0-2, the next conv), when the tile reads or writes a window.
    if (tid < 4 && (first || last)) {
      const int code = stage_code(a.state, s);
      const HistRef& h = tid < 3 ? a.unit[tid].hist : a.hist_next;
      misc[tid] = (a.state.pool && !(code & 2)) ? head_table(slot_base(a.state, code), code & 1)[h.index] : 0;
      if (tid == 0) misc[4] = code;
    }
    // The previous tile's plane stores have read their staging tiles (A and
    // P) before this tile writes them; the next tile's rows head into L2.
    if (tid == 0) {
      bulk_wait_read_all();
      if (t + 1 < t_end) {
        const int m1 = tile_m0(t + 1);
        prefetch_l2(a.x + (size_t)m1 * C, (uint32_t)(min(kSR, a.rows - m1) * C * 4));
      }
    }
    ok = __syncthreads_and(mbar_wait(xfull, k & 1, a.status, kDevTimeoutLoader, wl));
    if (!ok) break;
    const int code = misc[4];
    // Rows [-H, 0) of unit u's P: the history window at a stream's first
    // tile, the previous tile's carried rows inside a stream.
    auto fill_halo = [&](int u) {
      const int H = u == 0 ? 6 : u == 1 ? 18 : 54;
      const HistRef& hist = a.unit[u].hist;
      for (int r = rg; r < H; r += kGroups) {
        const uint2 val = first ? f16x4(stage_hist_quad(a.state, hist, code, misc[u], r - H, q))
                                : *reinterpret_cast<const uint2*>(carry + ((scarry_off(u) + r) * C + 4 * q) * 2);
        *reinterpret_cast<uint2*>(pbuf + p_off(kSPOff - H + r, q)) = val;
      }
    };
    // (a) P = f16 Snake_pre1(x), rows [0, 128), and unit 0's halo rows.
    {
      const float4 pa = lds4(cf + L::kPreA + 4 * q);
      const float4 pr = lds4(cf + L::kPreR + 4 * q);
      const float* xb = xbuf + (q >> 3) * kSR * 32;
      for (int i = rg; i < kSR; i += kGroups)
        *reinterpret_cast<uint2*>(pbuf + p_off(kSPOff + i, q)) = f16x4(snake4(lds4(xb + xq_off(i, q & 7)), pa, pr));
      fill_halo(0);
      __syncthreads();
    }
#pragma unroll
    for (int u = 0; u < 3; ++u) {
      const int d = u == 0 ? 1 : u == 1 ? 3 : 9, H = 6 * d;
      const HistRef& hist = a.unit[u].hist;
      const float* uc = cf + L::kUnitCoef + u * L::kUnitCoefFloats;
      // (b) A = Snake_post(depthwise(P)) in f16.
      if (u == 0) {
        stage_chains<stage_chain(kGroups, 1)>(uc, pbuf, aop, rg, q, 1);
      } else if (u == 1) {
        stage_chains<stage_chain(kGroups, 3)>(uc, pbuf, aop, rg, q, 3);
      } else {
        stage_chains<stage_chain(kGroups, 9)>(uc, pbuf, aop, rg, q, 9);
      }
      // The unit's last H input rows: carried to the next tile of the stream
      // (full tiles), and at the stream's last tile the new history window
      // (rows [v - H, v), partly carried rows when v < H).
      if (!last) {
        for (int r = rg; r < H; r += kGroups)
          *reinterpret_cast<uint2*>(carry + ((scarry_off(u) + r) * C + 4 * q) * 2) =
              *reinterpret_cast<const uint2*>(pbuf + p_off(kSPOff + kSR - H + r, q));
      } else if (a.state.pool) {
        for (int r = rg; r < H; r += kGroups) {
          const float4 val = f16x4_to_float(*reinterpret_cast<const uint2*>(pbuf + p_off(kSPOff + v - H + r, q)));
          *reinterpret_cast<float4*>(hist_new_row(a.state, hist, code, misc[u], N - H + r, N) + 4 * q) = val;
        }
      }
      fence_async_smem();
      tc_fence_before();
      __syncthreads();
      // (c) D = A W^T, M = 128, N = C, K = C (K blocks of 64 in order, four K = 16 steps each).
      if (tid == 0) {
        ok = (a.gate == nullptr || n_mma > 0 || flag_wait(a.gate, a.status, kDevTimeoutGate, wl)) &&
             mbar_wait(wfull, (n_w - 1) & 1, a.status, kDevTimeoutLoader, wl);
        if (ok) {
          tc_fence_after();
          const uint32_t a0 = smem_u32(aop), b0 = smem_u32(wop);
          constexpr uint32_t idesc = instr_desc_f16(0u, C);
#pragma unroll
          for (int kb = 0; kb < kKB; ++kb)
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              mma_f16(tmem, smem_desc_sw128(a0 + kb * kSR * 128 + ks * 32), smem_desc_sw128(b0 + kb * C * 128 + ks * 32),
                      idesc, (kb | ks) ? 1u : 0u);
          mma_commit(mma_done);
        }
      }
      if (!__syncthreads_and(ok)) {
        ok = false;
        break;
      }
      ++n_mma;
      ok = __syncthreads_and(mbar_wait(mma_done, (n_mma - 1) & 1, a.status, kDevTimeoutMma, wl));
      tc_fence_after();
      if (!ok) break;
      // The MMAs have read W: the next unit's weights (after unit 2: unit 0's,
      // for the next tile) stream in during this epilogue and the next
      // unit's depthwise phase.
      if (tid == 0 && (u < 2 || t + 1 < t_end)) load_w(u < 2 ? u + 1 : 0);
      if (u < 2 || t + 1 < t_end) ++n_w;
      // (d) y = input + (D + b) over the input in X; units 0-1 write the next
      // unit's f16 Snake_pre(y) into P rows [0, 128) and fill its halo rows
      // (disjoint rows); unit 2 writes the next conv's planes. A lane reads
      // TMEM lane i (its warp's lane quarter) and owns row i's kCW columns.
      {
        const int lq = warp & 3, cg = warp >> 2;
        const int i = lq * 32 + lane;
        const int c0 = cg * kCW;
        uint32_t r[kCW];
#pragma unroll
        for (int h = 0; h < kCW / 16; ++h)
          tmem_ld16_async(tmem + ((uint32_t)(lq * 32) << 16) + (uint32_t)(c0 + 16 * h),
                          *reinterpret_cast<uint32_t(*)[16]>(r + 16 * h));
#pragma unroll
        for (int h = 0; h < kCW / 16; ++h) tmem_wait_ld(*reinterpret_cast<uint32_t(*)[16]>(r + 16 * h));
        const float* pb = cf + L::kPwBias + u * C;
        uint32_t hi[kCW / 2], lo[kCW / 2];  // unit 2: split-bf16 planes of this row's columns
#pragma unroll
        for (int qq = 0; qq < kCW / 4; ++qq) {
          const int c = c0 + 4 * qq;
          float* xp = xbuf + (c >> 5) * kSR * 32 + xq_off(i, (c & 31) >> 2);
          const float4 x = lds4(xp);
          const float4 b = lds4(pb + c);
          const float4 y = make_float4(x.x + (__uint_as_float(r[4 * qq]) + b.x), x.y + (__uint_as_float(r[4 * qq + 1]) + b.y),
                                       x.z + (__uint_as_float(r[4 * qq + 2]) + b.z),
                                       x.w + (__uint_as_float(r[4 * qq + 3]) + b.w));
          if (u < 2) {
            *reinterpret_cast<float4*>(xp) = y;
            *reinterpret_cast<uint2*>(pbuf + p_off(kSPOff + i, c >> 2)) =
                f16x4(snake4(y, lds4(cf + L::kPreA + (u + 1) * C + c), lds4(cf + L::kPreR + (u + 1) * C + c)));
          } else {
            const float4 sc = lds4(cf + L::kNScale + c), of = lds4(cf + L::kNOffset + c);
            float4 w4 = make_float4(__fadd_rn(__fmul_rn(y.x, sc.x), of.x), __fadd_rn(__fmul_rn(y.y, sc.y), of.y),
                                    __fadd_rn(__fmul_rn(y.z, sc.z), of.z), __fadd_rn(__fmul_rn(y.w, sc.w), of.w));
            w4 = snake4(w4, lds4(cf + L::kNAlpha + c), lds4(cf + L::kNRecip + c));
            split_bf16(w4.x, w4.y, hi[2 * qq], lo[2 * qq]);
            split_bf16(w4.z, w4.w, hi[2 * qq + 1], lo[2 * qq + 1]);
          }
        }
        if (u == 2) {
          // This row's planes into the staging tiles the TMA stores read: hi
          // over A (the MMA has read it), lo over P (the depthwise has read
          // it), [C / 64][128 rows][128 B] in the 128-byte swizzle.
#pragma unroll
          for (int e = 0; e < kCW / 8; ++e) {
            const int c = c0 + 8 * e;
            const int off = (c >> 6) * kSR * 128 + sw128_offset(i, c & 63);
            *reinterpret_cast<uint4*>(aop + off) = make_uint4(hi[4 * e], hi[4 * e + 1], hi[4 * e + 2], hi[4 * e + 3]);
            *reinterpret_cast<uint4*>(pbuf + off) = make_uint4(lo[4 * e], lo[4 * e + 1], lo[4 * e + 2], lo[4 * e + 3]);
          }
        }
        if (u == 2 && !discard && i < v) {
          // A stream's first row of the shifted planes holds the conv's history
          // (the previous activated input, packed (hi << 16) | lo); the
          // stream's last row becomes the new history row. (The TMA stores
          // write every other row of both plane copies.)
          const int g = m0 + i, tj = j * kSR + i;
          const size_t plane = (size_t)a.rows * C;
          const bool have = a.state.pool && !(code & 2);
          if (tj == 0) {
            uint4* qh = reinterpret_cast<uint4*>(a.out_planes_prev + (size_t)g * C + c0);
            uint4* ql = reinterpret_cast<uint4*>(a.out_planes_prev + plane + (size_t)g * C + c0);
            const uint4* old = have ? reinterpret_cast<const uint4*>(slot_base(a.state, code) + a.hist_next.ring +
                                                                     misc[3] * a.hist_next.width + c0)
                                    : nullptr;
#pragma unroll
            for (int e = 0; e < kCW / 8; ++e) {
              const uint4 w0 = old ? __ldg(old + 2 * e) : make_uint4(0u, 0u, 0u, 0u);
              const uint4 w1 = old ? __ldg(old + 2 * e + 1) : make_uint4(0u, 0u, 0u, 0u);
              qh[e] = make_uint4(__byte_perm(w0.x, w0.y, 0x7632), __byte_perm(w0.z, w0.w, 0x7632),
                                 __byte_perm(w1.x, w1.y, 0x7632), __byte_perm(w1.z, w1.w, 0x7632));
              ql[e] = make_uint4(__byte_perm(w0.x, w0.y, 0x5410), __byte_perm(w0.z, w0.w, 0x5410),
                                 __byte_perm(w1.x, w1.y, 0x5410), __byte_perm(w1.z, w1.w, 0x5410));
            }
          }
          if (tj == N - 1 && a.state.pool) {  // a fresh stream too (its window starts at head 0)
            uint4* dst = reinterpret_cast<uint4*>(slot_base(a.state, code) + a.hist_next.ring +
                                                  (misc[3] ^ 1) * a.hist_next.width + c0);
#pragma unroll
            for (int e = 0; e < kCW / 4; ++e)
              dst[e] = make_uint4(__byte_perm(lo[2 * e], hi[2 * e], 0x5410), __byte_perm(lo[2 * e], hi[2 * e], 0x7632),
                                  __byte_perm(lo[2 * e + 1], hi[2 * e + 1], 0x5410),
                                  __byte_perm(lo[2 * e + 1], hi[2 * e + 1], 0x7632));
          }
        }
      }
      if (u < 2) fill_halo(u + 1);
      // The stream's advanced heads, before the barrier that ends the tile:
      // after it, threads 1-3 may already write the next tile's heads into misc.
      if (u == 2 && last && a.state.pool && tid == 0) {
        for (int v2 = 0; v2 < 3; ++v2) hist_commit_head(a.state, a.unit[v2].hist, code, misc[v2], N);
        hist_commit_head(a.state, a.hist_next, code, misc[3], N);
      }
      // X was written in place (units 0-1) and the next tile's TMA box goes
      // over it; the staged planes are read by TMA stores: order those
      // generic writes before the async proxy's accesses.
      if (u == 2) fence_async_smem();
      tc_fence_before();
      __syncthreads();
    }
    if (!ok) break;
    // The tile's planes: rows [j*128, j*128 + 128) of stream s, and the same
    // rows one time step later in the shifted planes; the maps' row extent is
    // the stream's N, so rows past the stream's end are not written.
    if (!discard && tid == 0) {
#pragma unroll
      for (int kb = 0; kb < kKB; ++kb) {
        tma_store_4d(&a.planes_map, aop + kb * kSR * 128, 64 * kb, j * kSR, s, 0);
        tma_store_4d(&a.planes_map, pbuf + kb * kSR * 128, 64 * kb, j * kSR, s, 1);
        tma_store_4d(&a.prev_map, aop + kb * kSR * 128, 64 * kb, j * kSR + 1, s, 0);
        tma_store_4d(&a.prev_map, pbuf + kb * kSR * 128, 64 * kb, j * kSR + 1, s, 1);
      }
      bulk_commit();
    }
    // X has had its last reader (unit 2's epilogue): the next tile's y goes in now.
    if (t + 1 < t_end) {
      if (tid == 0) load_x(tile_m0(t + 1));
      ++loads;
    }
  }
  // After a timeout: let the last loads and MMA group issued finish before the
  // CTA frees its TMEM and exits (a wait on a finished phase returns at once).
  if (!ok && tid == 0) {
    if (loads > 0) mbar_wait(xfull, (loads - 1) & 1, a.status, kDevTimeoutLoader);
    if (n_w > 0) mbar_wait(wfull, (n_w - 1) & 1, a.status, kDevTimeoutLoader);
    if (n_mma > 0) mbar_wait(mma_done, (n_mma - 1) & 1, a.status, kDevTimeoutMma);
  }
  if (tid == 0) bulk_wait_all();  // the last plane stores have landed
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, C);
}

// ------------------------------------------------------------ 256 channels
// Stage 2 (256 channels, 240 rows per stream and frame): a tile's y (128 rows
// x 256 channels fp32, 128 KB) does not fit in shared memory beside the
// operands, so y stays in TMEM, columns [0, 256), beside the projection's
// accumulator D, columns [256, 512) (a whole SM's TMEM: one CTA per SM). A
// unit runs two K blocks (128 channels) at a time: f16 Snake_pre of their y
// columns into P (with their carried or history halo rows), the depthwise
// chains into their A tiles, and their MMAs into D while the next pair is
// prepared; then y = y + (D + b) in TMEM. The weights stream through two
// 32 KB K-block buffers. The operations and their order are those
// of the per-layer kernels, so the result is the same bit for bit.
constexpr int kS2C = 256;
struct Stage2Smem {
  // byte offsets from the 1024-aligned base
  static constexpr int kA = 0;                               // A: [4][128][64] f16 (MMA layout); hi-plane staging
  static constexpr int kW = kA + 4 * kSR * 128;              // W: [2][256][64] f16 K blocks; lo-plane staging
  static constexpr int kP = kW + 2 * kS2C * 128;             // P of two K blocks: [2][182][64] f16, swizzled chunks
  static constexpr int kCarry = kP + 2 * kSPRows * 128;      // [78][256] f16, plain rows
  // The current K-block pair's coefficients: depthwise [2][w0..w6, bias,
  // alpha2, recip2][64], then Snake_pre alpha and reciprocal [128] each.
  static constexpr int kRC = kCarry + kSCarryRows * kS2C * 2;
  static constexpr int kRCFloats = 2 * kCoefResidual * 64 + 2 * 128;
  static constexpr int kMisc = kRC + kRCFloats * 4;          // ints: heads[4], code, pad
  static constexpr int kBars = ((kMisc + 8 * 4 + 7) / 8) * 8;    // wfull[2], mma_done[2], tmem slot
  static constexpr int kBytes = kBars + 5 * 8;
  static constexpr int kAlloc = kBytes + 1024;
};
static_assert(Stage2Smem::kAlloc <= 227 * 1024, "one C=256 stage CTA per SM");

__global__ void __launch_bounds__(512, 1) stage256_kernel(const __grid_constant__ StageArgs a) {
  using L = Stage2Smem;
  constexpr int C = kS2C;
  constexpr int kGroups = 512 / 32;  // row groups of the row-parallel phases over two K blocks (32 quads)
  constexpr uint32_t kWBytes = C * 128;
  extern __shared__ uint8_t stage2_smem_raw[];
  uint8_t* sm = stage2_smem_raw + ((1024u - (smem_u32(stage2_smem_raw) & 1023u)) & 1023u);
  uint8_t* aop = sm + L::kA;
  uint8_t* wop = sm + L::kW;
  uint8_t* pbuf = sm + L::kP;
  uint8_t* carry = sm + L::kCarry;
  int* misc = reinterpret_cast<int*>(sm + L::kMisc);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::kBars);
  uint64_t* wfull = bars;         // [2]
  uint64_t* mma_done = bars + 2;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);
  float* rc = reinterpret_cast<float*>(sm + L::kRC);
  // A unit's epilogue coefficients (bias; unit 2: the next stage's affine and
  // Snake), [5][256], kept in P while P is idle (after the unit's last
  // depthwise phase, until the next unit's first Snake_pre phase).
  float* ec = reinterpret_cast<float*>(pbuf);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t wl = a.wait_limit ? a.wait_limit : kWaitLimit;
  const int q = tid & 31, rg = tid >> 5;   // channel quad of a K-block pair and row group
  const int lq = warp & 3, cg = warp >> 2;  // TMEM lane quarter and column group
  const int row = lq * 32 + lane;           // this thread's tile row in the TMEM phases
  const int N = a.rows_per_stream;
  const int tps = (N + kSR - 1) / kSR;
  const int num_tiles = (a.rows / N) * tps;
  const int t_begin = (int)((long long)blockIdx.x * num_tiles / gridDim.x);
  const int t_end = (int)((long long)(blockIdx.x + 1) * num_tiles / gridDim.x);
  const int t_first = (t_begin < t_end && t_begin % tps != 0) ? t_begin - 1 : t_begin;

  if (tid == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&wfull[b], 1);
      mbar_init(&mma_done[b], 1);
    }
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  for (int i = tid; i < kSCarryRows * C / 2; i += 512) reinterpret_cast<uint32_t*>(carry)[i] = 0u;
  // Coefficients of K-block pair kp of unit u into rc (plan constants).
  auto load_round_coefs = [&](int u, int kp) {
    const float* src = a.unit[u].coef + 2 * kp * kCoefResidual * 64;
    for (int i = tid; i < 2 * kCoefResidual * 16; i += 512) reinterpret_cast<float4*>(rc)[i] = ldg4(src + 4 * i);
    if (tid < 32) {
      reinterpret_cast<float4*>(rc + 2 * kCoefResidual * 64)[tid] = ldg4(a.unit[u].pre_a + kp * 128 + 4 * tid);
      reinterpret_cast<float4*>(rc + 2 * kCoefResidual * 64 + 128)[tid] = ldg4(a.unit[u].pre_r + kp * 128 + 4 * tid);
    }
  };
  auto load_epi_coefs = [&](int u) {
    if (tid < 64) reinterpret_cast<float4*>(ec)[tid] = ldg4(a.unit[u].bias + 4 * tid);
    if (u == 2 && tid < 256) {
      const int k = tid >> 6, i = tid & 63;
      const float* src = k == 0 ? a.next_scale : k == 1 ? a.next_offset : k == 2 ? a.next_alpha : a.next_recip;
      reinterpret_cast<float4*>(ec + 256 * (k + 1))[i] = ldg4(src + 4 * i);
    }
  };
  load_round_coefs(0, 0);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t trow = tmem + ((uint32_t)(lq * 32) << 16);  // this warp's TMEM lanes
  grid_dependency_sync();

  // Steps: 12 per tile (unit u, K block kb); step g's weights go to buffer g & 1.
  auto load_w = [&](uint32_t g, int u, int kb) {
    mbar_arrive_expect_tx(&wfull[g & 1], kWBytes);
    bulk_g2s(wop + (g & 1) * kWBytes, a.unit[u].wimg + (size_t)kb * kWBytes, kWBytes, &wfull[g & 1]);
  };
  auto tile_m0 = [&](int t) { return (t / tps) * N + (t % tps) * kSR; };
  if (tid == 0 && t_first < t_end) {
    load_w(0, 0, 0);
    load_w(1, 0, 1);
  }
  uint32_t g = 0;                             // steps taken (counted alike by every thread)
  int last_load = t_first < t_end ? 1 : -1;   // thread 0: step of the last weight load issued
  int last_mma = -1;                          // thread 0: step of the last MMA group issued
  bool ok = true;
  for (int t = t_first; t < t_end && ok; ++t) {
    const bool discard = t < t_begin;
    const int s = t / tps, j = t - s * tps;
    const int m0 = s * N + j * kSR;
    const int v = min(kSR, N - j * kSR);
    const bool first = j == 0, last = !discard && j == tps - 1;
    if (tid < 4 && (first || last)) {
      const int code = stage_code(a.state, s);
      const HistRef& h = tid < 3 ? a.unit[tid].hist : a.hist_next;
      misc[tid] = (a.state.pool && !(code & 2)) ? head_table(slot_base(a.state, code), code & 1)[h.index] : 0;
      if (tid == 0) misc[4] = code;
    }
    // The previous tile's plane stores have read their staging (A and W);
    // then the first weights of this tile, and the next tile's rows into L2.
    if (tid == 0) {
      bulk_wait_read_all();
      if (t != t_first) {
        load_w(g, 0, 0);
        load_w(g + 1, 0, 1);
        last_load = (int)g + 1;
      }
      if (t + 1 < t_end) {
        const int m1 = tile_m0(t + 1);
        prefetch_l2(a.x + (size_t)m1 * C, (uint32_t)(min(kSR, a.rows - m1) * C * 4));
      }
    }
    // y rows into TMEM columns [0, 256): this thread's row, its 64 columns.
    {
      const int gr = m0 + row;
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        uint32_t r[16];
        const float4* src = reinterpret_cast<const float4*>(a.x + (size_t)gr * C + cg * 64 + h * 16);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float4 f = gr < a.rows ? __ldg(src + e) : make_float4(0.f, 0.f, 0.f, 0.f);
          r[4 * e] = __float_as_uint(f.x);
          r[4 * e + 1] = __float_as_uint(f.y);
          r[4 * e + 2] = __float_as_uint(f.z);
          r[4 * e + 3] = __float_as_uint(f.w);
        }
        tmem_st16(trow + (uint32_t)(cg * 64 + h * 16), r);
      }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const int code = misc[4];
#pragma unroll 1
    for (int u = 0; u < 3 && ok; ++u) {
      const int d = u == 0 ? 1 : u == 1 ? 3 : 9, H = 6 * d;
      const HistRef& hist = a.unit[u].hist;
#pragma unroll 1
      for (int kp = 0; kp < 2; ++kp) {
        // (a) P = f16 Snake_pre(y) of K blocks 2kp, 2kp + 1, rows [0, 128) (a
        // thread per row and 32 columns), and the blocks' halo rows [-H, 0).
        {
          uint32_t r[32];
          const int c = kp * 128 + cg * 32;
          tmem_ld16_async(trow + (uint32_t)c, *reinterpret_cast<uint32_t(*)[16]>(r));
          tmem_ld16_async(trow + (uint32_t)(c + 16), *reinterpret_cast<uint32_t(*)[16]>(r + 16));
          tmem_wait_ld(*reinterpret_cast<uint32_t(*)[16]>(r));
          tmem_wait_ld(*reinterpret_cast<uint32_t(*)[16]>(r + 16));
          const float* pa = rc + 2 * kCoefResidual * 64 + cg * 32;
          const float* pr = pa + 128;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float4 y4 = make_float4(__uint_as_float(r[4 * e]), __uint_as_float(r[4 * e + 1]),
                                          __uint_as_float(r[4 * e + 2]), __uint_as_float(r[4 * e + 3]));
            *reinterpret_cast<uint2*>(pbuf + p_off(kSPOff + row, cg * 8 + e)) =
                f16x4(snake4(y4, lds4(pa + 4 * e), lds4(pr + 4 * e)));
          }
          for (int hr = rg; hr < H; hr += kGroups) {
            const uint2 val = first ? f16x4(stage_hist_quad(a.state, hist, code, misc[u], hr - H, kp * 32 + q))
                                    : *reinterpret_cast<const uint2*>(carry + ((scarry_off(u) + hr) * C + kp * 128 + 4 * q) * 2);
            *reinterpret_cast<uint2*>(pbuf + p_off(kSPOff - H + hr, q)) = val;
          }
          tc_fence_before();
          __syncthreads();
        }
        // (b) depthwise + Snake_post of both blocks into their A tiles; their
        // carried rows or, at a stream's last tile, their new history rows.
        {
          const float* uc = rc;
          uint8_t* ab = aop + 2 * kp * kSR * 128;
          if (u == 0) {
            stage_chains<stage_chain(kGroups, 1)>(uc, pbuf, ab, rg, q, 1);
          } else if (u == 1) {
            stage_chains<stage_chain(kGroups, 3)>(uc, pbuf, ab, rg, q, 3);
          } else {
            stage_chains<stage_chain(kGroups, 9)>(uc, pbuf, ab, rg, q, 9);
          }
          if (!last) {
            for (int hr = rg; hr < H; hr += kGroups)
              *reinterpret_cast<uint2*>(carry + ((scarry_off(u) + hr) * C + kp * 128 + 4 * q) * 2) =
                  *reinterpret_cast<const uint2*>(pbuf + p_off(kSPOff + kSR - H + hr, q));
          } else if (a.state.pool) {
            for (int hr = rg; hr < H; hr += kGroups) {
              const float4 val = f16x4_to_float(*reinterpret_cast<const uint2*>(pbuf + p_off(kSPOff + v - H + hr, q)));
              *reinterpret_cast<float4*>(hist_new_row(a.state, hist, code, misc[u], N - H + hr, N) + kp * 128 + 4 * q) = val;
            }
          }
          fence_async_smem();
          tc_fence_before();
          __syncthreads();
        }
        // (c) the two blocks' MMAs into D (M = 128, N = 256, K = 64 each; one
        // step per block, its weights in buffer step & 1); then the next two
        // steps' weights, each once its buffer's last reader (the MMAs two
        // steps earlier) is done.
        const bool next_in_tile = kp == 0 || u < 2;
        if (tid == 0) {
          ok = a.gate == nullptr || g > 0 || flag_wait(a.gate, a.status, kDevTimeoutGate, wl);
#pragma unroll 1
          for (int b = 0; b < 2 && ok; ++b) {
            const uint32_t gs = g + b;
            const int kb = 2 * kp + b;
            if (!(ok = mbar_wait(&wfull[gs & 1], (gs >> 1) & 1, a.status, kDevTimeoutLoader, wl))) break;
            tc_fence_after();
            const uint32_t a0 = smem_u32(aop + kb * kSR * 128), b0 = smem_u32(wop + (gs & 1) * kWBytes);
            constexpr uint32_t idesc = instr_desc_f16(0u, C);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              mma_f16(tmem + C, smem_desc_sw128(a0 + ks * 32), smem_desc_sw128(b0 + ks * 32), idesc, (kb | ks) ? 1u : 0u);
            mma_commit(&mma_done[gs & 1]);
            last_mma = (int)gs;
          }
          if (ok && next_in_tile) {
            const int nu = kp == 0 ? u : u + 1, nkb = kp == 0 ? 2 : 0;
#pragma unroll 1
            for (int b = 0; b < 2 && ok; ++b) {
              const uint32_t gs = g + 2 + b;  // its buffer's last reader: step gs - 2
              if (!(ok = mbar_wait(&mma_done[gs & 1], ((gs - 2) >> 1) & 1, a.status, kDevTimeoutMma, wl))) break;
              load_w(gs, nu, nkb + b);
              last_load = (int)gs;
            }
          }
        }
        g += 2;
        // Every thread is past this pair's depthwise phase: the next pair's
        // coefficients go into rc and, after the unit's last pair, its
        // epilogue coefficients into P (both published by the barrier below).
        load_round_coefs(kp == 0 ? u : u < 2 ? u + 1 : 0, kp ^ 1);
        if (kp == 1) load_epi_coefs(u);
        if (!__syncthreads_and(ok)) {
          ok = false;
          break;
        }
      }
      if (!ok) break;
      // Every MMA of the unit has finished (the last commit tracks them all).
      ok = __syncthreads_and(mbar_wait(&mma_done[(g - 1) & 1], ((g - 1) >> 1) & 1, a.status, kDevTimeoutMma, wl));
      tc_fence_after();
      if (!ok) break;
      // (d) y = y + (D + b) for this thread's row and 64 columns; unit 2 writes
      // the next conv's planes instead, staged (hi over A, lo over W: both
      // idle now) for the TMA stores.
      {
        const float* pb = ec;
#pragma unroll 1
        for (int h = 0; h < 4; ++h) {
          const int c = cg * 64 + h * 16;
          uint32_t ry[16], rd[16];
          tmem_ld16_async(trow + (uint32_t)c, ry);
          tmem_ld16_async(trow + (uint32_t)(C + c), rd);
          tmem_wait_ld(ry);
          tmem_wait_ld(rd);
          float y[16];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float4 b = lds4(pb + c + 4 * e);
            y[4 * e] = __uint_as_float(ry[4 * e]) + (__uint_as_float(rd[4 * e]) + b.x);
            y[4 * e + 1] = __uint_as_float(ry[4 * e + 1]) + (__uint_as_float(rd[4 * e + 1]) + b.y);
            y[4 * e + 2] = __uint_as_float(ry[4 * e + 2]) + (__uint_as_float(rd[4 * e + 2]) + b.z);
            y[4 * e + 3] = __uint_as_float(ry[4 * e + 3]) + (__uint_as_float(rd[4 * e + 3]) + b.w);
          }
          if (u < 2) {
            uint32_t w[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) w[e] = __float_as_uint(y[e]);
            tmem_st16(trow + (uint32_t)c, w);
            continue;
          }
          uint32_t hi[8], lo[8];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float4 sc = lds4(ec + 256 + c + 4 * e), of = lds4(ec + 512 + c + 4 * e);
            float4 w4 = make_float4(__fadd_rn(__fmul_rn(y[4 * e], sc.x), of.x), __fadd_rn(__fmul_rn(y[4 * e + 1], sc.y), of.y),
                                    __fadd_rn(__fmul_rn(y[4 * e + 2], sc.z), of.z),
                                    __fadd_rn(__fmul_rn(y[4 * e + 3], sc.w), of.w));
            w4 = snake4(w4, lds4(ec + 768 + c + 4 * e), lds4(ec + 1024 + c + 4 * e));
            split_bf16(w4.x, w4.y, hi[2 * e], lo[2 * e]);
            split_bf16(w4.z, w4.w, hi[2 * e + 1], lo[2 * e + 1]);
          }
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int off = (c >> 6) * kSR * 128 + sw128_offset(row, (c & 63) + 8 * e);
            *reinterpret_cast<uint4*>(aop + off) = make_uint4(hi[4 * e], hi[4 * e + 1], hi[4 * e + 2], hi[4 * e + 3]);
            *reinterpret_cast<uint4*>(wop + off) = make_uint4(lo[4 * e], lo[4 * e + 1], lo[4 * e + 2], lo[4 * e + 3]);
          }
          if (!discard && row < v) {
            const int gr = m0 + row, tj = j * kSR + row;
            const size_t plane = (size_t)a.rows * C;
            const bool have = a.state.pool && !(code & 2);
            if (tj == 0) {
              uint4* qh = reinterpret_cast<uint4*>(a.out_planes_prev + (size_t)gr * C + c);
              uint4* ql = reinterpret_cast<uint4*>(a.out_planes_prev + plane + (size_t)gr * C + c);
              const uint4* old = have ? reinterpret_cast<const uint4*>(slot_base(a.state, code) + a.hist_next.ring +
                                                                       misc[3] * a.hist_next.width + c)
                                      : nullptr;
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const uint4 w0 = old ? __ldg(old + 2 * e) : make_uint4(0u, 0u, 0u, 0u);
                const uint4 w1 = old ? __ldg(old + 2 * e + 1) : make_uint4(0u, 0u, 0u, 0u);
                qh[e] = make_uint4(__byte_perm(w0.x, w0.y, 0x7632), __byte_perm(w0.z, w0.w, 0x7632),
                                   __byte_perm(w1.x, w1.y, 0x7632), __byte_perm(w1.z, w1.w, 0x7632));
                ql[e] = make_uint4(__byte_perm(w0.x, w0.y, 0x5410), __byte_perm(w0.z, w0.w, 0x5410),
                                   __byte_perm(w1.x, w1.y, 0x5410), __byte_perm(w1.z, w1.w, 0x5410));
              }
            }
            if (tj == N - 1 && a.state.pool) {
              uint4* dst = reinterpret_cast<uint4*>(slot_base(a.state, code) + a.hist_next.ring +
                                                    (misc[3] ^ 1) * a.hist_next.width + c);
#pragma unroll
              for (int e = 0; e < 4; ++e)
                dst[e] = make_uint4(__byte_perm(lo[2 * e], hi[2 * e], 0x5410), __byte_perm(lo[2 * e], hi[2 * e], 0x7632),
                                    __byte_perm(lo[2 * e + 1], hi[2 * e + 1], 0x5410),
                                    __byte_perm(lo[2 * e + 1], hi[2 * e + 1], 0x7632));
            }
          }
        }
      }
      // The stream's advanced heads, before the barrier that ends the tile:
      // after it, threads 1-3 may already write the next tile's heads into misc.
      if (u == 2 && last && a.state.pool && tid == 0) {
        for (int v2 = 0; v2 < 3; ++v2) hist_commit_head(a.state, a.unit[v2].hist, code, misc[v2], N);
        hist_commit_head(a.state, a.hist_next, code, misc[3], N);
      }
      if (u == 2) fence_async_smem();  // the staged planes are read by TMA stores
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
    }
    if (!ok) break;
    if (!discard && tid == 0) {
#pragma unroll
      for (int kb = 0; kb < 4; ++kb) {
        tma_store_4d(&a.planes_map, aop + kb * kSR * 128, 64 * kb, j * kSR, s, 0);
        tma_store_4d(&a.planes_map, wop + kb * kSR * 128, 64 * kb, j * kSR, s, 1);
        tma_store_4d(&a.prev_map, aop + kb * kSR * 128, 64 * kb, j * kSR + 1, s, 0);
        tma_store_4d(&a.prev_map, wop + kb * kSR * 128, 64 * kb, j * kSR + 1, s, 1);
      }
      bulk_commit();
    }
  }
  // After a timeout: let the last weight load and MMA group issued finish
  // before the CTA frees its TMEM and exits.
  if (!ok && tid == 0) {
    // (The two buffers' latest loads: steps last_load and last_load - 1.)
    for (int l = last_load; l >= 0 && l >= last_load - 1; --l)
      mbar_wait(&wfull[l & 1], (l >> 1) & 1, a.status, kDevTimeoutLoader);
    if (last_mma >= 0) mbar_wait(&mma_done[last_mma & 1], (last_mma >> 1) & 1, a.status, kDevTimeoutMma);
  }
  if (tid == 0) bulk_wait_all();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

int g_stage_sms = 0;

}  // namespace

cudaError_t prepare_stage() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&g_stage_sms, cudaDevAttrMultiProcessorCount, dev);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(stage_kernel<64, 512>, cudaFuncAttributeMaxDynamicSharedMemorySize, StageSmem<64>::kAlloc);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(stage_kernel<64, 256>, cudaFuncAttributeMaxDynamicSharedMemorySize, StageSmem<64>::kAlloc);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(stage_kernel<128, 512>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             StageSmem<128>::kAlloc);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(stage256_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Stage2Smem::kAlloc);
  return e;
}

int stage_sm_count() { return g_stage_sms; }

cudaError_t launch_stage(const StageArgs& a, cudaStream_t stream) {
  if (a.rows <= 0) return cudaSuccess;
  const int N = a.rows_per_stream;
  if (N <= 0 || a.rows % N) return cudaErrorInvalidValue;
  const int tiles = (a.rows / N) * ((N + kSR - 1) / kSR);
  if (a.channels == 64) {
    // At most one tile per SM: one 512-thread CTA per tile. Otherwise two
    // 256-thread CTAs per SM, each over a contiguous range of tiles.
    if (tiles <= g_stage_sms) return launch_overlapped(stage_kernel<64, 512>, tiles, 512, StageSmem<64>::kAlloc, stream, a);
    const int grid = tiles < 2 * g_stage_sms ? tiles : 2 * g_stage_sms;
    return launch_overlapped(stage_kernel<64, 256>, grid, 256, StageSmem<64>::kAlloc, stream, a);
  }
  if (a.channels == 128) {
    const int grid = tiles < g_stage_sms ? tiles : g_stage_sms;
    return launch_overlapped(stage_kernel<128, 512>, grid, 512, StageSmem<128>::kAlloc, stream, a);
  }
  if (a.channels == kS2C) {
    const int grid = tiles < g_stage_sms ? tiles : g_stage_sms;
    return launch_overlapped(stage256_kernel, grid, 512, Stage2Smem::kAlloc, stream, a);
  }
  return cudaErrorInvalidValue;
}

}  // namespace fav
