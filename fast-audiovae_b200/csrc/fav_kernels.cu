// sm_100a kernels of the AudioVAE2 decoder step.
//
// One persistent GEMM engine serves every dense layer: rows = time steps of all
// streams (M tile 128), columns = output channels (N tile 32..256), K = input
// channels. One CTA per SM loops over output tiles; the K-block pipeline runs
// across tile boundaries and two TMEM accumulators let the epilogue of one tile
// overlap the mainloop of the next.
//
// Each epilogue also applies the *next* layer's pointwise prologue, so a
// producer only does the work that needs neighbouring rows:
//   stem, last residual unit of stages 0-4 -> split-bf16 planes of
//     Snake(y * scale + offset), which the next transposed conv TMA-loads
//     straight into its MMA tiles (its producers only patch stream starts);
//   transposed conv, residual units 0-1 -> y and Snake_pre(y) of the next
//     residual unit, whose producers then run depthwise k=7 + Snake only;
//   last residual unit of stage 5 -> Snake_final(y) for the final conv.
//
// Warp roles (512 threads):
//   warps 0-7   A-operand producers (stem depthwise conv; residual depthwise
//               conv + Snake from a TMA-staged box; transposed-conv patches)
//   warps 8-11  epilogue: TMEM -> registers -> bias / skip / next prologue ->
//               global stores, one output row per lane
//   warp 12     loader: weight tiles (bulk copies) and transposed-conv planes
//   warp 13     TMEM owner and MMA issuer (tcgen05.mma, one elected lane)
//   warp 14     scheduler: per-tile stream/row tables, one tile ahead
//   warp 15     residual input loader (TMA boxes + coefficient blocks)
// Each single-thread role has a warp of its own, so no role's spin-wait
// delays another's issue.
// Every wait is bounded and records an error code in the caller's status word
// instead of hanging.
#include "fav_common.cuh"

namespace fav {

constexpr int kProducerWarps = 8;
constexpr int kEpilogueWarps = 4;
constexpr int kThreads = (kProducerWarps + kEpilogueWarps + 4) * 32;
constexpr int kProducerThreads = kProducerWarps * 32;
constexpr int kLoaderWarp = kProducerWarps + kEpilogueWarps;
constexpr int kMmaWarp = kLoaderWarp + 1;
constexpr int kSchedWarp = kMmaWarp + 1;
constexpr int kRawWarp = kSchedWarp + 1;
constexpr int kSmemBudget = 227 * 1024;
constexpr int kMaxHalo = 54;                 // 6 * largest dilation
constexpr int kMaxTileStreams = kTileM + 1;  // streams one 128-row tile can touch
constexpr int kTableInts = 2 * kMaxTileStreams + 2 * kTileM;  // one tile's stream and row tables
constexpr int kEpiCols = 16;                 // epilogue chunk: 16 columns x 32 rows per warp

// Residual producer input of one K block: the TMA box (tile + halo rows of 128
// bytes: 64 channels of f16 s, or stage 5's 32 channels of fp32 s) followed by
// the block's coefficients.
constexpr int kResBoxBytes = (kTileM + kMaxHalo) * 128;
constexpr int kResCoefBytes = kCoefResidual * 64 * 4;

// Split-bf16 operand modes store hi and lo tiles.
template <int MODE>
constexpr bool kSplitOperands = MODE == kModeSplit || MODE == kModeSplit4;

template <int NT, int MODE, int KIND>
struct GemmCfg {
  static constexpr bool kI8 = MODE == kModeI8;
  static constexpr bool kI8Tconv = kI8 && (KIND == kTconv || KIND == kTconvPre);
  // Operand tiles per stage: split-bf16 hi and lo, or the int8 transposed
  // conv's two taps (separately scaled, separate accumulators).
  static constexpr int kTerms = (kSplitOperands<MODE> || kI8Tconv) ? 2 : 1;
  static constexpr int kATile = kTileM * 128;
  static constexpr int kBTile = NT * 128;
  static constexpr int kAStage = kTerms * kATile;
  static constexpr int kBStage = kTerms * kBTile;
  static constexpr int kStage = kAStage + kBStage;
  static constexpr int kRaw =
      KIND == kResidual ? kResBoxBytes + kResCoefBytes : (kI8 && KIND == kTconv) ? (kTileM + 1) * 64 * 4 : 0;
  // Per-tile tables: streams and rows, plus the int8 transposed conv's row scales.
  static constexpr int kTableI = kTableInts + (kI8Tconv ? 2 * kTileM : 0);
  static constexpr int kTable = KIND == kTestGemm ? 0 : 2 * ((kTableI * 4 + 15) / 16) * 16;  // two tiles
  // int8 transposed conv: row scales for the epilogue [2 buffers][current, previous tap][128].
  static constexpr int kScales = kI8 ? 2 * 2 * kTileM * 4 : 0;
  static constexpr int kFixed = 1024 /*align slack*/ + 512 /*barriers*/ + kTable + kScales;
  // Epilogue column coefficients, double-buffered per tile.
  static constexpr int kEpi = 2 * 7 * NT * 4;
  // A layer whose A operand is TMA-loaded by a pre-pass (preformed residual
  // operand, int8 conv taps) has no producer work: its eight producer warps
  // join the epilogue, three warps per TMEM lane quarter, each taking every
  // third 16-column chunk of the tile.
  static constexpr bool kWide = (KIND == kResidualPre || KIND == kTconvPre) && NT >= 64;
  static constexpr int kEpiWarps = kWide ? kEpilogueWarps + kProducerWarps : kEpilogueWarps;
  // Per epilogue warp: one 32-row x 16-column fp32 chunk staged for coalesced stores.
  static constexpr int kEpiStage = kEpiWarps * 32 * kEpiCols * 4;
  static constexpr int kStagesFit = (kSmemBudget - 2 * kRaw - kFixed - kEpi - kEpiStage) / kStage;
  static constexpr int kStages = kStagesFit > 4 ? 4 : kStagesFit;
  static_assert(kStages >= 2, "pipeline needs two stages");
  static constexpr int kSmem = kFixed + kStages * kStage + kEpi + 2 * kRaw + kEpiStage;
  // Two accumulator buffers; one buffer holds NT fp32/s32 columns per accumulator.
  static constexpr int kAccCols = kI8Tconv ? 2 * NT : NT;
  static constexpr uint32_t kTmemCols = 2 * kAccCols < 32 ? 32 : 2 * kAccCols;
  static_assert(kTmemCols <= 512, "TMEM holds 512 columns");
  static constexpr uint32_t kIdesc = kI8 ? instr_desc_i8(NT) : instr_desc_f16(kSplitOperands<MODE> ? 1u : 0u, NT);
};

// ----------------------------------------------------------- history rings
// Per-tile tables, filled one tile ahead by the scheduler warp: for each stream
// the tile touches, its slot code and window head; for each tile row, its
// stream (table entry, -1 past the last row) and time within the chunk.
struct StreamTable {
  int* code;
  int* head;
  int* row_e;
  int* row_t;
  int s_lo;
};

__device__ __forceinline__ StreamTable table_at(int* base, int m0, int rows_per_stream) {
  return StreamTable{base, base + kMaxTileStreams, base + 2 * kMaxTileStreams, base + 2 * kMaxTileStreams + kTileM,
                     m0 / rows_per_stream};
}

__device__ void fill_table(const LayerArgs& a, int m0, const StreamTable& tab, int lane) {
  const int N = a.rows_per_stream;
  const int s_hi = (min(m0 + kTileM, a.rows) - 1) / N;
  for (int i = lane; i <= s_hi - tab.s_lo; i += 32) {
    const int s = tab.s_lo + i;
    const int code = a.state.slot_codes ? a.state.slot_codes[s] : ((s << 2) | a.state.uniform_code);
    int head = 0;
    if (a.state.pool && !(code & 2)) head = head_table(slot_base(a.state, code), code & 1)[a.hist.index];
    tab.code[i] = code;
    tab.head[i] = head;
  }
  for (int r = lane; r < kTileM; r += 32) {
    const int g = m0 + r;
    int e = -1, t = 0;
    if (g < a.rows) {
      const int s = g / N;
      e = s - tab.s_lo;
      t = g - s * N;
    }
    tab.row_e[r] = e;
    tab.row_t[r] = t;
  }
}

// Each stage's last residual unit (a plane writer): the shifted planes' first
// row of every stream starting in tile m0, columns n0 .. n0+nt-1, is the
// stream's previous activated row, kept packed as (hi << 16) | lo in the next
// layer's one-row history (zero for a fresh stream or without a state pool).
// The epilogue writes every other row of both planes. (The stem, whose tiles
// start a stream at nearly every row, copies these rows in its epilogue.)
__device__ void first_rows_prev_planes(const LayerArgs& a, int m0, int n0, int nt, const StreamTable& tab, int lane) {
  const int N = a.rows_per_stream;
  const int g_end = min(m0 + kTileM, a.rows);
  const int s_first = (m0 + N - 1) / N;
  const int nf = (g_end - 1) / N - s_first + 1;
  const int quads = nt / 4;
  const size_t plane = (size_t)a.rows * a.c_out;
  for (int it = lane; it < nf * quads; it += 32) {
    const int e = it / quads, c4 = n0 + 4 * (it - e * quads);
    const int s = s_first + e;
    const int code = tab.code[s - tab.s_lo];
    uint4 w = make_uint4(0u, 0u, 0u, 0u);
    if (a.state.pool && !(code & 2)) {
      float* slot = slot_base(a.state, code);
      const int head = head_table(slot, code & 1)[a.hist_next.index];
      w = __ldg(reinterpret_cast<const uint4*>(slot + a.hist_next.ring + head * a.hist_next.width + c4));
    }
    uint16_t* dst = a.out_planes_prev + (size_t)s * N * a.c_out + c4;
    *reinterpret_cast<uint2*>(dst) = make_uint2(__byte_perm(w.x, w.y, 0x7632), __byte_perm(w.z, w.w, 0x7632));
    *reinterpret_cast<uint2*>(dst + plane) = make_uint2(__byte_perm(w.x, w.y, 0x5410), __byte_perm(w.z, w.w, 0x5410));
  }
}

// Window row holding time tp (-H <= tp < 0, relative to the chunk start) of
// table entry i; nullptr when the history is zero.
__device__ __forceinline__ const float* hist_row(const LayerArgs& a, const StreamTable& tab, int i, int tp) {
  const int code = tab.code[i];
  if (!a.state.pool || (code & 2)) return nullptr;
  const int H = a.hist.rows;
  int row = tab.head[i] + H + tp;  // in [head, head + H)
  if (row >= 2 * H) row -= 2 * H;
  return slot_base(a.state, code) + a.hist.ring + row * a.hist.width;
}

// A-operand stores use plain shared-memory stores (no compiler barrier), so
// loads for later rows can be scheduled ahead of them; fence.proxy.async before
// the stage's barrier arrival publishes them to the tensor core.
// Writes two adjacent channels (k, k+1) of tile row r in the A operand.
template <int MODE>
__device__ __forceinline__ void put_a(uint8_t* a_stage, int r, int k, float v0, float v1) {
  const uint32_t off = sw128_offset(r, k);
  if (kSplitOperands<MODE>) {
    uint32_t hi, lo;
    split_bf16(v0, v1, hi, lo);
    *reinterpret_cast<uint32_t*>(a_stage + off) = hi;
    *reinterpret_cast<uint32_t*>(a_stage + kTileM * 128 + off) = lo;
  } else {
    *reinterpret_cast<uint32_t*>(a_stage + off) = pack_f16(v0, v1);
  }
}

// Writes four adjacent channels (k..k+3, k % 4 == 0) of tile row r.
template <int MODE>
__device__ __forceinline__ void put_a4(uint8_t* a_stage, int r, int k, float4 v) {
  const uint32_t off = sw128_offset(r, k);
  if (kSplitOperands<MODE>) {
    uint32_t h0, l0, h1, l1;
    split_bf16(v.x, v.y, h0, l0);
    split_bf16(v.z, v.w, h1, l1);
    *reinterpret_cast<uint2*>(a_stage + off) = make_uint2(h0, h1);
    *reinterpret_cast<uint2*>(a_stage + kTileM * 128 + off) = make_uint2(l0, l1);
  } else {
    *reinterpret_cast<uint2*>(a_stage + off) = make_uint2(pack_f16(v.x, v.y), pack_f16(v.z, v.w));
  }
}

// Positions n*group .. n*group+n-1 (n <= 8) of warp ``warp``'s 16-row share of
// the tile in residue-class order (rows 0, d, 2d, ..., then 1, 1+d, ...),
// packed as bytes.
__device__ __forceinline__ void class_rows(int d, int warp, int group, int n, uint32_t& lo, uint32_t& hi) {
  int rho = 0, k = 16 * warp + n * group;
  while (k >= (kTileM - rho + d - 1) / d) {
    k -= (kTileM - rho + d - 1) / d;
    ++rho;
  }
  lo = hi = 0;
  for (int u = 0; u < n; ++u) {
    const uint32_t r = rho + k * d;
    if (u < 4) lo |= r << (8 * u);
    else hi |= r << (8 * (u - 4));
    if (++k >= (kTileM - rho + d - 1) / d) {
      ++rho;
      k = 0;
    }
  }
}

__device__ __forceinline__ int walk_row(uint32_t lo, uint32_t hi, int u) {
  return ((u < 4 ? lo : hi) >> (8 * (u & 3))) & 255;
}

// A loader's last fills of a ring of n full barriers: waits (with the full
// kWaitLimit, whatever the launch's own limit) until the copies of the last
// min(issued, n) fills have landed, so that no CTA exits, after a timeout
// elsewhere, with an asynchronous copy still writing its shared memory. A fill
// whose copies have landed (every fill on the success path) returns at once.
__device__ __forceinline__ void drain_fills(uint64_t* full, uint32_t issued, uint32_t n, uint32_t* status,
                                            uint32_t code) {
  for (uint32_t i = issued > n ? issued - n : 0; i < issued; ++i) mbar_wait(&full[i % n], (i / n) & 1, status, code);
}

// ------------------------------------------------------------------ producers
// Stem: depthwise causal conv k=7 (d=1) on latents [S][64][z_stride]; history =
// last six raw latent frames [6][64]. Two channels per lane, one row per warp step.
template <int MODE>
__device__ void produce_stem(const LayerArgs& a, uint8_t* a_stage, int warp, int lane, bool write_state,
                             const StreamTable& tab) {
  const int c = 2 * lane;
  const int T = a.rows_per_stream;
  float w0[7], w1[7];
#pragma unroll
  for (int j = 0; j < 7; ++j) {
    w0[j] = __ldg(a.dw_w + c * 7 + j);
    w1[j] = __ldg(a.dw_w + (c + 1) * 7 + j);
  }
  const float b0 = __ldg(a.dw_b + c), b1 = __ldg(a.dw_b + c + 1);
#pragma unroll 1
  for (int i0 = 0; i0 < 16; i0 += 4) {
    float v0[4][7], v1[4][7];
#pragma unroll
    for (int ii = 0; ii < 4; ++ii) {
      const int r = warp + 8 * (i0 + ii);
      const int e = tab.row_e[r], t = tab.row_t[r];
#pragma unroll
      for (int j = 0; j < 7; ++j) v0[ii][j] = v1[ii][j] = 0.f;
      if (e >= 0) {
        const float* z0 = a.x + ((size_t)(tab.s_lo + e) * kLatentChannels + c) * a.z_stride + a.z_offset;
#pragma unroll
        for (int j = 0; j < 7; ++j) {
          const int tp = t - 6 + j;
          if (tp >= 0) {
            v0[ii][j] = __ldg(z0 + tp);
            v1[ii][j] = __ldg(z0 + a.z_stride + tp);
          } else {
            const float* h = hist_row(a, tab, e, tp);
            if (h) {
              const float2 hv = ldg2(h + c);
              v0[ii][j] = hv.x;
              v1[ii][j] = hv.y;
            }
          }
        }
      }
    }
#pragma unroll
    for (int ii = 0; ii < 4; ++ii) {
      const int r = warp + 8 * (i0 + ii);
      const int e = tab.row_e[r], t = tab.row_t[r];
      float y0 = 0.f, y1 = 0.f;
      if (e >= 0) {
        float acc0 = w0[0] * v0[ii][0], acc1 = w1[0] * v1[ii][0];
#pragma unroll
        for (int j = 1; j < 7; ++j) {
          acc0 = fmaf(w0[j], v0[ii][j], acc0);
          acc1 = fmaf(w1[j], v1[ii][j], acc1);
        }
        y0 = acc0 + b0;
        y1 = acc1 + b1;
        if (write_state && t == T - 1 && a.state.pool) {
          // New window rows: the last min(T, 6) latent frames; zero the rest of a fresh window.
          const int code = tab.code[e], head = tab.head[e];
          const float* z0 = a.x + ((size_t)(tab.s_lo + e) * kLatentChannels + c) * a.z_stride + a.z_offset;
          for (int tp = T > 6 ? T - 6 : 0; tp < T; ++tp) {
            float* dst = hist_new_row(a.state, a.hist, code, head, tp, T);
            *reinterpret_cast<float2*>(dst + c) = make_float2(__ldg(z0 + tp), __ldg(z0 + a.z_stride + tp));
          }
          if ((code & 2) && T < 6) {
            float* ring = slot_base(a.state, code) + a.hist.ring;
            for (int j = T; j < 6; ++j)
              *reinterpret_cast<float2*>(ring + j * kLatentChannels + c) = make_float2(0.f, 0.f);
          }
          if (lane == 0) hist_commit_head(a.state, a.hist, code, head, T);
        }
      }
      put_a<MODE>(a_stage, r, c, y0, y1);
    }
  }
}

// Residual unit, K block kb: depthwise causal k=7 (dilation d) -> Snake on
// s = Snake_pre(x), which the previous layer's epilogue wrote. ``raw`` holds s
// rows m0-H .. m0+127 of the K block (pitch P) followed by the block's
// coefficients [w0..w6, bias, alpha2, recip2][64]. Each lane group walks its
// rows in residue-class order (packed in walk_lo/hi) so the seven taps slide
// through registers; a regular chain (one stream, every tap inside the chunk)
// runs branch-free. History = last 6d rows of s [6d][C]. LPR lanes cover one
// row (16 for 64-channel K blocks, 8 for C = 32).
template <int MODE, int LPR>
__device__ void produce_residual(const LayerArgs& a, int m0, int kb, uint8_t* a_stage, const float* raw, int warp,
                                 int lane, bool hist_writer, const StreamTable& tab, uint32_t walk_lo,
                                 uint32_t walk_hi, bool regular) {
  constexpr int kRpg = 16 * LPR / 32;  // rows walked per lane group
  const int C = a.k_channels;
  const int d = a.dilation;
  const int H = 6 * d;
  const int N = a.rows_per_stream;
  const int P = a.raw_pitch;
  const int cq = lane % LPR;
  const int kl = 4 * cq;
  const int c = kb * kKBlock + kl;
  const bool valid = kl < P;
  const int tid = warp * 32 + lane;
  const float* cf = raw + kResBoxBytes / 4 + kl;
  // New window rows of the streams whose last row lies in this tile (table
  // entries 0 .. ns-1): one flat loop over (stream, row, quad) so every
  // producer thread stores independent items.
  if (hist_writer && a.state.pool) {
    const int g_end = min(m0 + kTileM, a.rows);
    const int ns = g_end / N - tab.s_lo;
    const int n_new = N < H ? N : H;
    const int quads = P / 4;
    const int per = n_new * quads;
#pragma unroll 2
    for (int it = tid; it < ns * per; it += kProducerThreads) {
      const int e = it / per, rem = it - e * per;
      const int q = rem / quads, k4 = 4 * (rem - q * quads);
      const int tp = N - n_new + q;
      *reinterpret_cast<float4*>(hist_new_row(a.state, a.hist, tab.code[e], tab.head[e], tp, N) + kb * kKBlock + k4) =
          lds4(raw + ((tab.s_lo + e) * N + tp - m0 + H) * P + k4);
    }
    if (N < H) {
      // A fresh stream's window starts as H - N zero rows before its N new ones.
      const int zper = (H - N) * quads;
      for (int it = tid; it < ns * zper; it += kProducerThreads) {
        const int e = it / zper, rem = it - e * zper;
        const int code = tab.code[e];
        if (!(code & 2)) continue;
        const int q = rem / quads, k4 = 4 * (rem - q * quads);
        *reinterpret_cast<float4*>(slot_base(a.state, code) + a.hist.ring + (N + q) * C + kb * kKBlock + k4) =
            make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    if (kb == 0)
      for (int e = tid; e < ns; e += kProducerThreads) hist_commit_head(a.state, a.hist, tab.code[e], tab.head[e], N);
  }
  const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 w[7];
#pragma unroll
  for (int j = 0; j < 7; ++j) w[j] = valid ? lds4(cf + j * 64) : zero4;
  const float4 bias = valid ? lds4(cf + 7 * 64) : zero4;
  const float4 al2 = valid ? lds4(cf + 8 * 64) : zero4;
  const float4 rc2 = valid ? lds4(cf + 9 * 64) : zero4;
  float4 win[7];
  if (regular) {
    // The lane group's rows are r0, r0+d, ..., r0+(kRpg-1)d of one stream with
    // every tap inside the chunk: a branch-free sliding window.
    const int r0 = walk_lo & 255;
    const float* base = raw + (r0 - 6 * d + H) * P + kl;
    const int step = d * P;
#pragma unroll
    for (int j = 0; j < 6; ++j) win[j] = valid ? lds4(base + j * step) : zero4;
#pragma unroll
    for (int u = 0; u < kRpg; ++u) {
      win[6] = valid ? lds4(base + (6 + u) * step) : zero4;
      const float4 h = dw7<false>(w, win, bias);
      put_a4<MODE>(a_stage, r0 + u * d, kl, valid ? snake4(h, al2, rc2) : zero4);
#pragma unroll
      for (int j = 0; j < 6; ++j) win[j] = win[j + 1];
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < 7; ++j) win[j] = zero4;
  int prev_r = -1000000, prev_e = -2;
#pragma unroll 1
  for (int u = 0; u < kRpg; ++u) {
    const int r = walk_row(walk_lo, walk_hi, u);
    const int e = tab.row_e[r];
    float4 y = zero4;
    if (valid && e >= 0) {
      if (prev_r == r - d && prev_e == e) {
#pragma unroll
        for (int j = 0; j < 6; ++j) win[j] = win[j + 1];
      } else {
        const int t = tab.row_t[r];
#pragma unroll
        for (int j = 0; j < 6; ++j) {
          const int back = (6 - j) * d;
          const int tp = t - back;
          if (tp >= 0) {
            win[j] = lds4(raw + (r - back + H) * P + kl);
          } else {
            const float* hr = hist_row(a, tab, e, tp);
            win[j] = hr ? ldg4(hr + c) : zero4;
          }
        }
      }
      win[6] = lds4(raw + (r + H) * P + kl);
      const float4 h = dw7<false>(w, win, bias);
      y = snake4(h, al2, rc2);
      prev_r = r;
      prev_e = e;
    } else {
      prev_e = -2;
    }
    put_a4<MODE>(a_stage, r, kl, y);
  }
}

// The one stream start that bears on a residual tile's depthwise taps, for
// units that stage f16 Snake_pre(y) (s16) on streams of at least 128 + 6d rows: the
// start b of the stream holding the tile's last row, when it lies after
// m0 - 6d (its first 6d rows, which reach into the stream's history, overlap
// the tile); at most one stream starts in (m0 - 6d, m0 + 128).
struct TileStart {
  int b;      // global row of the start; meaningless when !on
  int entry;  // its stream's table entry
  bool on;
};
__device__ __forceinline__ TileStart tile_start(const LayerArgs& a, int m0, const StreamTable& tab) {
  const int N = a.rows_per_stream;
  const int s = (min(m0 + kTileM, a.rows) - 1) / N;
  const int b = s * N;
  return TileStart{b, s - tab.s_lo, b > m0 - 6 * a.dilation};
}

// The history window rows a producer thread loads for produce_residual_s16:
// items tid + k * 256 (k < 4) of [H rows][16 quads] of K block kb, zero for a
// fresh stream, without a pool, or past the rows the tile can reach. With
// ``prefetch`` the thread only asks for their lines in L1 (no registers held
// across the walk); the loads after the walk then hit L1.
template <bool PREFETCH>
__device__ __forceinline__ void load_tile_history(const LayerArgs& a, int m0, int kb, const StreamTable& tab,
                                                  const TileStart& ts, int tid, float4 (&hist_reg)[4]) {
  const int H = 6 * a.dilation;
  const int code = tab.code[ts.entry];
  const bool have = a.state.pool && !(code & 2);
  const float* ring = have ? slot_base(a.state, code) + a.hist.ring + kb * kKBlock : nullptr;
  const int head = tab.head[ts.entry];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int it = tid + k * kProducerThreads;
    const int j = it >> 4;
    hist_reg[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (have && j < H && ts.b - m0 + j >= 0) {
      int row = head + j;  // window row j (time j - H), ring of 2H rows
      if (row >= 2 * H) row -= 2 * H;
      const float* src = ring + row * a.hist.width + 4 * (it & 15);
      if constexpr (PREFETCH) {
        asm volatile("prefetch.global.L1 [%0];" ::"l"(src));
      } else {
        hist_reg[k] = ldg4(src);
      }
    }
  }
}

// Channel quad k .. k+3 of f16 box row r (64 channels, 128 bytes per row).
__device__ __forceinline__ float4 box_quad(const float* raw, int r, int k) {
  const uint2 h = *reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(raw) + r * kKBlock + k);
  const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
  const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&h.y));
  return make_float4(lo.x, lo.y, hi.x, hi.y);
}
// Stores a quad into f16 box row r (exact for history rows, which hold f16 values).
__device__ __forceinline__ void put_box_quad(float* raw, int r, int k, float4 v) {
  *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(raw) + r * kKBlock + k) =
      make_uint2(pack_f16(v.x, v.y), pack_f16(v.z, v.w));
}

// Residual unit staging s = Snake_pre(y) in f16 (s16, written by the previous
// epilogue), K block kb, 64-channel blocks: depthwise k=7 (dilation d) +
// Snake_post of the box. Every lane group walks its eight rows in
// residue-class order with a sliding window of taps from the box: rows
// r, r + d, ... of one class, and where its positions cross into the next
// class (at most once: classes hold at least 14 rows) the window is reloaded
// once. The walk ignores streams; rows whose taps reach before their stream's
// start (its first 6d rows) get wrong taps there and are recomputed after the
// walk: the producers overwrite the box rows before that start (the previous
// stream's last rows, no longer read) with the stream's history window (whose
// lines they prefetched into L1 before the walk), and recompute those rows one
// (row, channel quad) per thread. ``hist_writer``: this N tile writes
// the new window rows of streams ending in the tile (first, from the box).
// Producer-collective (named barrier 2).
__device__ void produce_residual_s16(const LayerArgs& a, int m0, int kb, uint8_t* a_stage, float* raw, int warp,
                                   int lane, bool hist_writer, const StreamTable& tab, uint32_t walk_lo,
                                   uint32_t walk_hi, int ubreak, const TileStart& ts) {
  const int d = a.dilation;
  const int H = 6 * d;
  const int N = a.rows_per_stream;
  constexpr int P = kKBlock;
  const int q = lane & 15;
  const int kl = 4 * q;
  const int tid = warp * 32 + lane;
  const float* cf = raw + kResBoxBytes / 4 + kl;
  if (hist_writer && a.state.pool) {
    // New window rows (the last min(N, H) rows of s) of the streams whose last row lies in this tile.
    const int g_end = min(m0 + kTileM, a.rows);
    const int ns = g_end / N - tab.s_lo;
    const int per = H * (P / 4);
#pragma unroll 2
    for (int it = tid; it < ns * per; it += kProducerThreads) {
      const int e = it / per, rem = it - e * per;
      const int row = rem / (P / 4), k4 = 4 * (rem - row * (P / 4));
      const int tp = N - H + row;
      *reinterpret_cast<float4*>(hist_new_row(a.state, a.hist, tab.code[e], tab.head[e], tp, N) + kb * kKBlock + k4) =
          box_quad(raw, (tab.s_lo + e) * N + tp - m0 + H, k4);
    }
    if (kb == 0)
      for (int e = tid; e < ns; e += kProducerThreads) hist_commit_head(a.state, a.hist, tab.code[e], tab.head[e], N);
  }
  float4 w[7];
#pragma unroll
  for (int j = 0; j < 7; ++j) w[j] = lds4(cf + j * 64);
  const float4 bias = lds4(cf + 7 * 64), al2 = lds4(cf + 8 * 64), rc2 = lds4(cf + 9 * 64);
  {
    const int r0 = walk_row(walk_lo, walk_hi, 0);
    const int r1 = ubreak < 8 ? walk_row(walk_lo, walk_hi, ubreak) : 0;
    float4 win[7];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int r = u < ubreak ? r0 + u * d : r1 + (u - ubreak) * d;
      if (u == 0 || u == ubreak) {
#pragma unroll
        for (int j = 0; j < 6; ++j) win[j] = box_quad(raw, r - (6 - j) * d + H, kl);
      }
      win[6] = box_quad(raw, r + H, kl);
      put_a4<kModeF16>(a_stage, r, kl, snake4(dw7<false>(w, win, bias), al2, rc2));
#pragma unroll
      for (int j = 0; j < 6; ++j) win[j] = win[j + 1];
    }
  }
  if (!ts.on) return;
  // Rows [b, b + H) of the stream starting at b: its history window replaces
  // box rows [b - H, b) (box position of global row g: g - m0 + H), then those
  // rows are recomputed. Every walk has finished reading the box first.
  float4 hist_reg[4];
  load_tile_history<false>(a, m0, kb, tab, ts, tid, hist_reg);
  named_barrier(2, kProducerThreads);
  const int pos0 = ts.b - m0;  // box position of history row 0
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int it = tid + k * kProducerThreads;
    const int j = it >> 4;  // history row; quad = it & 15 = q
    if (j < H && pos0 + j >= 0) put_box_quad(raw, pos0 + j, 4 * (it & 15), hist_reg[k]);
  }
  named_barrier(2, kProducerThreads);
  const int lo = max(ts.b, m0) - m0, hi = min(min(ts.b + H, m0 + kTileM), a.rows) - m0;
  for (int it = tid; it < (hi - lo) * 16; it += kProducerThreads) {
    const int r = lo + (it >> 4), k4 = 4 * (it & 15);
    float4 wq[7], win[7];
#pragma unroll
    for (int j = 0; j < 7; ++j) {
      wq[j] = lds4(raw + kResBoxBytes / 4 + k4 + j * 64);
      win[j] = box_quad(raw, r - (6 - j) * d + H, k4);
    }
    const float4 bq = lds4(raw + kResBoxBytes / 4 + k4 + 7 * 64);
    const float4 aq = lds4(raw + kResBoxBytes / 4 + k4 + 8 * 64), rq = lds4(raw + kResBoxBytes / 4 + k4 + 9 * 64);
    put_a4<kModeF16>(a_stage, r, k4, snake4(dw7<false>(wq, win, bq), aq, rq));
  }
}

// Transposed conv, int8, half h (64 channels) of K block kb8: ``raw`` holds the
// activated input rows m0-1 .. m0+127 (fp32, 64 channels). Each box row is
// quantised once with its own scale and written to both taps: row r of the
// current-tap tile holds input row m0+r, row r of the previous-tap tile input
// row m0+r-1, or, at a stream's first step, the history (previous activated
// input) quantised with its own scale. scale[r] is the scale of input row
// m0+r; scale_prev[r] the previous-tap scale of tile row r.
__device__ void produce_tconv_i8(const LayerArgs& a, int kb8, int h, uint8_t* a_stage, const float* raw,
                                 const float* scale, const float* scale_prev, int warp, int lane,
                                 const StreamTable& tab) {
  constexpr int kATile = kTileM * 128;
  const int cq = lane & 15, rs = lane >> 4;
  const int kl = 4 * cq;
  const int byte = h * 64 + kl;  // byte within the 128-byte operand row
  const int c = kb8 * kKBlockI8 + byte;
#pragma unroll 1
  for (int j = 0; j < 9; ++j) {
    const int i = 2 * (warp + 8 * j) + rs;  // box row: input row m0 - 1 + i
    if (i > kTileM) break;
    const float4 v = lds4(raw + i * 64 + kl);
    if (i >= 1)
      *reinterpret_cast<uint32_t*>(a_stage + sw128_offset(i - 1, byte >> 1)) = quant4(v, scale[i - 1]);
    if (i < kTileM) {
      const int e = tab.row_e[i];
      float4 pv = v;
      if (e >= 0 && tab.row_t[i] == 0) {
        const float* hr = hist_row(a, tab, e, -1);
        pv = hr ? ldg4(hr + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      *reinterpret_cast<uint32_t*>(a_stage + kATile + sw128_offset(i, byte >> 1)) = quant4(pv, scale_prev[i]);
    }
  }
}

// Plain GEMM operand for the engine self-test: A [rows][K] fp32 row-major
// (int8 mode: integer values in [-127, 127], taken as they are).
template <int MODE>
__device__ void produce_test(const LayerArgs& a, int m0, int kb, uint8_t* a_stage, int warp, int lane) {
  if constexpr (MODE == kModeI8) {
#pragma unroll 1
    for (int j = 0; j < 16; ++j) {
      const int r = warp + 8 * j, g = m0 + r, c = kb * kKBlockI8 + 4 * lane;
      uint32_t word = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float v = (g < a.rows && c + e < a.k_channels) ? __ldg(a.x + (size_t)g * a.k_channels + c + e) : 0.f;
        word |= (static_cast<uint32_t>(__float2int_rn(v)) & 0xffu) << (8 * e);
      }
      *reinterpret_cast<uint32_t*>(a_stage + sw128_offset(r, 2 * lane)) = word;
    }
    return;
  }
  const int c = kb * kKBlock + 2 * lane;
  float2 v[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int g = m0 + warp + 8 * i;
    v[i] = (g < a.rows && c < a.k_channels) ? ldg2(a.x + (size_t)g * a.k_channels + c) : make_float2(0.f, 0.f);
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) put_a<MODE>(a_stage, warp + 8 * i, 2 * lane, v[i].x, v[i].y);
}

// ------------------------------------------------------------------ epilogue
// Epilogue chunks move between registers (one row per lane) and global memory
// (eight rows of 64 bytes per instruction) through the warp's 32-row x
// 64-byte staging buffer. The 16-byte granule j of row r sits at granule
// j ^ ((r >> 1) & 3), so both the row-wise and the column-wise accesses touch
// each bank group four times (four wavefronts per 512-byte access).
__device__ __forceinline__ int stage_granule(int r, int j) { return r * 4 + (j ^ ((r >> 1) & 3)); }

// Skip input of a residual unit, rows row0 .. row0+31, columns n .. n+15, in
// the coalesced order: xr[k] = granule (lane & 3) of row 8k + lane/4 (zeros
// past the last row).
template <int KIND>
__device__ __forceinline__ void load_skip(const LayerArgs& a, int row0, int n, int lane, float4 (&xr)[4]) {
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int g = row0 + 8 * k + (lane >> 2);
    xr[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    if ((KIND == kResidual || KIND == kResidualPre) && g < a.rows) xr[k] = __ldg(reinterpret_cast<const float4*>(a.x + (size_t)g * a.c_out + n) + (lane & 3));
  }
}

// The coalesced skip chunk xr, transposed to this lane's row. Warp-collective.
__device__ __forceinline__ void transpose_skip(float* stage, int lane, const float4 (&xr)[4], float4 (&x)[4]) {
  float4* sg = reinterpret_cast<float4*>(stage);
  __syncwarp();  // the previous chunk's reads of the buffer are done
#pragma unroll
  for (int k = 0; k < 4; ++k) sg[stage_granule(8 * k + (lane >> 2), lane & 3)] = xr[k];
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 4; ++j) x[j] = sg[stage_granule(lane, j)];
}

// Coalesced store of a warp's 32-row x 16-column fp32 chunk (this lane's row
// in v): row r to dst0 + r * pitch, rows r >= valid skipped. Warp-collective.
__device__ __forceinline__ void store_chunk(float* stage, int lane, const float (&v)[16], float* dst0, size_t pitch,
                                            int valid) {
  float4* sg = reinterpret_cast<float4*>(stage);
  __syncwarp();  // the previous reads of the buffer are done
#pragma unroll
  for (int j = 0; j < 4; ++j) sg[stage_granule(lane, j)] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  __syncwarp();
  const int gq = lane & 3;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int r = 8 * k + (lane >> 2);
    const float4 u = sg[stage_granule(r, gq)];
    if (r < valid) *reinterpret_cast<float4*>(dst0 + r * pitch + 4 * gq) = u;
  }
}

// Coalesced store of a warp's 32-row x 16-column chunk of split-bf16 planes
// (this lane's row in hi/lo): row r's 32-byte hi and lo segments go to the
// current planes at cur + off0 + r * c_out (lo one plane later) and, unless
// the row is its stream's last step, one row later in the shifted planes.
// tq[k]: time step of row 8k + lane/4 within its stream, -1 past the last row.
// Warp-collective.
__device__ __forceinline__ void store_planes_chunk(float* stage, int lane, const uint32_t (&hi)[8],
                                                   const uint32_t (&lo)[8], uint16_t* cur, uint16_t* prev,
                                                   size_t plane, size_t off0, int c_out, int N, const int (&tq)[4]) {
  uint4* sg = reinterpret_cast<uint4*>(stage);
  __syncwarp();  // the previous reads of the buffer are done
  sg[stage_granule(lane, 0)] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
  sg[stage_granule(lane, 1)] = make_uint4(hi[4], hi[5], hi[6], hi[7]);
  sg[stage_granule(lane, 2)] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  sg[stage_granule(lane, 3)] = make_uint4(lo[4], lo[5], lo[6], lo[7]);
  __syncwarp();
  const int gq = lane & 3;
  const size_t part = (gq >> 1) * plane + (gq & 1) * 8;  // hi or lo plane, first or second 8 columns
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int r = 8 * k + (lane >> 2);
    const uint4 u = sg[stage_granule(r, gq)];
    if (tq[k] >= 0) {
      const size_t o = off0 + (size_t)r * c_out + part;
      *reinterpret_cast<uint4*>(cur + o) = u;
      if (tq[k] + 1 < N) *reinterpret_cast<uint4*>(prev + o + c_out) = u;
    }
  }
}

__device__ __forceinline__ void st4(float* dst, const float (&v)[16]) {
#pragma unroll
  for (int j = 0; j < 4; ++j)
    reinterpret_cast<float4*>(dst)[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
}

// Per-column epilogue coefficients of one tile, staged in shared memory:
// [bias, next_alpha, next_recip, next_scale, next_offset, w_scale, w_scale2][NT].
constexpr int kEpiCoefVectors = 7;

// --------------------------------------------------------------------- engine
// Epilogue output class (besides y, written when the layer's kEpiX flag is set).
enum EpilogueOut : int { kOutNone = 0, kOutS = 1, kOutPlanes = 2, kOutAct = 3, kOutS16 = 4 };

template <int NT, int MODE, int KIND, int OUT>
__global__ void __launch_bounds__(kThreads, 1) gemm_layer_kernel(const __grid_constant__ LayerArgs a) {
  using Cfg = GemmCfg<NT, MODE, KIND>;
  constexpr bool kOutPl = OUT == kOutPlanes;
  constexpr bool kOutA = OUT == kOutAct;
  constexpr int S = Cfg::kStages;
  constexpr bool kI8 = Cfg::kI8;
  constexpr bool kI8Tconv = Cfg::kI8Tconv;
  constexpr bool kStaged = KIND == kResidual || (kI8 && KIND == kTconv);  // producers read TMA-staged boxes
  constexpr bool kConv = KIND == kTconv || KIND == kTconvPre;
  constexpr bool kSkipAdd = KIND == kResidual || KIND == kResidualPre;  // y = x + (D + b)
  // The A operand is TMA-loaded whole (no producer work): a bf16 transposed
  // conv's planes, or a residual unit's preformed depthwise output.
  constexpr bool kTmaA = (KIND == kTconv && !kI8) || KIND == kResidualPre || KIND == kTconvPre;
  constexpr int kLpr = NT == 32 ? 8 : 16;  // residual lanes per row (C = 32 uses eight)
  constexpr bool kWide = Cfg::kWide;
  constexpr int kEW = Cfg::kEpiWarps;               // epilogue warps
  constexpr int kEpiFirst = kWide ? 0 : kProducerWarps;  // the first of them
  constexpr int kCG = kEW / 4;                        // epilogue warps per TMEM lane quarter
  extern __shared__ uint8_t smem_raw[];
  // Aligned by an offset from the shared array (not through an integer), so
  // the compiler keeps every access through it in the shared state space.
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* a_base = smem;
  uint8_t* b_base = a_base + S * Cfg::kAStage;
  float* epi_coef = reinterpret_cast<float*>(b_base + S * Cfg::kBStage);  // [2][kEpiCoefVectors][NT]
  uint8_t* raw_base = reinterpret_cast<uint8_t*>(epi_coef) + Cfg::kEpi;
  float* epi_stage = reinterpret_cast<float*>(raw_base + 2 * Cfg::kRaw);  // [kEpilogueWarps][32][kEpiCols]
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(epi_stage) + Cfg::kEpiStage);
  uint64_t* a_full = bars;
  uint64_t* b_full = bars + S;
  uint64_t* empty = bars + 2 * S;
  uint64_t* acc_full = bars + 3 * S;          // [2]
  uint64_t* acc_empty = bars + 3 * S + 2;     // [2]
  uint64_t* raw_full = bars + 3 * S + 4;      // [2]
  uint64_t* raw_empty = bars + 3 * S + 6;     // [2]
  uint64_t* table_full = bars + 3 * S + 8;    // [2]
  uint64_t* table_empty = bars + 3 * S + 10;  // [2]
  uint64_t* scale_full = bars + 3 * S + 12;   // [2] int8: a tile's row scales are written
  uint64_t* scale_empty = bars + 3 * S + 14;  // [2] int8: the epilogue has read them
  uint64_t* mma_drain = bars + 3 * S + 16;    // every MMA the issuer started has finished
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * S + 17);
  int* table = reinterpret_cast<int*>(bars + 3 * S + 18);
  float* scales = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 512 + Cfg::kTable);  // [2][2][128]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t wl = a.wait_limit ? a.wait_limit : kWaitLimit;  // polls before a wait gives up
  const int num_kb = a.num_kblocks;
  const int num_m = (a.rows + kTileM - 1) / kTileM;
  const int num_n = a.n_total / NT;
  const int num_tiles = num_m * num_n;
  // Tile t -> (M tile, N tile): M fastest by default, so concurrently running
  // CTAs share weight tiles in L2; N fastest when the A operand is the larger
  // one, so they share A instead.
  auto tile_m = [&](int t) { return a.n_major ? t / num_n : t % num_m; };
  auto tile_n = [&](int t) { return a.n_major ? t % num_n : t / num_m; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      // A bf16 transposed conv's A operand is one TMA load (transaction count only).
      mbar_init(&a_full[s], kTmaA ? 1 : kProducerWarps);
      mbar_init(&b_full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEW);
      mbar_init(&raw_full[b], 1);
      mbar_init(&raw_empty[b], kProducerWarps);
      mbar_init(&table_full[b], 1);
      mbar_init(&table_empty[b], kProducerWarps);
      mbar_init(&scale_full[b], 1);
      mbar_init(&scale_empty[b], kEW);
    }
    mbar_init(mma_drain, 1);
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dependency_sync();

  if (!kWide && warp < kProducerWarps) {
    // ---- A producers (a bf16 transposed conv has none: its A operand is TMA-loaded whole)
    if (kTmaA) goto done;
    if (KIND == kResidual && kLpr == 8) {
      // C = 32: channels 32-63 of every A stage stay zero.
      for (int s = 0; s < S; ++s)
        for (int r = threadIdx.x; r < kTileM; r += kProducerThreads)
          for (int k = 32; k < 64; k += 4)
            put_a4<MODE>(a_base + s * Cfg::kAStage, r, k, make_float4(0.f, 0.f, 0.f, 0.f));
    }
    uint32_t g = 0, g2 = 0, ti = 0;  // stage, staged-box and tile counters
    bool ok = true;
    uint32_t walk_lo = 0, walk_hi = 0;
    constexpr int kRpg = 16 * kLpr / 32;
    bool chain = false;  // this lane group's rows form one arithmetic chain of step d
    int ubreak = 8;      // position where this lane group's rows move to the next residue class (8: none)
    // A tile with empty rows (the last M tile, e.g. one stream) walks rows
    // interleaved across the lane groups instead, so the valid rows spread
    // over every warp.
    uint32_t iwalk_lo = 0, iwalk_hi = 0;
    if (KIND == kResidual) {
      constexpr int kGroups = kProducerThreads / kLpr;
      const int grp = (warp * 32 + lane) / kLpr;
      for (int u = 0; u < kRpg; ++u) {
        const uint32_t r = grp + kGroups * u;
        if (u < 4) iwalk_lo |= r << (8 * u);
        else iwalk_hi |= r << (8 * (u - 4));
      }
      class_rows(a.dilation, warp, lane / kLpr, kRpg, walk_lo, walk_hi);
      chain = true;
      for (int u = 1; u < kRpg; ++u) {
        const bool step = walk_row(walk_lo, walk_hi, u) == walk_row(walk_lo, walk_hi, u - 1) + a.dilation;
        chain = chain && walk_row(walk_lo, walk_hi, u) == (int)(walk_lo & 255) + u * a.dilation;
        if (!step && ubreak == 8) ubreak = u;
      }
    }
    const int res_boxes = a.k_channels < kKBlock ? 1 : a.k_channels / kKBlock;  // residual boxes per tile
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++ti) {
      const int m0 = tile_m(t) * kTileM;
      const bool write_state = tile_n(t) == 0;
      int* tbase = table + (ti & 1) * Cfg::kTableI;
      const StreamTable tab = table_at(tbase, m0, a.rows_per_stream);
      bool regular = false;
      if (KIND != kTestGemm) {
        ok = named_barrier_and(2, kProducerThreads,
                               mbar_wait(&table_full[ti & 1], (ti >> 1) & 1, a.status, kDevTimeoutProducer, wl));
        if (!ok) break;
        if (KIND == kResidual && chain) {
          const int r0 = walk_lo & 255, rl = walk_row(walk_lo, walk_hi, kRpg - 1), e0 = tab.row_e[r0];
          regular = e0 >= 0 && e0 == tab.row_e[rl] && tab.row_t[r0] >= 6 * a.dilation;
        }
        if (KIND == kResidual && a.rows - m0 < kTileM) regular = false;
      }
      const bool partial = a.rows - m0 < kTileM;
      if constexpr (kI8Tconv) {
        const float* sc = reinterpret_cast<const float*>(tbase + kTableInts);
        for (int kb = 0; kb < num_kb && ok; ++kb, ++g) {
          const int s = g % S;
          const uint32_t ph = (g / S) & 1;
          ok = named_barrier_and(2, kProducerThreads, mbar_wait(&empty[s], ph ^ 1, a.status, kDevTimeoutProducer, wl));
          if (!ok) break;
          uint8_t* a_stage = a_base + s * Cfg::kAStage;
          for (int h = 0; h < 2 && ok; ++h, ++g2) {
            const int rb = g2 & 1;
            ok = named_barrier_and(2, kProducerThreads,
                                   mbar_wait(&raw_full[rb], (g2 >> 1) & 1, a.status, kDevTimeoutProducer, wl));
            if (!ok) break;
            produce_tconv_i8(a, kb, h, a_stage, reinterpret_cast<const float*>(raw_base + rb * Cfg::kRaw), sc,
                             sc + kTileM, warp, lane, tab);
            __syncwarp();
            if (lane == 0) mbar_arrive(&raw_empty[rb]);
          }
          if (!ok) break;
          fence_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&a_full[s]);
        }
      } else {
        for (int kb = 0; kb < num_kb; ++kb, ++g) {
          const int s = g % S;
          const uint32_t ph = (g / S) & 1;
          const int rb = g & 1;
          // All producer threads leave together on a timeout, so none is left
          // waiting at a named barrier inside a producer.
          bool ready = mbar_wait(&empty[s], ph ^ 1, a.status, kDevTimeoutProducer, wl);
          if (kStaged && ready) ready = mbar_wait(&raw_full[rb], (g >> 1) & 1, a.status, kDevTimeoutProducer, wl);
          ok = named_barrier_and(2, kProducerThreads, ready);
          if (!ok) break;
          uint8_t* a_stage = a_base + s * Cfg::kAStage;
          if (KIND == kStem) {
            produce_stem<MODE>(a, a_stage, warp, lane, write_state, tab);
          } else if (KIND == kResidual) {
            float* raw = reinterpret_cast<float*>(raw_base + rb * Cfg::kRaw);
            if (kLpr == 16 && !kI8 && a.s16) {
              const TileStart ts = tile_start(a, m0, tab);
              if (ts.on) {
                float4 unused[4];
                load_tile_history<true>(a, m0, kb, tab, ts, threadIdx.x, unused);
              }
              produce_residual_s16(a, m0, kb, a_stage, raw, warp, lane, kb % num_n == tile_n(t), tab, walk_lo, walk_hi,
                                   ubreak, ts);
            } else {
              produce_residual<MODE, kLpr>(a, m0, kb, a_stage, raw, warp, lane, kb % num_n == tile_n(t), tab,
                                           partial ? iwalk_lo : walk_lo, partial ? iwalk_hi : walk_hi, regular);
            }
          } else {
            produce_test<MODE>(a, m0, kb, a_stage, warp, lane);
          }
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (kStaged) mbar_arrive(&raw_empty[rb]);
            mbar_arrive(&a_full[s]);
          }
        }
      }
      __syncwarp();
      if (KIND != kTestGemm && lane == 0) mbar_arrive(&table_empty[ti & 1]);
    }
  } else if (warp < kLoaderWarp) {
    // ---- epilogue: per 16-column chunk, TMEM -> registers -> (int8: integer
    // accumulators rescaled by weight-row and activation-row scales) + bias
    // (+ skip) -> next layer's pointwise prologue -> global stores (one row per
    // lane). The next chunk's TMEM load and skip input are in flight while a
    // chunk computes (bf16 paths).
    constexpr int kChunks = NT / kEpiCols;
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int cg = (warp - kEpiFirst) >> 2;  // column group: chunks cg, cg + kCG, ...
    const int etid = threadIdx.x - kEpiFirst * 32;
    float* stage = epi_stage + (warp - kEpiFirst) * 32 * kEpiCols;
    const int epi = a.epi;
    bool ok = true;
    uint32_t i = 0;
    int cbuf = 1, staged_n0 = -1;  // coefficient buffer in use and the N tile it holds
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++i) {
      const int buf = i & 1;
      const int m0 = tile_m(t) * kTileM, n0 = tile_n(t) * NT;
      // Stage the column coefficients when the N tile changes, into the other
      // buffer (every warp has passed the previous tile's barrier, so no warp
      // still reads it); the barrier also makes every epilogue warp leave
      // together after a timeout.
      const bool restage = n0 != staged_n0;
      if (restage) {
        cbuf ^= 1;
        staged_n0 = n0;
      }
      float* cf = epi_coef + cbuf * kEpiCoefVectors * NT;
      for (int j = etid; restage && j < NT; j += kEW * 32) {
        const int n = n0 + j;
        const int ch = kConv ? n % a.c_out : n;
        cf[j] = a.bias ? __ldg(a.bias + ch) : 0.f;
        if (OUT != kOutNone) {
          cf[NT + j] = __ldg(a.next_alpha + ch);
          cf[2 * NT + j] = __ldg(a.next_recip + ch);
        }
        if (kOutPl || kOutA) {
          cf[3 * NT + j] = __ldg(a.next_scale + ch);
          cf[4 * NT + j] = __ldg(a.next_offset + ch);
        }
        if (kI8 && a.w_scale) cf[5 * NT + j] = __ldg(a.w_scale + n);
        if (kI8Tconv) cf[6 * NT + j] = __ldg(a.w_scale2 + n);
      }
      if (!named_barrier_and(3, kEW * 32, ok)) break;
      const int row0 = m0 + q * 32;
      const int g = row0 + lane;
      const int N = a.rows_per_stream;
      // Plane / activation writers: this row's time step and, at a stream's
      // last step, the next layer's new history row; the stem also reads the
      // old one at a stream's first step.
      constexpr bool kStemPl = kOutPl && KIND == kStem;
      int t_row = -1;
      const uint32_t* hist_old = nullptr;
      uint32_t* hist_new = nullptr;
      int* head_out = nullptr;
      int head_next = 0;
      if ((kOutPl || kOutA) && g < a.rows) {
        const int sid = g / N;
        t_row = g - sid * N;
        if (a.state.pool && (t_row == N - 1 || (kStemPl && t_row == 0))) {
          const int code = a.state.slot_codes ? a.state.slot_codes[sid] : ((sid << 2) | a.state.uniform_code);
          float* slot = slot_base(a.state, code);
          const HistRef& h = a.hist_next;  // one row (H = 1): window = ring row head
          const int head = (code & 2) ? 0 : head_table(slot, code & 1)[h.index];
          if (kStemPl && t_row == 0 && !(code & 2))
            hist_old = reinterpret_cast<const uint32_t*>(slot + h.ring + head * h.width);
          if (t_row == N - 1) {
            hist_new = reinterpret_cast<uint32_t*>(slot + h.ring + (head ^ 1) * h.width);
            if (n0 == 0 && cg == 0) {
              head_out = head_table(slot, (code & 1) ^ 1) + h.index;
              head_next = head ^ 1;
            }
          }
        }
      }
      int tq[4];  // plane writers: time step of row 8k + lane/4 (-1 past the last row)
      if constexpr (kOutPl) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int gr = row0 + 8 * k + (lane >> 2);
          tq[k] = gr < a.rows ? gr - (gr / N) * N : -1;
        }
      }
      // The tile's skip input rows into L2 while the accumulator is produced
      // (one bulk prefetch per row), so the chunk loads below hit L2.
      if (kSkipAdd && g < a.rows && cg == 0) prefetch_l2(a.x + (size_t)g * a.c_out + n0, NT * 4);
      float4 xr[4];  // skip input of the current chunk, coalesced order
      load_skip<KIND>(a, row0, n0 + cg * kEpiCols, lane, xr);
      uint4 hw[4];  // stem: history bits of this chunk (zero without a history row)
      if constexpr (kStemPl) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          hw[j] = hist_old ? __ldg(reinterpret_cast<const uint4*>(hist_old + n0) + j) : make_uint4(0u, 0u, 0u, 0u);
      }
      // Waits whose outcome steers warp-collective code (tcgen05.ld, __syncwarp)
      // are made warp-uniform: a warp goes on only if every lane saw the phase.
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[buf], (i >> 1) & 1, a.status, kDevTimeoutEpilogue, wl))))
        continue;
      tc_fence_after();
      // int8: this row's activation scales (current and previous tap).
      float sx = 1.f, sxp = 1.f;
      if constexpr (kI8 && KIND == kResidualPre) {
        sx = g < a.rows ? __ldg(a.row_scale + g) : 1.f;  // written by the quantising pre-pass
      } else if constexpr (kI8 && KIND != kTestGemm) {
        if (!(ok = __all_sync(0xffffffffu, mbar_wait(&scale_full[buf], (i >> 1) & 1, a.status, kDevTimeoutEpilogue, wl))))
          continue;
        const float* sb = scales + buf * 2 * kTileM;
        sx = sb[q * 32 + lane];
        if (kI8Tconv) sxp = sb[kTileM + q * 32 + lane];
        __syncwarp();
        if (lane == 0) mbar_arrive(&scale_empty[buf]);
      }
      const uint32_t base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * Cfg::kAccCols);
      float rmax = 0.f;  // kEpiAct: max |output| of this row over the tile's columns
      uint32_t r[16];
      tmem_ld16_async(base + cg * kEpiCols, r);
      tmem_wait_ld(r);
#pragma unroll 1
      for (int c = cg; c < kChunks; c += kCG) {
        const int n = n0 + c * kEpiCols;
        const int j0 = c * kEpiCols;
        uint32_t rn[16];
        uint32_t rp[16];  // int8 transposed conv: previous-tap accumulator
        if constexpr (kI8Tconv) {
          tmem_ld16_async(base + NT + c * kEpiCols, rp);
          tmem_wait_ld(rp);
        }
        // Next chunk's accumulator columns (the last chunk reloads its own):
        // issued and waited for unconditionally, so the registers the load
        // writes asynchronously never meet a control-flow merge before the wait.
        tmem_ld16_async(base + (c + kCG < kChunks ? c + kCG : c) * kEpiCols, rn);
        float4 x[4];  // this lane's row of the skip input
        if (kSkipAdd) transpose_skip(stage, lane, xr, x);
        uint4 wn[4];  // stem: next chunk's history bits
        if (kStemPl && hist_old && c + kCG < kChunks) {
#pragma unroll
          for (int j = 0; j < 4; ++j) wn[j] = __ldg(reinterpret_cast<const uint4*>(hist_old + n + kCG * kEpiCols) + j);
        }
        float4 xn[4];  // next chunk's skip input
        load_skip<KIND>(a, c + kCG < kChunks ? row0 : a.rows, n + kCG * kEpiCols, lane, xn);
        float v[16];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float4 b = lds4(cf + j0 + 4 * j);
          float4 acc;
          if constexpr (kI8) {
            // Reference ip_run_rows: float(dot) * (s_w * s_x); transposed conv:
            // (current + previous) + bias; residual: x + (product + bias).
            const float4 sw = lds4(cf + 5 * NT + j0 + 4 * j);
            acc.x = __fmul_rn(__int2float_rn((int)r[4 * j]), __fmul_rn(sw.x, sx));
            acc.y = __fmul_rn(__int2float_rn((int)r[4 * j + 1]), __fmul_rn(sw.y, sx));
            acc.z = __fmul_rn(__int2float_rn((int)r[4 * j + 2]), __fmul_rn(sw.z, sx));
            acc.w = __fmul_rn(__int2float_rn((int)r[4 * j + 3]), __fmul_rn(sw.w, sx));
            if constexpr (kI8Tconv) {
              const float4 sw2 = lds4(cf + 6 * NT + j0 + 4 * j);
              acc.x = __fadd_rn(acc.x, __fmul_rn(__int2float_rn((int)rp[4 * j]), __fmul_rn(sw2.x, sxp)));
              acc.y = __fadd_rn(acc.y, __fmul_rn(__int2float_rn((int)rp[4 * j + 1]), __fmul_rn(sw2.y, sxp)));
              acc.z = __fadd_rn(acc.z, __fmul_rn(__int2float_rn((int)rp[4 * j + 2]), __fmul_rn(sw2.z, sxp)));
              acc.w = __fadd_rn(acc.w, __fmul_rn(__int2float_rn((int)rp[4 * j + 3]), __fmul_rn(sw2.w, sxp)));
            }
            if (KIND == kTestGemm) {
              acc = make_float4(__int2float_rn((int)r[4 * j]), __int2float_rn((int)r[4 * j + 1]),
                                __int2float_rn((int)r[4 * j + 2]), __int2float_rn((int)r[4 * j + 3]));
            }
          } else {
            acc = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]), __uint_as_float(r[4 * j + 2]),
                              __uint_as_float(r[4 * j + 3]));
          }
          v[4 * j] = acc.x + b.x;
          v[4 * j + 1] = acc.y + b.y;
          v[4 * j + 2] = acc.z + b.z;
          v[4 * j + 3] = acc.w + b.w;
          if (kSkipAdd) {
            v[4 * j] = x[j].x + v[4 * j];
            v[4 * j + 1] = x[j].y + v[4 * j + 1];
            v[4 * j + 2] = x[j].z + v[4 * j + 2];
            v[4 * j + 3] = x[j].w + v[4 * j + 3];
          }
        }
        {
          // fp32 outputs: row g, column n at g * pitch + n (a transposed conv's
          // output row g * stride + p holds GEMM columns p * c_out ..).
          const size_t pitch = kConv ? (size_t)a.stride * a.c_out : (size_t)a.c_out;
          const size_t off0 = (size_t)row0 * pitch + n;
          if (epi & kEpiX) store_chunk(stage, lane, v, a.out_x + off0, pitch, a.rows - row0);
          if constexpr (OUT != kOutNone) {
            float s[16];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              float4 u = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
              if (kOutPl || kOutA) {
                const float4 sc = lds4(cf + 3 * NT + j0 + 4 * j), of = lds4(cf + 4 * NT + j0 + 4 * j);
                u = make_float4(__fadd_rn(__fmul_rn(u.x, sc.x), of.x), __fadd_rn(__fmul_rn(u.y, sc.y), of.y),
                                __fadd_rn(__fmul_rn(u.z, sc.z), of.z), __fadd_rn(__fmul_rn(u.w, sc.w), of.w));
              }
              u = snake4<kI8 || kOutA>(u, lds4(cf + NT + j0 + 4 * j), lds4(cf + 2 * NT + j0 + 4 * j));
              s[4 * j] = u.x;
              s[4 * j + 1] = u.y;
              s[4 * j + 2] = u.z;
              s[4 * j + 3] = u.w;
            }
            if constexpr (kOutPl) {
              uint32_t hi[8], lo[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) split_bf16(s[2 * j], s[2 * j + 1], hi[j], lo[j]);
              const size_t plane = (size_t)a.rows * a.c_out;
              store_planes_chunk(stage, lane, hi, lo, a.out_planes, a.out_planes_prev, plane,
                                 (size_t)row0 * a.c_out + n, a.c_out, N, tq);
              if (g < a.rows) {
              if (t_row + 1 >= N && hist_new) {
                // New history row, packed per channel as (hi << 16) | lo.
                uint4* dst = reinterpret_cast<uint4*>(hist_new + n);
#pragma unroll
                for (int j = 0; j < 4; ++j)
                  dst[j] = make_uint4(__byte_perm(lo[2 * j], hi[2 * j], 0x5410), __byte_perm(lo[2 * j], hi[2 * j], 0x7632),
                                      __byte_perm(lo[2 * j + 1], hi[2 * j + 1], 0x5410),
                                      __byte_perm(lo[2 * j + 1], hi[2 * j + 1], 0x7632));
              }
              if (kStemPl && t_row == 0) {
                // A stream's first row of the shifted planes: the previous activated input.
                uint4* ph = reinterpret_cast<uint4*>(a.out_planes_prev + (size_t)g * a.c_out + n);
                uint4* pl = reinterpret_cast<uint4*>(a.out_planes_prev + (size_t)g * a.c_out + n + plane);
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                  ph[j] = make_uint4(__byte_perm(hw[2 * j].x, hw[2 * j].y, 0x7632), __byte_perm(hw[2 * j].z, hw[2 * j].w, 0x7632),
                                     __byte_perm(hw[2 * j + 1].x, hw[2 * j + 1].y, 0x7632),
                                     __byte_perm(hw[2 * j + 1].z, hw[2 * j + 1].w, 0x7632));
                  pl[j] = make_uint4(__byte_perm(hw[2 * j].x, hw[2 * j].y, 0x5410), __byte_perm(hw[2 * j].z, hw[2 * j].w, 0x5410),
                                     __byte_perm(hw[2 * j + 1].x, hw[2 * j + 1].y, 0x5410),
                                     __byte_perm(hw[2 * j + 1].z, hw[2 * j + 1].w, 0x5410));
                }
              }
              }
            } else if constexpr (OUT == kOutS16) {
              // f16 Snake output: this lane's row, 16 columns as 32 contiguous bytes.
              if (g < a.rows) {
                uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(a.out_s) + off0 + (size_t)lane * pitch);
                dst[0] = make_uint4(pack_f16(s[0], s[1]), pack_f16(s[2], s[3]), pack_f16(s[4], s[5]), pack_f16(s[6], s[7]));
                dst[1] = make_uint4(pack_f16(s[8], s[9]), pack_f16(s[10], s[11]), pack_f16(s[12], s[13]),
                                    pack_f16(s[14], s[15]));
              }
            } else {
              store_chunk(stage, lane, s, a.out_s + off0, pitch, a.rows - row0);
              if constexpr (kOutA) {
                if (g < a.rows) {
#pragma unroll
                  for (int j = 0; j < 16; ++j) rmax = fmaxf(rmax, fabsf(s[j]));
                  if (hist_new) st4(reinterpret_cast<float*>(hist_new) + n, s);
                }
              }
            }
          }
        }
        tmem_wait_ld(rn);
#pragma unroll
        for (int j = 0; j < 16; ++j) r[j] = rn[j];
#pragma unroll
        for (int j = 0; j < 4; ++j) xr[j] = xn[j];
        if (kStemPl && hist_old && c + kCG < kChunks) {
#pragma unroll
          for (int j = 0; j < 4; ++j) hw[j] = wn[j];
        }
      }
      // One partial maximum per N tile and column group.
      if (kOutA && g < a.rows) a.rowmax_out[(size_t)g * a.rowmax_parts + (n0 / NT) * kCG + cg] = rmax;
      if (head_out) *head_out = head_next;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  } else if (warp == kLoaderWarp) {
    if (lane == 0) {
      // ---- weight tiles: one bulk copy per stage, or, from an image packed
      // for wider N tiles, one copy per operand term of this tile's rows
      const int img_nt = a.img_nt ? a.img_nt : NT;
      uint32_t g = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const int n0 = tile_n(t) * NT;
        const uint8_t* src = a.wimg + (size_t)(n0 / img_nt) * num_kb * Cfg::kTerms * img_nt * 128 +
                             (size_t)(n0 % img_nt) * 128;
        for (int kb = 0; kb < num_kb; ++kb, ++g) {
          const int s = g % S;
          const uint32_t ph = (g / S) & 1;
          if (!(ok = mbar_wait(&empty[s], ph ^ 1, a.status, kDevTimeoutLoader, wl))) break;
          mbar_arrive_expect_tx(&b_full[s], Cfg::kBStage);
          if (img_nt == NT) {
            bulk_g2s(b_base + s * Cfg::kBStage, src + (size_t)kb * Cfg::kBStage, Cfg::kBStage, &b_full[s]);
          } else {
#pragma unroll
            for (int term = 0; term < Cfg::kTerms; ++term)
              bulk_g2s(b_base + s * Cfg::kBStage + term * Cfg::kBTile,
                       src + ((size_t)kb * Cfg::kTerms + term) * img_nt * 128, Cfg::kBTile, &b_full[s]);
          }
        }
      }
      drain_fills(b_full, g, S, a.status, kDevTimeoutLoader);
    }
  } else if (warp == kRawWarp) {
    if (lane == 0 && KIND == kResidualPre) {
      // ---- preformed residual A operand: one 128-row box of 128 bytes per row
      // per K block (64 f16 channels, or an int8 plan's 128 s8 channels)
      uint32_t g = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const int m0 = tile_m(t) * kTileM;
        for (int kb = 0; kb < num_kb; ++kb, ++g) {
          const int s = g % S;
          const uint32_t ph = (g / S) & 1;
          if (!(ok = mbar_wait(&empty[s], ph ^ 1, a.status, kDevTimeoutLoader, wl))) break;
          mbar_arrive_expect_tx(&a_full[s], Cfg::kAStage);
          tma_load_2d(a_base + s * Cfg::kAStage, &a.tmap, kb * (kI8 ? kKBlockI8 : kKBlock), m0, &a_full[s]);
        }
      }
      drain_fills(a_full, g, S, a.status, kDevTimeoutLoader);
    } else if (lane == 0 && KIND == kTconvPre) {
      // ---- preformed int8 transposed-conv taps: one 128-channel x 128-row s8
      // box per tap per K block
      uint32_t g = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const int m0 = tile_m(t) * kTileM;
        for (int kb = 0; kb < num_kb; ++kb, ++g) {
          const int s = g % S;
          const uint32_t ph = (g / S) & 1;
          if (!(ok = mbar_wait(&empty[s], ph ^ 1, a.status, kDevTimeoutLoader, wl))) break;
          mbar_arrive_expect_tx(&a_full[s], Cfg::kAStage);
          tma_load_2d(a_base + s * Cfg::kAStage, &a.tmap, kb * kKBlockI8, m0, &a_full[s]);
          tma_load_2d(a_base + s * Cfg::kAStage + Cfg::kATile, &a.tmap2, kb * kKBlockI8, m0, &a_full[s]);
        }
      }
      drain_fills(a_full, g, S, a.status, kDevTimeoutLoader);
    } else if (lane == 0 && KIND == kTconv && !kI8) {
      // ---- transposed-conv A operand: tap 0 from the planes, tap 1 from the
      // shifted planes, hi and lo tiles in one 3-D box
      const int kpt = a.k_channels / kKBlock;
      uint32_t g = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const int m0 = tile_m(t) * kTileM;
        for (int kb = 0; kb < num_kb; ++kb, ++g) {
          const int s = g % S;
          const uint32_t ph = (g / S) & 1;
          if (!(ok = mbar_wait(&empty[s], ph ^ 1, a.status, kDevTimeoutLoader, wl))) break;
          const int tap = kb / kpt, cb = kb - tap * kpt;
          mbar_arrive_expect_tx(&a_full[s], Cfg::kAStage);
          tma_load_3d(a_base + s * Cfg::kAStage, tap ? &a.tmap2 : &a.tmap, cb * kKBlock, m0, 0, &a_full[s]);
        }
      }
      drain_fills(a_full, g, S, a.status, kDevTimeoutLoader);
    } else if (lane == 0 && (KIND == kResidual || kI8Tconv)) {
      // ---- staged producer inputs. Residual: per 64-channel block the tile +
      // causal halo rows of s and the block's coefficients. int8 transposed
      // conv: per 64-channel half of a K block, input rows m0-1 .. m0+127.
      const int halo = KIND == kResidual ? a.box_rows - kTileM : 1;
      const uint32_t bytes = KIND == kResidual ? (uint32_t)a.box_rows * a.raw_pitch * (a.s16 ? 2 : 4) + kResCoefBytes
                                               : (uint32_t)(kTileM + 1) * 64 * 4;
      const int boxes = KIND == kResidual ? (a.k_channels < kKBlock ? 1 : a.k_channels / kKBlock) : 2 * num_kb;
      uint32_t g = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const int m0 = tile_m(t) * kTileM;
        for (int kb = 0; kb < boxes; ++kb, ++g) {
          const int rb = g & 1;
          if (!(ok = mbar_wait(&raw_empty[rb], ((g >> 1) & 1) ^ 1, a.status, kDevTimeoutLoader, wl))) break;
          uint8_t* dst = raw_base + rb * Cfg::kRaw;
          mbar_arrive_expect_tx(&raw_full[rb], bytes);
          tma_load_2d(dst, &a.tmap, kb * kKBlock, m0 - halo, &raw_full[rb]);
          if (KIND == kResidual)
            bulk_g2s(dst + kResBoxBytes, a.coef + (size_t)kb * kCoefResidual * 64, kResCoefBytes, &raw_full[rb]);
        }
      }
      drain_fills(raw_full, g, 2, a.status, kDevTimeoutLoader);
    }
  } else if (warp == kSchedWarp) {
    // ---- scheduler: per-tile stream/row tables (and the int8 transposed
    // conv's row scales), one tile ahead of the producers
    if (KIND == kResidualPre && (a.epi & kEpiPlanes)) {
      // No producers: the table only serves the stream-start plane rows.
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
        const int m0 = tile_m(t) * kTileM;
        const StreamTable tab = table_at(table, m0, a.rows_per_stream);
        fill_table(a, m0, tab, lane);
        __syncwarp();
        first_rows_prev_planes(a, m0, tile_n(t) * NT, NT, tab, lane);
        __syncwarp();
      }
    } else if (KIND == kStem || KIND == kResidual || kI8Tconv) {
      uint32_t ti = 0;
      for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++ti) {
        const int m0 = tile_m(t) * kTileM;
        // (A TMA-fed int8 conv has no producers to hand the table to.)
        if (!kTmaA && !__all_sync(0xffffffffu, mbar_wait(&table_empty[ti & 1], ((ti >> 1) & 1) ^ 1, a.status,
                                                         kDevTimeoutProducer, wl)))
          break;
        int* tbase = table + (ti & 1) * Cfg::kTableI;
        const StreamTable tab = table_at(tbase, m0, a.rows_per_stream);
        fill_table(a, m0, tab, lane);
        __syncwarp();
        if constexpr (kI8Tconv) {
          // Row scales of the input rows (max over the previous layer's N tiles).
          float* sc = reinterpret_cast<float*>(tbase + kTableInts);
          auto row_max = [&](int gr) {
            float m = 0.f;
            for (int p = 0; p < a.rowmax_in_parts; ++p) m = fmaxf(m, __ldg(a.rowmax_in + (size_t)gr * a.rowmax_in_parts + p));
            return m;
          };
          const bool write_state = tile_n(t) == 0;
          for (int r = lane; r < kTileM; r += 32) {
            const int gr = m0 + r;
            const int e = tab.row_e[r];
            const float mx = e >= 0 ? row_max(gr) : 0.f;
            sc[r] = quant_scale(mx);
            float prev = 0.f;  // max |x| of the previous time step
            if (e >= 0) {
              if (tab.row_t[r] > 0) {
                prev = row_max(gr - 1);
              } else if (a.state.pool && !(tab.code[e] & 2)) {
                prev = __int_as_float(head_table(slot_base(a.state, tab.code[e]), tab.code[e] & 1)[a.hist_max_slot]);
              }
              // The history of the next step: this stream's last step's max.
              if (write_state && a.state.pool && tab.row_t[r] == a.rows_per_stream - 1)
                head_table(slot_base(a.state, tab.code[e]), (tab.code[e] & 1) ^ 1)[a.hist_max_slot] = __float_as_int(mx);
            }
            sc[kTileM + r] = quant_scale(prev);
          }
          __syncwarp();
          if (!__all_sync(0xffffffffu, mbar_wait(&scale_empty[ti & 1], ((ti >> 1) & 1) ^ 1, a.status,
                                                 kDevTimeoutProducer, wl)))
            break;
          float* sb = scales + (ti & 1) * 2 * kTileM;
          for (int r = lane; r < 2 * kTileM; r += 32) sb[r] = sc[r];
          __syncwarp();
          if (lane == 0) mbar_arrive(&scale_full[ti & 1]);
        }
        if (lane == 0 && !kTmaA) mbar_arrive(&table_full[ti & 1]);
        // After publishing the table: nothing in this kernel reads these rows.
        if (KIND == kResidual && (a.epi & kEpiPlanes)) first_rows_prev_planes(a, m0, tile_n(t) * NT, NT, tab, lane);
      }
    }
  } else {
    // ---- MMA issuer
    if (lane == 0) {
      uint32_t g = 0, i = 0;
      bool ok = a.gate == nullptr || flag_wait(a.gate, a.status, kDevTimeoutGate, wl);
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++i) {
        const int buf = i & 1;
        if (!(ok = mbar_wait(&acc_empty[buf], ((i >> 1) & 1) ^ 1, a.status, kDevTimeoutMma, wl))) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * Cfg::kAccCols);
        for (int kb = 0; kb < num_kb; ++kb, ++g) {
          const int s = g % S;
          const uint32_t ph = (g / S) & 1;
          ok = mbar_wait(&a_full[s], ph, a.status, kDevTimeoutMma, wl) &&
               mbar_wait(&b_full[s], ph, a.status, kDevTimeoutMma, wl);
          if (!ok) break;
          tc_fence_after();
          const uint32_t a0 = smem_u32(a_base + s * Cfg::kAStage);
          const uint32_t b0 = smem_u32(b_base + s * Cfg::kBStage);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t ko = k * 32;  // 32 bytes of K per MMA (16 f16/bf16 or 32 s8)
            const uint32_t acc = (kb | k) ? 1u : 0u;
            if constexpr (kI8) {
              mma_i8(d, smem_desc_sw128(a0 + ko), smem_desc_sw128(b0 + ko), Cfg::kIdesc, acc);
              if (kI8Tconv)
                mma_i8(d + NT, smem_desc_sw128(a0 + Cfg::kATile + ko), smem_desc_sw128(b0 + Cfg::kBTile + ko),
                       Cfg::kIdesc, acc);
            } else {
              mma_f16(d, smem_desc_sw128(a0 + ko), smem_desc_sw128(b0 + ko), Cfg::kIdesc, acc);
              if (kSplitOperands<MODE>) {
                mma_f16(d, smem_desc_sw128(a0 + ko), smem_desc_sw128(b0 + Cfg::kBTile + ko), Cfg::kIdesc, 1u);
                mma_f16(d, smem_desc_sw128(a0 + Cfg::kATile + ko), smem_desc_sw128(b0 + ko), Cfg::kIdesc, 1u);
              }
              if (MODE == kModeSplit4)
                mma_f16(d, smem_desc_sw128(a0 + Cfg::kATile + ko), smem_desc_sw128(b0 + Cfg::kBTile + ko),
                        Cfg::kIdesc, 1u);
            }
          }
          mma_commit(&empty[s]);
        }
        if (ok) mma_commit(&acc_full[buf]);
      }
      // Every MMA this thread issued has finished before TMEM is freed (after a
      // timeout, MMAs committed to a stage barrier nobody waits for may still run).
      mma_commit(mma_drain);
      mbar_wait(mma_drain, 0, a.status, kDevTimeoutMma);
    }
  }
done:
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

static int g_sm_count = 0;

template <int NT, int MODE, int KIND, int OUT>
static cudaError_t launch_cfg(const LayerArgs& a, cudaStream_t stream) {
  using Cfg = GemmCfg<NT, MODE, KIND>;
  const int tiles = ((a.rows + kTileM - 1) / kTileM) * (a.n_total / NT);
  int grid = tiles < g_sm_count ? tiles : g_sm_count;
  return launch_overlapped(gemm_layer_kernel<NT, MODE, KIND, OUT>, grid, kThreads, Cfg::kSmem, stream, a);
}

template <int NT, int MODE, int KIND, int OUT>
static cudaError_t set_smem() {
  using Cfg = GemmCfg<NT, MODE, KIND>;
  return cudaFuncSetAttribute(gemm_layer_kernel<NT, MODE, KIND, OUT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              Cfg::kSmem);
}

// The (N tile, operand mode, layer kind, epilogue output) combinations the
// step schedules use; anything else is rejected at launch.
#define FAV_CONFIGS(X)                                                                                      \
  X(256, kModeSplit4, kStem, kOutPlanes) X(64, kModeSplit4, kStem, kOutPlanes)                            \
  X(256, kModeSplit4, kStem, kOutAct)                                                                      \
  X(256, kModeSplit, kTconv, kOutS) X(128, kModeSplit, kTconv, kOutS) X(64, kModeSplit, kTconv, kOutS)      \
  X(128, kModeI8, kTconv, kOutS) X(128, kModeI8, kTconvPre, kOutS) X(128, kModeI8, kTconv, kOutS16)       \
  X(128, kModeI8, kTconvPre, kOutS16)                                                                      \
  X(64, kModeSplit, kTconv, kOutNone) X(128, kModeSplit, kTconv, kOutNone) X(128, kModeI8, kTconv, kOutNone) \
  X(256, kModeSplit, kTconv, kOutNone)                                                                     \
  X(256, kModeF16, kResidual, kOutS) X(128, kModeF16, kResidual, kOutS) X(64, kModeF16, kResidual, kOutS)  \
  X(256, kModeSplit, kTconv, kOutS16) X(128, kModeSplit, kTconv, kOutS16) X(64, kModeSplit, kTconv, kOutS16)   \
  X(256, kModeF16, kResidual, kOutS16) X(128, kModeF16, kResidual, kOutS16) X(64, kModeF16, kResidual, kOutS16) \
  X(256, kModeF16, kResidualPre, kOutS) X(256, kModeF16, kResidualPre, kOutPlanes)                          \
  X(64, kModeF16, kResidualPre, kOutS) X(64, kModeF16, kResidualPre, kOutPlanes)                            \
  X(256, kModeI8, kResidualPre, kOutS) X(128, kModeI8, kResidualPre, kOutS)                                \
  X(256, kModeI8, kResidualPre, kOutAct) X(128, kModeI8, kResidualPre, kOutAct)                            \
  X(32, kModeF16, kResidual, kOutS) X(256, kModeF16, kResidual, kOutPlanes)                                \
  X(128, kModeF16, kResidual, kOutPlanes) X(64, kModeF16, kResidual, kOutPlanes)                           \
  X(256, kModeF16, kTestGemm, kOutNone) X(128, kModeF16, kTestGemm, kOutNone)                              \
  X(64, kModeF16, kTestGemm, kOutNone) X(32, kModeF16, kTestGemm, kOutNone)                                \
  X(256, kModeSplit, kTestGemm, kOutNone) X(128, kModeSplit, kTestGemm, kOutNone)                          \
  X(64, kModeSplit, kTestGemm, kOutNone) X(32, kModeSplit, kTestGemm, kOutNone)                            \
  X(256, kModeI8, kTestGemm, kOutNone) X(128, kModeI8, kTestGemm, kOutNone)                                \
  X(64, kModeI8, kTestGemm, kOutNone) X(32, kModeI8, kTestGemm, kOutNone)

cudaError_t prepare_kernels() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&g_sm_count, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
#define FAV_SET(NT, MODE, KIND, OUT) \
  if ((e = set_smem<NT, MODE, KIND, OUT>()) != cudaSuccess) return e;
  FAV_CONFIGS(FAV_SET)
#undef FAV_SET
  if ((e = prepare_stage()) != cudaSuccess) return e;
  return prepare_tail();
}

int epilogue_column_groups(int n_tile, int kind) {
  return (kind == kResidualPre || kind == kTconvPre) && n_tile >= 64 ? (kEpilogueWarps + kProducerWarps) / 4 : 1;
}

cudaError_t launch_gemm_layer(const LayerArgs& a, cudaStream_t stream) {
  if (a.rows <= 0) return cudaSuccess;
  if ((a.epi & kEpiAct) &&
      (a.rowmax_parts != (a.n_total / a.n_tile) * epilogue_column_groups(a.n_tile, a.kind) ||
       a.rowmax_parts > kMaxRowmaxParts))
    return cudaErrorInvalidValue;
  if (a.n_total % a.n_tile) return cudaErrorInvalidValue;
  if (a.img_nt && (a.img_nt % a.n_tile || a.n_total % a.img_nt)) return cudaErrorInvalidValue;
  // A residual unit's staged box (tile + halo rows) must fit its raw buffer.
  if (a.kind == kResidual && (size_t)a.box_rows * a.raw_pitch * (a.s16 ? 2 : 4) > (size_t)kResBoxBytes)
    return cudaErrorInvalidValue;
  const int out = (a.epi & kEpiPlanes) ? kOutPlanes : (a.epi & kEpiAct) ? kOutAct : (a.epi & kEpiS) ? kOutS
                  : (a.epi & kEpiS16) ? kOutS16 : kOutNone;
#define FAV_LAUNCH(NT, MODE, KIND, OUT) \
  if (a.n_tile == NT && a.mode == MODE && a.kind == KIND && out == OUT) return launch_cfg<NT, MODE, KIND, OUT>(a, stream);
  FAV_CONFIGS(FAV_LAUNCH)
#undef FAV_LAUNCH
  return cudaErrorInvalidValue;
}

// ------------------------------------------------------------------ final conv
// Causal conv 32->1 (k=7) -> tanh on CUDA cores over s = Snake_final(y), which
// the last residual unit's epilogue wrote. 256 output rows per block with a
// 6-row halo staged in shared memory; a stream has at least 1920 rows here, so
// a block touches at most two streams. History = last six rows of s [6][32].
constexpr int kFinalRows = 256;
constexpr int kFinalPitch = 33;
constexpr int kFinalLoads = ((kFinalRows + 6) * kFinalChannels + kFinalRows - 1) / kFinalRows;

__device__ __forceinline__ int final_code(const StateRef& st, int s) {
  return st.slot_codes ? st.slot_codes[s] : ((s << 2) | st.uniform_code);
}

__global__ void __launch_bounds__(kFinalRows) final_kernel(const FinalArgs a) {
  __shared__ float act[(kFinalRows + 6) * kFinalPitch];
  __shared__ float wsm[kFinalChannels * 7];
  const int g0 = blockIdx.x * kFinalRows;
  const int N = a.rows_per_stream;
  for (int i = threadIdx.x; i < kFinalChannels * 7; i += kFinalRows) wsm[i] = __ldg(a.w + i);
  const int ch = threadIdx.x & (kFinalChannels - 1);
  {
    float v[kFinalLoads];
#pragma unroll
    for (int j = 0; j < kFinalLoads; ++j) {
      const int i = threadIdx.x + j * kFinalRows;
      const int g = g0 - 6 + i / kFinalChannels;
      v[j] = (i < (kFinalRows + 6) * kFinalChannels && g >= 0 && g < a.rows)
                 ? __ldg(a.x + (size_t)g * kFinalChannels + ch)
                 : 0.f;
    }
#pragma unroll
    for (int j = 0; j < kFinalLoads; ++j) {
      const int i = threadIdx.x + j * kFinalRows;
      if (i < (kFinalRows + 6) * kFinalChannels) act[(i / kFinalChannels) * kFinalPitch + ch] = v[j];
    }
  }
  __syncthreads();
  const int g_end = min(g0 + kFinalRows, a.rows);
  const HistRef& h = a.hist;
  // New window (last six rows of s) of streams ending in this block.
  if (a.state.pool) {
    const int s_lo = g0 / N, s_hi = (g_end - 1) / N;
    for (int s = s_lo; s <= s_hi; ++s) {
      const int last = s * N + N - 1;
      if (last < g0 || last >= g_end) continue;
      const int code = final_code(a.state, s);
      const int head = (code & 2) ? 0 : head_table(slot_base(a.state, code), code & 1)[h.index];
      for (int i = threadIdx.x; i < 6 * kFinalChannels; i += kFinalRows) {
        const int q = i / kFinalChannels, c = i - q * kFinalChannels;
        hist_new_row(a.state, h, code, head, N - 6 + q, N)[c] = act[(last - 5 + q - g0 + 6) * kFinalPitch + c];
      }
      if (threadIdx.x == 0) hist_commit_head(a.state, h, code, head, N);
    }
  }
  const int g = g0 + threadIdx.x;
  if (g < a.rows) {
    const int s = g / N, t = g - s * N;
    const float* hist = nullptr;
    int head = 0;
    if (t < 6 && a.state.pool) {
      const int code = final_code(a.state, s);
      if (!(code & 2)) {
        head = head_table(slot_base(a.state, code), code & 1)[h.index];
        hist = slot_base(a.state, code) + h.ring;
      }
    }
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 7; ++j) {
      const int tp = t - 6 + j;
      const float* row = act + (threadIdx.x + j) * kFinalPitch;
      const float* hrow = nullptr;
      if (tp < 0 && hist) hrow = hist + ((head + 6 + tp) % 12) * kFinalChannels;
#pragma unroll 8
      for (int c = 0; c < kFinalChannels; ++c) {
        const float v = tp >= 0 ? row[c] : (hrow ? __ldg(hrow + c) : 0.f);
        acc = fmaf(wsm[c * 7 + j], v, acc);
      }
    }
    const float y = tanhf(acc + __ldg(a.b));
    // The reference checks the audio is finite (gpu.py:182-184); the step's
    // status word carries that check, so the host need not scan the audio.
    if (!(fabsf(y) <= 1.f)) record_error(a.status, kDevNonFinite);
    a.audio[(size_t)s * a.audio_stride + a.audio_offset + t] = y;
  }
}

cudaError_t launch_final(const FinalArgs& a, cudaStream_t stream) {
  if (a.rows <= 0) return cudaSuccess;
  final_kernel<<<(a.rows + kFinalRows - 1) / kFinalRows, kFinalRows, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace fav

namespace fav {

// ------------------------------------------------------------- int8 stem
// The int8 plan's stem on CUDA cores: a quantised cascade follows, so every
// sum runs in the int8 oracle's order (oracle/exact.py): depthwise taps oldest
// first then the bias, the 1x1 over input channels in order then the bias,
// then stage 0's affine and Snake (kEpiAct). Eight rows per block of 256
// threads; a thread owns 8 output channels.
constexpr int kStemRows = 8;

__global__ void __launch_bounds__(256) stem_exact_kernel(const __grid_constant__ LayerArgs a) {
  __shared__ float dwc[kStemRows][kLatentChannels];
  __shared__ float wmax[kStemRows][8];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g0 = blockIdx.x * kStemRows;
  const int T = a.rows_per_stream;
  // Depthwise conv (history = last six latent frames) for this block's rows.
  for (int i = tid; i < kStemRows * kLatentChannels; i += 256) {
    const int r = i / kLatentChannels, c = i - r * kLatentChannels;
    const int g = g0 + r;
    float y = 0.f;
    if (g < a.rows) {
      const int s = g / T, t = g - s * T;
      const float* z0 = a.x + ((size_t)s * kLatentChannels + c) * a.z_stride + a.z_offset;
      int code = 0, head = 0;
      const float* ring = nullptr;
      if (a.state.pool) {
        code = a.state.slot_codes ? a.state.slot_codes[s] : ((s << 2) | a.state.uniform_code);
        if (!(code & 2)) {
          head = head_table(slot_base(a.state, code), code & 1)[a.hist.index];
          ring = slot_base(a.state, code) + a.hist.ring;
        }
      }
      for (int j = 0; j < 7; ++j) {
        const int tp = t - 6 + j;
        float v = 0.f;
        if (tp >= 0) v = __ldg(z0 + tp);
        else if (ring) v = ring[((head + 6 + tp) % 12) * kLatentChannels + c];
        const float p = __fmul_rn(__ldg(a.dw_w + c * 7 + j), v);
        y = j ? __fadd_rn(y, p) : p;
      }
      y = __fadd_rn(y, __ldg(a.dw_b + c));
      // The stem history of the next step: the last min(T, 6) frames (zeros
      // before a fresh stream's first frame), written at the stream's last row.
      if (t == T - 1 && a.state.pool) {
        for (int tp = T > 6 ? T - 6 : 0; tp < T; ++tp)
          hist_new_row(a.state, a.hist, code, head, tp, T)[c] = __ldg(z0 + tp);
        if ((code & 2) && T < 6) {
          float* fresh = slot_base(a.state, code) + a.hist.ring;
          for (int j = T; j < 6; ++j) fresh[j * kLatentChannels + c] = 0.f;
        }
        if (c == 0) hist_commit_head(a.state, a.hist, code, head, T);
      }
    }
    dwc[r][c] = y;
  }
  __syncthreads();
  // 1x1 64 -> 2048: channels n = 8*tid .. 8*tid+7 for all eight rows.
  const int n0 = 8 * tid;
  float acc[8][kStemRows];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int r = 0; r < kStemRows; ++r) acc[i][r] = 0.f;
  for (int k = 0; k < kLatentChannels; ++k) {
    float wk[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) wk[i] = __ldg(a.dense_w + (size_t)(n0 + i) * kLatentChannels + k);
#pragma unroll
    for (int r = 0; r < kStemRows; ++r) {
      const float x = dwc[r][k];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float p = __fmul_rn(wk[i], x);
        acc[i][r] = k ? __fadd_rn(acc[i][r], p) : p;
      }
    }
  }
  // Epilogue: y = sum + bias; activation Snake(y * scale + offset); per-row max.
  float rmax[kStemRows];
#pragma unroll
  for (int r = 0; r < kStemRows; ++r) {
    const int g = g0 + r;
    rmax[r] = 0.f;
    float act[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int n = n0 + i;
      const float y = __fadd_rn(acc[i][r], __ldg(a.bias + n));
      if ((a.epi & kEpiX) && g < a.rows) a.out_x[(size_t)g * a.c_out + n] = y;
      const float u = __fadd_rn(__fmul_rn(y, __ldg(a.next_scale + n)), __ldg(a.next_offset + n));
      act[i] = snake_exact(u, __ldg(a.next_alpha + n), __ldg(a.next_recip + n));
      rmax[r] = fmaxf(rmax[r], fabsf(act[i]));
    }
    if (g < a.rows) {
      float4* dst = reinterpret_cast<float4*>(a.out_s + (size_t)g * a.c_out + n0);
      dst[0] = make_float4(act[0], act[1], act[2], act[3]);
      dst[1] = make_float4(act[4], act[5], act[6], act[7]);
      const int s = g / T, t = g - s * T;
      if (t == T - 1 && a.state.pool) {
        // The next layer's (stage 0 transposed conv's) one-row history.
        const int code = a.state.slot_codes ? a.state.slot_codes[s] : ((s << 2) | a.state.uniform_code);
        float* slot = slot_base(a.state, code);
        const HistRef& h = a.hist_next;
        const int head = (code & 2) ? 0 : head_table(slot, code & 1)[h.index];
        float4* hn = reinterpret_cast<float4*>(slot + h.ring + (head ^ 1) * h.width + n0);
        hn[0] = dst[0];
        hn[1] = dst[1];
        if (tid == 0) head_table(slot, (code & 1) ^ 1)[h.index] = head ^ 1;
      }
    }
  }
  // Row maxima over all 2048 channels (rowmax_parts = 1).
#pragma unroll
  for (int r = 0; r < kStemRows; ++r) {
    float m = rmax[r];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) wmax[r][warp] = m;
  }
  __syncthreads();
  if (tid < kStemRows && g0 + tid < a.rows) {
    float m = 0.f;
    for (int w = 0; w < 8; ++w) m = fmaxf(m, wmax[tid][w]);
    a.rowmax_out[(size_t)(g0 + tid) * a.rowmax_parts] = m;
  }
}

__global__ void sine_test_kernel(const float* x, int n, float* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = sin_cw(x[i]);
}

cudaError_t launch_sine_test(const float* x, int n, float* out, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  sine_test_kernel<<<(n + 255) / 256, 256, 0, stream>>>(x, n, out);
  return cudaGetLastError();
}

cudaError_t launch_stem_exact(const LayerArgs& a, cudaStream_t stream) {
  if (a.rows <= 0) return cudaSuccess;
  if (a.n_total != 256 * 8 || a.k_channels != kLatentChannels || a.rowmax_parts != 1) return cudaErrorInvalidValue;
  stem_exact_kernel<<<(a.rows + kStemRows - 1) / kStemRows, 256, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace fav
