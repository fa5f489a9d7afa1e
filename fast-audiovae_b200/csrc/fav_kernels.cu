// sm_100a kernels of the AudioVAE2 decoder step.
//
// One GEMM engine serves every dense layer: rows = time steps of all streams
// (M tile 128), columns = output channels (N tile 32..256), K = input channels.
// Warp roles per CTA (320 threads):
//   warps 0-7  A-operand producers: fused prologue (stage affine + Snake, or
//              Snake -> depthwise k=7 -> Snake, or the stem depthwise conv)
//              written straight into the 128-byte-swizzled K-major MMA tile;
//              afterwards the same warps run the epilogue out of TMEM;
//   warp 8     weight loader: one bulk copy of pre-swizzled weight tiles per stage;
//   warp 9     TMEM owner and MMA issuer (tcgen05.mma, one elected lane).
// Pipelines run through mbarriers; every wait is bounded and records an error
// code in the caller's status word instead of hanging.
#include "fav_device.cuh"
#include "fav_internal.h"

namespace fav {

constexpr int kThreads = 320;
constexpr int kProducerThreads = 256;
constexpr int kSmemBudget = 227 * 1024;
constexpr int kMaxHalo = 54;  // 6 * largest dilation

template <int NT, int MODE, int KIND>
struct GemmCfg {
  static constexpr int kTerms = MODE == kModeSplit ? 2 : 1;
  static constexpr int kATile = kTileM * 128;
  static constexpr int kBTile = NT * 128;
  static constexpr int kAStage = kTerms * kATile;
  static constexpr int kBStage = kTerms * kBTile;
  static constexpr int kStage = kAStage + kBStage;
  static constexpr int kStaging = KIND == kResidual ? (kTileM + kMaxHalo) * 64 * 4 : 0;
  static constexpr int kFixed = 1024 /*align slack*/ + 256 /*barriers*/;
  static constexpr int kStagesFit = (kSmemBudget - kStaging - kFixed) / kStage;
  static constexpr int kStages = kStagesFit > 4 ? 4 : kStagesFit;
  static_assert(kStages >= 2, "pipeline needs two stages");
  static constexpr int kSmem = kFixed + kStages * kStage + kStaging;
  static constexpr uint32_t kTmemCols = NT < 32 ? 32 : NT;
  static constexpr uint32_t kIdesc = instr_desc_f16(MODE == kModeSplit ? 1u : 0u, NT);
};

__device__ __forceinline__ const float* slot_in(const StateRef& st, int s, int off) {
  if (!st.pool_in) return nullptr;
  const int code = st.slot_codes ? st.slot_codes[s] : ((s << 2) | st.uniform_code);
  if (code & 2) return nullptr;  // fresh stream: zero history
  const int slot = code >> 2, parity = code & 1;
  return st.pool_in + ((size_t)parity * st.num_slots + slot) * kSlotFloats + off;
}
__device__ __forceinline__ float* slot_out(const StateRef& st, int s, int off) {
  if (!st.pool_out) return nullptr;
  const int code = st.slot_codes ? st.slot_codes[s] : ((s << 2) | st.uniform_code);
  const int slot = code >> 2, parity = (code & 1) ^ 1;
  return st.pool_out + ((size_t)parity * st.num_slots + slot) * kSlotFloats + off;
}

__device__ __forceinline__ float2 ldg2(const float* p) { return __ldg(reinterpret_cast<const float2*>(p)); }

// Writes two adjacent channels (k, k+1) of tile row r in the A operand.
template <int MODE>
__device__ __forceinline__ void put_a(uint32_t a_stage, int r, int k, float v0, float v1) {
  const uint32_t off = sw128_offset(r, k);
  if (MODE == kModeSplit) {
    uint32_t hi, lo;
    split_bf16(v0, v1, hi, lo);
    st_shared_u32(a_stage + off, hi);
    st_shared_u32(a_stage + kTileM * 128 + off, lo);
  } else {
    st_shared_u32(a_stage + off, pack_f16(v0, v1));
  }
}

// ------------------------------------------------------------------ producers
// Stem: depthwise causal conv k=7 (d=1) on latents [S][64][T]; history = last
// six raw latent frames [6][64].
template <int MODE>
__device__ void produce_stem(const LayerArgs& a, int m0, uint32_t a_stage, int warp, int lane, bool write_state) {
  const int c = 2 * lane;
  const int T = a.rows_per_stream;
  float w0[7], w1[7];
#pragma unroll
  for (int j = 0; j < 7; ++j) {
    w0[j] = __ldg(a.dw_w + c * 7 + j);
    w1[j] = __ldg(a.dw_w + (c + 1) * 7 + j);
  }
  const float b0 = __ldg(a.dw_b + c), b1 = __ldg(a.dw_b + c + 1);
  for (int r = warp; r < kTileM; r += 8) {
    const int g = m0 + r;
    float y0 = 0.f, y1 = 0.f;
    if (g < a.rows) {
      const int s = g / T, t = g - s * T;
      const float* z0 = a.x + ((size_t)s * kLatentChannels + c) * a.z_stride + a.z_offset;
      const float* z1 = z0 + a.z_stride;
      const float* hist = slot_in(a.state, s, a.state_off);
      float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
      for (int j = 0; j < 7; ++j) {
        const int tp = t - 6 + j;
        float v0, v1;
        if (tp >= 0) {
          v0 = __ldg(z0 + tp);
          v1 = __ldg(z1 + tp);
        } else if (hist) {
          const float2 h = ldg2(hist + (6 + tp) * kLatentChannels + c);
          v0 = h.x;
          v1 = h.y;
        } else {
          v0 = v1 = 0.f;
        }
        acc0 = j == 0 ? w0[0] * v0 : fmaf(w0[j], v0, acc0);
        acc1 = j == 0 ? w1[0] * v1 : fmaf(w1[j], v1, acc1);
      }
      y0 = acc0 + b0;
      y1 = acc1 + b1;
      if (write_state && t == T - 1) {
        float* dst = slot_out(a.state, s, a.state_off);
        if (dst) {
          for (int q = 0; q < 6; ++q) {
            const int tp = T - 6 + q;
            float v0, v1;
            if (tp >= 0) {
              v0 = __ldg(z0 + tp);
              v1 = __ldg(z1 + tp);
            } else if (hist) {
              const float2 h = ldg2(hist + (6 + tp) * kLatentChannels + c);
              v0 = h.x;
              v1 = h.y;
            } else {
              v0 = v1 = 0.f;
            }
            *reinterpret_cast<float2*>(dst + q * kLatentChannels + c) = make_float2(v0, v1);
          }
        }
      }
    }
    put_a<MODE>(a_stage, r, c, y0, y1);
  }
}

// Transposed conv, virtual K block kb: tap 0 reads x[t], tap 1 reads x[t-1];
// both through affine (x*scale, +offset) and Snake. History = previous
// activated input [1][C_in].
template <int MODE>
__device__ void produce_tconv(const LayerArgs& a, int m0, int kb, uint32_t a_stage, int warp, int lane,
                              bool write_state) {
  const int C = a.k_channels;
  const int kpt = C / kKBlock;
  const int tap = kb / kpt;
  const int c = (kb - tap * kpt) * kKBlock + 2 * lane;
  const int N = a.rows_per_stream;
  const float sc0 = __ldg(a.scale + c), sc1 = __ldg(a.scale + c + 1);
  const float of0 = __ldg(a.offset + c), of1 = __ldg(a.offset + c + 1);
  const float al0 = __ldg(a.alpha1 + c), al1 = __ldg(a.alpha1 + c + 1);
  const float rc0 = __ldg(a.recip1 + c), rc1 = __ldg(a.recip1 + c + 1);
  for (int r = warp; r < kTileM; r += 8) {
    const int g = m0 + r;
    float y0 = 0.f, y1 = 0.f;
    if (g < a.rows) {
      const int s = g / N, t = g - s * N;
      if (t - tap >= 0) {
        const float2 v = ldg2(a.x + (size_t)(g - tap) * C + c);
        const float u0 = __fadd_rn(__fmul_rn(v.x, sc0), of0);
        const float u1 = __fadd_rn(__fmul_rn(v.y, sc1), of1);
        y0 = snake(u0, al0, rc0);
        y1 = snake(u1, al1, rc1);
        if (write_state && tap == 0 && t == N - 1) {
          float* dst = slot_out(a.state, s, a.state_off);
          if (dst) *reinterpret_cast<float2*>(dst + c) = make_float2(y0, y1);
        }
      } else {
        const float* hist = slot_in(a.state, s, a.state_off);
        if (hist) {
          const float2 h = ldg2(hist + c);
          y0 = h.x;
          y1 = h.y;
        }
      }
    }
    put_a<MODE>(a_stage, r, c & (kKBlock - 1), y0, y1);
  }
}

// Residual unit, K block kb: Snake -> depthwise causal k=7 (dilation d) ->
// Snake. Phase 1 stages Snake(x) for the tile's rows and its 6d-row halo in
// shared memory (fp32); phase 2 walks each channel pair down rows of equal
// residue mod d so the seven taps slide through registers. History = last 6d
// Snake(x) rows [6d][C] (the depthwise conv's activated input).
template <int MODE>
__device__ void produce_residual(const LayerArgs& a, int m0, int kb, uint32_t a_stage, float* staging, int warp,
                                 int lane, bool write_state) {
  const int C = a.k_channels;
  const int d = a.dilation;
  const int H = 6 * d;
  const int N = a.rows_per_stream;
  const int kl = 2 * lane;                  // channel pair inside the K block
  const int c = kb * kKBlock + kl;
  const bool valid = kl < (C < kKBlock ? C : kKBlock);
  float a10 = 0.f, a11 = 0.f, r10 = 0.f, r11 = 0.f, a20 = 0.f, a21 = 0.f, r20 = 0.f, r21 = 0.f;
  float w0[7], w1[7], b0 = 0.f, b1 = 0.f;
#pragma unroll
  for (int j = 0; j < 7; ++j) w0[j] = w1[j] = 0.f;
  if (valid) {
    a10 = __ldg(a.alpha1 + c); a11 = __ldg(a.alpha1 + c + 1);
    r10 = __ldg(a.recip1 + c); r11 = __ldg(a.recip1 + c + 1);
    a20 = __ldg(a.alpha2 + c); a21 = __ldg(a.alpha2 + c + 1);
    r20 = __ldg(a.recip2 + c); r21 = __ldg(a.recip2 + c + 1);
#pragma unroll
    for (int j = 0; j < 7; ++j) {
      w0[j] = __ldg(a.dw_w + c * 7 + j);
      w1[j] = __ldg(a.dw_w + (c + 1) * 7 + j);
    }
    b0 = __ldg(a.dw_b + c);
    b1 = __ldg(a.dw_b + c + 1);
  }
  // Phase 1: staging[i] = Snake(x[m0 - H + i]) for i in [0, 128 + H).
  for (int i = warp; i < kTileM + H; i += 8) {
    const int g = m0 - H + i;
    float2 v = make_float2(0.f, 0.f);
    if (valid && g >= 0 && g < a.rows) {
      v = ldg2(a.x + (size_t)g * C + c);
      v.x = snake(v.x, a10, r10);
      v.y = snake(v.y, a11, r11);
    }
    *reinterpret_cast<float2*>(staging + i * 64 + kl) = v;
  }
  named_barrier(1, kProducerThreads);
  // Advanced history for streams whose last row lies in this tile.
  if (write_state && valid) {
    const int g_end = min(m0 + kTileM, a.rows);
    const int s_lo = m0 / N, s_hi = (g_end - 1) / N;
    for (int s = s_lo + warp; s <= s_hi; s += 8) {
      const int last = s * N + N - 1;
      if (last < m0 || last >= g_end) continue;
      float* dst = slot_out(a.state, s, a.state_off);
      if (!dst) continue;
      const float* hist = slot_in(a.state, s, a.state_off);
      for (int q = 0; q < H; ++q) {
        const int tp = N - H + q;
        float2 v;
        if (tp >= 0) {
          v = *reinterpret_cast<const float2*>(staging + (s * N + tp - m0 + H) * 64 + kl);
        } else {
          v = hist ? ldg2(hist + (N + q) * C + c) : make_float2(0.f, 0.f);
        }
        *reinterpret_cast<float2*>(dst + q * C + c) = v;
      }
    }
  }
  // Phase 2: 16 rows per warp in residue-class order.
  int rho = 0, k = 16 * warp;
  while (true) {
    const int n_rho = (kTileM - rho + d - 1) / d;
    if (k < n_rho) break;
    k -= n_rho;
    ++rho;
  }
  float2 win[7];
#pragma unroll
  for (int j = 0; j < 7; ++j) win[j] = make_float2(0.f, 0.f);
  int prev_r = -1000000, prev_s = -1;
  for (int it = 0; it < 16; ++it) {
    const int r = rho + k * d;
    const int g = m0 + r;
    float y0 = 0.f, y1 = 0.f;
    if (g < a.rows && valid) {
      const int s = g / N, t = g - s * N;
      if (prev_r == r - d && prev_s == s) {
#pragma unroll
        for (int j = 0; j < 6; ++j) win[j] = win[j + 1];
      } else {
        const float* hist = slot_in(a.state, s, a.state_off);
#pragma unroll
        for (int j = 0; j < 6; ++j) {
          const int back = (6 - j) * d;
          const int tp = t - back;
          if (tp >= 0) {
            win[j] = *reinterpret_cast<const float2*>(staging + (r - back + H) * 64 + kl);
          } else {
            win[j] = hist ? ldg2(hist + (H + tp) * C + c) : make_float2(0.f, 0.f);
          }
        }
      }
      win[6] = *reinterpret_cast<const float2*>(staging + (r + H) * 64 + kl);
      float h0 = w0[0] * win[0].x, h1 = w1[0] * win[0].y;
#pragma unroll
      for (int j = 1; j < 7; ++j) {
        h0 = fmaf(w0[j], win[j].x, h0);
        h1 = fmaf(w1[j], win[j].y, h1);
      }
      h0 += b0;
      h1 += b1;
      y0 = snake(h0, a20, r20);
      y1 = snake(h1, a21, r21);
      prev_r = r;
      prev_s = s;
    }
    put_a<MODE>(a_stage, r, kl, y0, y1);
    if (++k >= (kTileM - rho + d - 1) / d) {
      ++rho;
      k = 0;
    }
  }
  named_barrier(1, kProducerThreads);  // staging reused by the next K block
}

// Plain GEMM operand for the engine self-test: A [rows][K] fp32 row-major.
template <int MODE>
__device__ void produce_test(const LayerArgs& a, int m0, int kb, uint32_t a_stage, int warp, int lane) {
  const int c = kb * kKBlock + 2 * lane;
  for (int r = warp; r < kTileM; r += 8) {
    const int g = m0 + r;
    float2 v = make_float2(0.f, 0.f);
    if (g < a.rows && c < a.k_channels) v = ldg2(a.x + (size_t)g * a.k_channels + c);
    put_a<MODE>(a_stage, r, 2 * lane, v.x, v.y);
  }
}

// ------------------------------------------------------------------ epilogues
template <int KIND>
__device__ __forceinline__ void epilogue_chunk(const LayerArgs& a, int g, int n, const float (&v)[16]) {
  if (KIND == kTconv) {
    const int p = n / a.c_out, o = n - p * a.c_out;
    float* dst = a.out + ((size_t)g * a.stride + p) * a.c_out + o;
#pragma unroll
    for (int i = 0; i < 16; i += 4) {
      const float4 b = __ldg(reinterpret_cast<const float4*>(a.bias + o + i));
      *reinterpret_cast<float4*>(dst + i) = make_float4(v[i] + b.x, v[i + 1] + b.y, v[i + 2] + b.z, v[i + 3] + b.w);
    }
  } else if (KIND == kResidual) {
    const size_t base = (size_t)g * a.c_out + n;
#pragma unroll
    for (int i = 0; i < 16; i += 4) {
      const float4 b = __ldg(reinterpret_cast<const float4*>(a.bias + n + i));
      const float4 x = __ldg(reinterpret_cast<const float4*>(a.x + base + i));
      *reinterpret_cast<float4*>(a.out + base + i) =
          make_float4(x.x + (v[i] + b.x), x.y + (v[i + 1] + b.y), x.z + (v[i + 2] + b.z), x.w + (v[i + 3] + b.w));
    }
  } else {
    const size_t base = (size_t)g * a.n_total + n;
#pragma unroll
    for (int i = 0; i < 16; i += 4) {
      float4 b = make_float4(0.f, 0.f, 0.f, 0.f);
      if (a.bias) b = __ldg(reinterpret_cast<const float4*>(a.bias + n + i));
      *reinterpret_cast<float4*>(a.out + base + i) = make_float4(v[i] + b.x, v[i + 1] + b.y, v[i + 2] + b.z, v[i + 3] + b.w);
    }
  }
}

// --------------------------------------------------------------------- engine
template <int NT, int MODE, int KIND>
__global__ void __launch_bounds__(kThreads, 1) gemm_layer_kernel(const LayerArgs a) {
  using Cfg = GemmCfg<NT, MODE, KIND>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_base = smem;
  uint8_t* b_base = a_base + S * Cfg::kAStage;
  float* staging = reinterpret_cast<float*>(b_base + S * Cfg::kBStage);
  uint64_t* bars = reinterpret_cast<uint64_t*>(b_base + S * Cfg::kBStage + Cfg::kStaging);
  uint64_t* a_full = bars;
  uint64_t* b_full = bars + S;
  uint64_t* empty = bars + 2 * S;
  uint64_t* acc_full = bars + 3 * S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * S + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kTileM;
  const int n_tile = blockIdx.y;
  const int num_kb = a.num_kblocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&a_full[s], 8);
      mbar_init(&b_full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 8) {
    // ---- A producers
    bool ok = true;
    const bool write_state = n_tile == 0;
    for (int kb = 0; kb < num_kb && ok; ++kb) {
      const int s = kb % S;
      const uint32_t ph = (kb / S) & 1;
      // All producer threads leave together on a timeout, so none is left
      // waiting at a named barrier inside a producer.
      ok = named_barrier_and(2, kProducerThreads, mbar_wait(&empty[s], ph ^ 1, a.status, kDevTimeoutProducer));
      if (!ok) break;
      const uint32_t a_stage = smem_u32(a_base + s * Cfg::kAStage);
      if (KIND == kStem) produce_stem<MODE>(a, m0, a_stage, warp, lane, write_state);
      else if (KIND == kTconv) produce_tconv<MODE>(a, m0, kb, a_stage, warp, lane, write_state);
      else if (KIND == kResidual) produce_residual<MODE>(a, m0, kb, a_stage, staging, warp, lane, write_state);
      else produce_test<MODE>(a, m0, kb, a_stage, warp, lane);
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&a_full[s]);
    }
    // ---- epilogue
    if (ok && mbar_wait(acc_full, 0, a.status, kDevTimeoutEpilogue)) {
      tc_fence_after();
      const int q = warp & 3, half = warp >> 2;
      const int r = q * 32 + lane;
      const int g = m0 + r;
      constexpr int kHalfCols = NT / 2;
      for (int col = half * kHalfCols; col < (half + 1) * kHalfCols; col += 16) {
        float v[16];
        tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)col, v);
        if (g < a.rows) epilogue_chunk<KIND>(a, g, n_tile * NT + col, v);
      }
    }
  } else if (warp == 8) {
    // ---- weight loader
    if (lane == 0) {
      const uint8_t* src = a.wimg + (size_t)n_tile * num_kb * Cfg::kBStage;
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % S;
        const uint32_t ph = (kb / S) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, a.status, kDevTimeoutLoader)) break;
        mbar_arrive_expect_tx(&b_full[s], Cfg::kBStage);
        bulk_g2s(b_base + s * Cfg::kBStage, src + (size_t)kb * Cfg::kBStage, Cfg::kBStage, &b_full[s]);
      }
    }
  } else {
    // ---- MMA issuer
    if (lane == 0) {
      bool ok = true;
      for (int kb = 0; kb < num_kb; ++kb) {
        const int s = kb % S;
        const uint32_t ph = (kb / S) & 1;
        ok = mbar_wait(&a_full[s], ph, a.status, kDevTimeoutMma) &&
             mbar_wait(&b_full[s], ph, a.status, kDevTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(a_base + s * Cfg::kAStage);
        const uint32_t b0 = smem_u32(b_base + s * Cfg::kBStage);
#pragma unroll
        for (int k = 0; k < kKBlock / 16; ++k) {
          const uint32_t ko = k * 32;
          const uint32_t acc = (kb | k) ? 1u : 0u;
          mma_f16(tmem, smem_desc_sw128(a0 + ko), smem_desc_sw128(b0 + ko), Cfg::kIdesc, acc);
          if (MODE == kModeSplit) {
            mma_f16(tmem, smem_desc_sw128(a0 + ko), smem_desc_sw128(b0 + Cfg::kBTile + ko), Cfg::kIdesc, 1u);
            mma_f16(tmem, smem_desc_sw128(a0 + Cfg::kATile + ko), smem_desc_sw128(b0 + ko), Cfg::kIdesc, 1u);
          }
        }
        mma_commit(&empty[s]);
      }
      if (ok) mma_commit(acc_full);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

template <int NT, int MODE, int KIND>
static cudaError_t launch_cfg(const LayerArgs& a, cudaStream_t stream) {
  using Cfg = GemmCfg<NT, MODE, KIND>;
  const dim3 grid((a.rows + kTileM - 1) / kTileM, a.n_total / NT);
  gemm_layer_kernel<NT, MODE, KIND><<<grid, kThreads, Cfg::kSmem, stream>>>(a);
  return cudaGetLastError();
}

template <int NT, int MODE, int KIND>
static cudaError_t set_smem() {
  using Cfg = GemmCfg<NT, MODE, KIND>;
  return cudaFuncSetAttribute(gemm_layer_kernel<NT, MODE, KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              Cfg::kSmem);
}

template <int MODE, int KIND>
static cudaError_t set_smem_all() {
  cudaError_t e;
  if ((e = set_smem<256, MODE, KIND>()) != cudaSuccess) return e;
  if ((e = set_smem<128, MODE, KIND>()) != cudaSuccess) return e;
  if ((e = set_smem<64, MODE, KIND>()) != cudaSuccess) return e;
  return set_smem<32, MODE, KIND>();
}

template <int MODE, int KIND>
static cudaError_t launch_nt(const LayerArgs& a, cudaStream_t stream) {
  switch (a.n_tile) {
    case 256: return launch_cfg<256, MODE, KIND>(a, stream);
    case 128: return launch_cfg<128, MODE, KIND>(a, stream);
    case 64: return launch_cfg<64, MODE, KIND>(a, stream);
    case 32: return launch_cfg<32, MODE, KIND>(a, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t prepare_kernels() {
  cudaError_t e;
  if ((e = set_smem_all<kModeSplit, kStem>()) != cudaSuccess) return e;
  if ((e = set_smem_all<kModeSplit, kTconv>()) != cudaSuccess) return e;
  if ((e = set_smem_all<kModeF16, kResidual>()) != cudaSuccess) return e;
  if ((e = set_smem_all<kModeSplit, kTestGemm>()) != cudaSuccess) return e;
  return set_smem_all<kModeF16, kTestGemm>();
}

cudaError_t launch_gemm_layer(const LayerArgs& a, cudaStream_t stream) {
  if (a.rows <= 0) return cudaSuccess;
  if (a.n_total % a.n_tile) return cudaErrorInvalidValue;
  switch (a.kind) {
    case kStem:
      return a.mode == kModeSplit ? launch_nt<kModeSplit, kStem>(a, stream) : cudaErrorInvalidValue;
    case kTconv:
      return a.mode == kModeSplit ? launch_nt<kModeSplit, kTconv>(a, stream) : cudaErrorInvalidValue;
    case kResidual:
      return a.mode == kModeF16 ? launch_nt<kModeF16, kResidual>(a, stream) : cudaErrorInvalidValue;
    case kTestGemm:
      return a.mode == kModeSplit ? launch_nt<kModeSplit, kTestGemm>(a, stream)
                                  : launch_nt<kModeF16, kTestGemm>(a, stream);
    default: return cudaErrorInvalidValue;
  }
}

// ------------------------------------------------------------------ final conv
// Snake(32) -> causal conv 32->1 (k=7) -> tanh on CUDA cores. 256 output rows
// per block; Snake values for the rows and a 6-row halo staged in shared memory.
constexpr int kFinalRows = 256;
constexpr int kFinalPitch = 33;

__global__ void __launch_bounds__(kFinalRows) final_kernel(const FinalArgs a) {
  __shared__ float act[(kFinalRows + 6) * kFinalPitch];
  __shared__ float wsm[kFinalChannels * 7];
  const int g0 = blockIdx.x * kFinalRows;
  const int N = a.rows_per_stream;
  for (int i = threadIdx.x; i < kFinalChannels * 7; i += kFinalRows) wsm[i] = __ldg(a.w + i);
  for (int i = threadIdx.x; i < (kFinalRows + 6) * kFinalChannels; i += kFinalRows) {
    const int row = i / kFinalChannels, ch = i - row * kFinalChannels;
    const int g = g0 - 6 + row;
    float v = 0.f;
    if (g >= 0 && g < a.rows) v = snake(__ldg(a.x + (size_t)g * kFinalChannels + ch), __ldg(a.alpha + ch), __ldg(a.recip + ch));
    act[row * kFinalPitch + ch] = v;
  }
  __syncthreads();
  const int g_end = min(g0 + kFinalRows, a.rows);
  // Advanced history (last six activated rows) of streams ending in this block.
  if (a.state.pool_out) {
    const int s_lo = g0 / N, s_hi = (g_end - 1) / N;
    for (int s = s_lo; s <= s_hi; ++s) {
      const int last = s * N + N - 1;
      if (last < g0 || last >= g_end) continue;
      float* dst = slot_out(a.state, s, a.state_off);
      for (int i = threadIdx.x; i < 6 * kFinalChannels; i += kFinalRows) {
        const int q = i / kFinalChannels, ch = i - q * kFinalChannels;
        dst[q * kFinalChannels + ch] = act[(last - 5 + q - g0 + 6) * kFinalPitch + ch];
      }
    }
  }
  const int g = g0 + threadIdx.x;
  if (g < a.rows) {
    const int s = g / N, t = g - s * N;
    const float* hist = slot_in(a.state, s, a.state_off);
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 7; ++j) {
      const int tp = t - 6 + j;
      const float* row = act + (threadIdx.x + j) * kFinalPitch;
      for (int ch = 0; ch < kFinalChannels; ++ch) {
        float v;
        if (tp >= 0) v = row[ch];
        else v = hist ? __ldg(hist + (6 + tp) * kFinalChannels + ch) : 0.f;
        acc = fmaf(wsm[ch * 7 + j], v, acc);
      }
    }
    a.audio[(size_t)s * a.audio_stride + a.audio_offset + t] = tanhf(acc + __ldg(a.b));
  }
}

cudaError_t launch_final(const FinalArgs& a, cudaStream_t stream) {
  if (a.rows <= 0) return cudaSuccess;
  final_kernel<<<(a.rows + kFinalRows - 1) / kFinalRows, kFinalRows, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace fav
