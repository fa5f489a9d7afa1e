// C ABI of the decoder: plan creation (weight packing), the per-step layer
// schedule and batch decode. Declarations and contracts: include/fast_audiovae_cuda.h.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <functional>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "../../include/fast_audiovae_cuda.h"
#include "fav_internal.h"

static_assert(FAV_SLOT_FLOATS == fav::kSlotFloats, "slot size");
static_assert(FAV_SLOT_STRIDE_FLOATS == fav::kSlotStride, "slot stride");

namespace {

thread_local char g_error[512] = {0};

int32_t fail(int32_t status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
  return status;
}

int32_t cuda_fail(cudaError_t e, const char* what) {
  return fail(FAV_DEVICE_ERROR, "%s: %s", what, cudaGetErrorString(e));
}

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
std::once_flag g_encode_once;
EncodeTiledFn g_encode = nullptr;

bool load_encoder() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  });
  return g_encode != nullptr;
}

// Tiled TMA map over a dense tensor of ``rank`` dimensions (innermost first),
// zero fill outside the tensor.
int32_t encode_map(CUtensorMap* map, CUtensorMapDataType type, int elem_bytes, const void* base, int rank,
                   const cuuint64_t* dims, const cuuint32_t* box, CUtensorMapSwizzle swizzle, const char* what) {
  if (!load_encoder()) return fail(FAV_DEVICE_ERROR, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t strides[4];
  cuuint64_t pitch = (cuuint64_t)elem_bytes;
  for (int i = 0; i + 1 < rank; ++i) strides[i] = pitch *= dims[i];
  const cuuint32_t elem[5] = {1, 1, 1, 1, 1};
  const CUresult r = g_encode(map, type, rank, const_cast<void*>(base), dims, strides, box, elem,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FAV_DEVICE_ERROR, "cuTensorMapEncodeTiled (%s) failed (%d)", what, (int)r);
  return FAV_OK;
}

// Residual input s [rows][channels] fp32: boxes of min(channels, 64) channels x
// box_rows rows, unswizzled (the producers read it row by row).
int32_t encode_input_map(CUtensorMap* map, const float* x, int rows, int channels, int box_rows) {
  const cuuint64_t dims[2] = {(cuuint64_t)channels, (cuuint64_t)rows};
  const cuuint32_t box[2] = {(cuuint32_t)(channels < fav::kKBlock ? channels : fav::kKBlock), (cuuint32_t)box_rows};
  return encode_map(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, x, 2, dims, box, CU_TENSOR_MAP_SWIZZLE_NONE, "input");
}

// f16 residual input s [rows][channels] (Snake_pre(y) written by the previous
// epilogue with kEpiS16): boxes of 64 channels (128 bytes) x box_rows rows.
int32_t encode_input_map_f16(CUtensorMap* map, const void* s, int rows, int channels, int box_rows) {
  const cuuint64_t dims[2] = {(cuuint64_t)channels, (cuuint64_t)rows};
  const cuuint32_t box[2] = {(cuuint32_t)fav::kKBlock, (cuuint32_t)box_rows};
  return encode_map(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, s, 2, dims, box, CU_TENSOR_MAP_SWIZZLE_NONE, "s16");
}

// Split-bf16 planes [2][rows][channels] (hi, then lo) of a transposed conv's
// activated input, loaded in 64 x 128 x 2 boxes (hi tile, then lo tile) in the
// 128-byte swizzle, which is the MMA's K-major A layout.
int32_t encode_plane_map(CUtensorMap* map, const void* planes, int rows, int channels) {
  const cuuint64_t dims[3] = {(cuuint64_t)channels, (cuuint64_t)rows, 2};
  const cuuint32_t box[3] = {(cuuint32_t)fav::kKBlock, (cuuint32_t)fav::kTileM, 2};
  return encode_map(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, planes, 3, dims, box, CU_TENSOR_MAP_SWIZZLE_128B,
                    "planes");
}

// Preformed residual A operand [rows][channels] f16: boxes of 64 channels x
// 128 rows in the 128-byte swizzle (the MMA's K-major layout).
int32_t encode_operand_map(CUtensorMap* map, const uint16_t* a, int rows, int channels) {
  const cuuint64_t dims[2] = {(cuuint64_t)channels, (cuuint64_t)rows};
  const cuuint32_t box[2] = {(cuuint32_t)fav::kKBlock, (cuuint32_t)fav::kTileM};
  return encode_map(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a, 2, dims, box, CU_TENSOR_MAP_SWIZZLE_128B, "operand");
}

// Preformed int8 transposed-conv tap [rows][channels] s8: boxes of 128
// channels x 128 rows in the 128-byte swizzle.
int32_t encode_s8_map(CUtensorMap* map, const uint8_t* q, int rows, int channels) {
  const cuuint64_t dims[2] = {(cuuint64_t)channels, (cuuint64_t)rows};
  const cuuint32_t box[2] = {(cuuint32_t)fav::kKBlockI8, (cuuint32_t)fav::kTileM};
  return encode_map(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, q, 2, dims, box, CU_TENSOR_MAP_SWIZZLE_128B, "s8 taps");
}

// Stage-5 input y [rows][32] fp32 for the fused tail: boxes of 32 channels x
// box_rows rows in the 128-byte swizzle.
int32_t encode_tail_map(CUtensorMap* map, const float* x, int rows, int box_rows) {
  const cuuint64_t dims[2] = {(cuuint64_t)fav::kTailC, (cuuint64_t)rows};
  const cuuint32_t box[2] = {(cuuint32_t)fav::kTailC, (cuuint32_t)box_rows};
  return encode_map(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, x, 2, dims, box, CU_TENSOR_MAP_SWIZZLE_128B, "tail");
}

// Input y [rows][channels] fp32 of a fused residual stage: boxes of 32
// channels x 128 rows in the 128-byte swizzle.
int32_t encode_stage_map(CUtensorMap* map, const float* x, int rows, int channels) {
  const cuuint64_t dims[2] = {(cuuint64_t)channels, (cuuint64_t)rows};
  const cuuint32_t box[2] = {32, (cuuint32_t)fav::kTileM};
  return encode_map(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, x, 2, dims, box, CU_TENSOR_MAP_SWIZZLE_128B, "stage");
}

// Split-bf16 planes [2][streams][rows_per_stream][channels] written by a fused
// residual stage: store boxes of 64 channels x 128 rows in the 128-byte
// swizzle; rows past a stream's end fall outside the box's tensor and are not
// written.
int32_t encode_stage_planes_map(CUtensorMap* map, const void* planes, int streams, int rows_per_stream, int channels) {
  const cuuint64_t dims[4] = {(cuuint64_t)channels, (cuuint64_t)rows_per_stream, (cuuint64_t)streams, 2};
  const cuuint32_t box[4] = {64, (cuuint32_t)fav::kTileM, 1, 1};
  return encode_map(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, planes, 4, dims, box, CU_TENSOR_MAP_SWIZZLE_128B,
                    "stage planes");
}

std::once_flag g_prepare_once;
cudaError_t g_prepare_error = cudaSuccess;

cudaError_t prepare_once() {
  std::call_once(g_prepare_once, [] { g_prepare_error = fav::prepare_kernels(); });
  return g_prepare_error;
}

// --------------------------------------------------------------- packing
// Weight operand B[n][k] of a layer packed as [n_tile][kblock][term][NT rows][128 B],
// each 64-element row slice in the 128-byte swizzled K-major layout the MMA
// reads (16-byte chunk j of row r stored at chunk j ^ (r % 8)). K is padded with
// zeros to a multiple of 64.
std::vector<uint16_t> pack_operand(int n_total, int k_total, int nt, int mode,
                                   const std::function<float(int, int)>& value) {
  const int kblocks = (k_total + fav::kKBlock - 1) / fav::kKBlock;
  const int terms = mode == fav::kModeSplit ? 2 : 1;
  const int ntiles = n_total / nt;
  std::vector<uint16_t> img((size_t)ntiles * kblocks * terms * nt * 64, 0);
  for (int n = 0; n < n_total; ++n) {
    const int tile = n / nt, row = n % nt;
    for (int k = 0; k < kblocks * fav::kKBlock; ++k) {
      const float v = k < k_total ? value(n, k) : 0.f;
      const int kb = k / fav::kKBlock, kk = k % fav::kKBlock;
      const int chunk = (kk >> 3) ^ (row & 7);
      const size_t within = (size_t)row * 64 + chunk * 8 + (kk & 7);
      const size_t base = ((size_t)tile * kblocks + kb) * terms * nt * 64;
      if (mode == fav::kModeSplit) {
        const __nv_bfloat16 hi = __float2bfloat16_rn(v);
        const __nv_bfloat16 lo = __float2bfloat16_rn(v - __bfloat162float(hi));
        std::memcpy(&img[base + within], &hi, 2);
        std::memcpy(&img[base + (size_t)nt * 64 + within], &lo, 2);
      } else {
        const __half h = __float2half_rn(v);
        std::memcpy(&img[base + within], &h, 2);
      }
    }
  }
  return img;
}

// The reference's int8 weight quantisation (precision.cpp:82-92, ip_create
// :370-376): one scale per matrix row, scale = max|w| / 127 (1 for a zero row,
// max|w| when the quotient underflows), q = clamp(w / scale, -127, 127)
// rounded half to even.
float quant_scale_host(float mx) {
  if (mx == 0.f) return 1.f;
  const float s = mx / 127.f;
  return s > 0.f ? s : mx;
}
int8_t quant_host(float v, float scale) {
  float q = v / scale;
  q = q < -127.f ? -127.f : (q > 127.f ? 127.f : q);
  return static_cast<int8_t>(std::nearbyint(q));  // default rounding: half to even
}

// int8 weight operand: rows n of ``terms`` matrices value(term, n, k), each row
// quantised with its own scale (scales[term * n_total + n]), packed as
// [n_tile][kblock][term][NT rows][128 B] in the 128-byte swizzle (16-byte chunk
// j of row r at chunk j ^ (r % 8)); K padded with zeros to a multiple of 128.
std::vector<int8_t> pack_operand_i8(int n_total, int k_total, int nt, int terms,
                                    const std::function<float(int, int, int)>& value, std::vector<float>& scales) {
  const int kblocks = (k_total + fav::kKBlockI8 - 1) / fav::kKBlockI8;
  const int ntiles = n_total / nt;
  std::vector<int8_t> img((size_t)ntiles * kblocks * terms * nt * 128, 0);
  scales.assign((size_t)terms * n_total, 1.f);
  std::vector<float> row(k_total);
  for (int term = 0; term < terms; ++term)
    for (int n = 0; n < n_total; ++n) {
      float mx = 0.f;
      for (int k = 0; k < k_total; ++k) {
        row[k] = value(term, n, k);
        mx = std::fmax(mx, std::fabs(row[k]));
      }
      const float sc = quant_scale_host(mx);
      scales[(size_t)term * n_total + n] = sc;
      const int tile = n / nt, r = n % nt;
      for (int k = 0; k < k_total; ++k) {
        const int kb = k / fav::kKBlockI8, kk = k % fav::kKBlockI8;
        const size_t base = (((size_t)tile * kblocks + kb) * terms + term) * nt * 128;
        img[base + (size_t)r * 128 + ((((kk >> 4) ^ (r & 7)) << 4) | (kk & 15))] = quant_host(row[k], sc);
      }
    }
  return img;
}

struct DeviceArrays {
  std::vector<void*> owned;
  size_t bytes = 0;
  ~DeviceArrays() {
    for (void* p : owned) cudaFree(p);
  }
  template <class T>
  T* upload(const T* host, size_t count, cudaError_t* err) {
    void* p = nullptr;
    *err = cudaMalloc(&p, count * sizeof(T));
    if (*err != cudaSuccess) return nullptr;
    owned.push_back(p);
    bytes += count * sizeof(T);
    *err = cudaMemcpy(p, host, count * sizeof(T), cudaMemcpyHostToDevice);
    return static_cast<T*>(p);
  }
};

struct StageDev {
  int c_in, c_out, rate, n_tile_t;
  const float *scale, *offset, *alpha, *recip, *tbias;
  const uint8_t* timg;
  int state_t;
  bool int8 = false;                    // int8 plan and a selected transposed conv (W8A8)
  const float *tsw = nullptr;           // int8: row scales [2][n_total] (current tap, previous tap)
  struct Res {
    int dilation, n_tile;
    const float *pre_a, *pre_r, *pw_b, *coef;
    const uint8_t* img;
    int state_off;
    bool int8 = false;                  // int8 plan and a selected residual 1x1 (W8A8)
    const float* sw = nullptr;          // int8: row scales [C]
  } res[3];
};

}  // namespace

struct fav_plan {
  int device = 0;
  DeviceArrays mem;
  const float *stem_w = nullptr, *stem_b = nullptr, *pw_b = nullptr;
  const uint8_t* stem_img = nullptr;    // stem 1x1 weights for 256-column N tiles
  const uint8_t* stem_img64 = nullptr;  // the same for 64-column N tiles (steps of few rows)
  const float* stem_pw = nullptr;  // int8 plan: fp32 stem 1x1 weights [2048][64] for the CUDA-core stem
  StageDev stages[fav::kStages];
  const float *fin_a = nullptr, *fin_r = nullptr, *fin_w = nullptr, *fin_b = nullptr;
  int state_final = 0;
  int precision = FAV_PRECISION_BF16;
};

namespace {

size_t expected_count(int index) {
  if (index == 0) return 64 * 7;
  if (index == 1) return 64;
  if (index == 2) return 2048 * 64;
  if (index == 3) return 2048;
  if (index >= 184) {
    const size_t tail[4] = {32, 32, 32 * 7, 1};
    return tail[index - 184];
  }
  const int i = (index - 4) / 30, o = (index - 4) % 30;
  const size_t cin = 2048 >> i, cout = cin / 2, s = fav::kRates[i];
  if (o < 4) return cin;
  if (o == 4) return cin * cout * 2 * s;
  if (o == 5) return cout;
  const int r = (o - 6) % 8;
  const size_t sizes[8] = {cout, cout, cout * 7, cout, cout, cout, cout * cout, cout};
  return sizes[r];
}

// The int8 recipe's selection (tools/rewrite.py:19-30): matrices with
// min(rows, cols) >= 128. Transposed conv of stage i: rows C_out * rate per tap,
// cols C_in; residual 1x1: C x C.
bool int8_transpose(int i) {
  const int cin = 2048 >> i, cout = cin / 2;
  return std::min(cout * fav::kRates[i], cin) >= 128;
}
bool int8_residual(int i) { return (1024 >> i) >= 128; }

int32_t build_plan(fav_plan* plan, const float* const* w) {
  const bool i8 = plan->precision == FAV_PRECISION_INT8;
  cudaError_t e = cudaSuccess;
  auto up = [&](int index) -> const float* {
    return plan->mem.upload(w[index], expected_count(index), &e);
  };
  auto up_img = [&](const std::vector<uint16_t>& img) -> const uint8_t* {
    return reinterpret_cast<const uint8_t*>(plan->mem.upload(img.data(), img.size(), &e));
  };
  // Stem: depthwise coefficients + 1x1 64->2048 (split bf16).
  plan->stem_w = up(0);
  plan->stem_b = up(1);
  {
    const float* pw = w[2];
    plan->stem_img = up_img(pack_operand(2048, 64, 256, fav::kModeSplit,
                                         [pw](int n, int k) { return pw[(size_t)n * 64 + k]; }));
    plan->stem_img64 = up_img(pack_operand(2048, 64, 64, fav::kModeSplit,
                                           [pw](int n, int k) { return pw[(size_t)n * 64 + k]; }));
  }
  plan->pw_b = up(3);
  if (i8) plan->stem_pw = up(2);
  if (e != cudaSuccess) return cuda_fail(e, "plan upload");
  int off = 6 * fav::kLatentChannels;
  for (int i = 0; i < fav::kStages; ++i) {
    StageDev& st = plan->stages[i];
    const int base = 4 + 30 * i;
    st.c_in = 2048 >> i;
    st.c_out = st.c_in / 2;
    st.rate = fav::kRates[i];
    const int n_total = st.c_out * st.rate;
    // Wide layers (N >= 1024, stages 0-2) take N tiles of 256 columns (two
    // 256-column accumulators fill TMEM), halving the A operand's re-reads;
    // measured slower at stage 3 (N = 256, one tile), which keeps 128.
    st.n_tile_t = n_total % 256 == 0 && n_total >= 1024 ? 256 : n_total % 128 == 0 ? 128 : n_total;
    st.scale = up(base + 0);
    st.offset = up(base + 1);
    st.alpha = up(base + 2);
    st.recip = up(base + 3);
    {
      const float* tw = w[base + 4];
      const int cin = st.c_in, cout = st.c_out, s = st.rate;
      st.int8 = i8 && int8_transpose(i);
      if (st.int8) {
        // Two matrices (current tap p, previous tap p + s), each [C_out * s][C_in], row
        // n = phase * C_out + o, quantised per row like the reference's split projections
        // (graph/upsampling.py:122-127).
        std::vector<float> scales;
        auto img = pack_operand_i8(n_total, cin, 128, 2, [=](int term, int n, int k) {
          const int p = n / cout, o = n % cout;
          return tw[((size_t)k * cout + o) * 2 * s + p + term * s];
        }, scales);
        st.n_tile_t = 128;
        st.timg = reinterpret_cast<const uint8_t*>(plan->mem.upload(img.data(), img.size(), &e));
        st.tsw = plan->mem.upload(scales.data(), scales.size(), &e);
      } else {
        // n = phase * C_out + o; k < C_in: current tap W[k][o][p], else previous tap W[k-C_in][o][p+s].
        st.timg = up_img(pack_operand(n_total, 2 * cin, st.n_tile_t, fav::kModeSplit, [=](int n, int k) {
          const int p = n / cout, o = n % cout;
          const int i_ch = k < cin ? k : k - cin;
          const int tap = k < cin ? p : p + s;
          return tw[((size_t)i_ch * cout + o) * 2 * s + tap];
        }));
      }
    }
    st.tbias = up(base + 5);
    st.state_t = off;
    off += st.c_in;
    for (int j = 0; j < 3; ++j) {
      const int rb = base + 6 + 8 * j;
      auto& r = st.res[j];
      r.dilation = fav::kDilations[j];
      r.n_tile = st.c_out < 256 ? st.c_out : 256;
      r.pre_a = up(rb + 0);
      r.pre_r = up(rb + 1);
      const float* pw = w[rb + 6];
      const int c = st.c_out;
      r.int8 = i8 && int8_residual(i);
      if (r.int8) {
        std::vector<float> scales;
        auto img = pack_operand_i8(c, c, r.n_tile, 1, [pw, c](int, int n, int k) { return pw[(size_t)n * c + k]; },
                                   scales);
        r.img = reinterpret_cast<const uint8_t*>(plan->mem.upload(img.data(), img.size(), &e));
        r.sw = plan->mem.upload(scales.data(), scales.size(), &e);
      } else {
        r.img = up_img(pack_operand(c, c, r.n_tile, fav::kModeF16,
                                    [pw, c](int n, int k) { return pw[(size_t)n * c + k]; }));
      }
      r.pw_b = up(rb + 7);
      {
        // [block][w0..w6, bias, alpha2, recip2][64], zero padded past C (the
        // first Snake is applied by the previous layer's epilogue).
        const int c = st.c_out, blocks = (c + 63) / 64;
        std::vector<float> cf((size_t)blocks * fav::kCoefResidual * 64, 0.f);
        for (int b = 0; b < blocks; ++b)
          for (int ch = 0; ch < 64 && b * 64 + ch < c; ++ch) {
            const int cc = b * 64 + ch;
            float* o = &cf[(size_t)b * fav::kCoefResidual * 64 + ch];
            for (int j = 0; j < 7; ++j) o[j * 64] = w[rb + 2][(size_t)cc * 7 + j];
            o[7 * 64] = w[rb + 3][cc];
            o[8 * 64] = w[rb + 4][cc];
            o[9 * 64] = w[rb + 5][cc];
          }
        r.coef = plan->mem.upload(cf.data(), cf.size(), &e);
      }
      r.state_off = off;
      off += 6 * r.dilation * st.c_out;
    }
    if (e != cudaSuccess) return cuda_fail(e, "plan upload");
  }
  plan->fin_a = up(184);
  plan->fin_r = up(185);
  plan->fin_w = up(186);
  plan->fin_b = up(187);
  plan->state_final = off;
  off += 6 * fav::kFinalChannels;
  if (e != cudaSuccess) return cuda_fail(e, "plan upload");
  if (off != fav::kSlotFloats) return fail(FAV_INVALID_ARGUMENT, "internal state layout mismatch (%d)", off);
  return FAV_OK;
}

// Workspace regions of one step, each n_streams * frames * 61440 floats (the
// largest activation, [rows][channels], of any layer): y and Snake(y) of the
// residual chain in ping-pong pairs, and the split-bf16 planes a transposed
// conv reads for its two taps (rows as they are, and one time step later).
constexpr int kWorkspaceRegions = 6;
constexpr size_t kRegionFloatsPerFrame = 61440;

// Diagnostic settings for one engine launch of a step (fav_debug_step_gated);
// a residual unit of a fused stage gates the stage's kernel.
struct StepDiag {
  int layer;                // 0 = stem, 1 + 4i = stage i transposed conv, 2 + 4i + j = residual unit
  uint32_t wait_limit;      // polls before a wait of that launch gives up
  const uint32_t* gate;     // device flag its MMA issuer waits for first
};

// Launches the kernels of one decoder step. Layers are numbered 0 (stem),
// 1 + 4i (stage i transposed conv), 2 + 4i + j (stage i residual j) and 25
// (final conv); the schedule stops after ``last_layer`` and reports the buffer
// holding that layer's output y (a layer whose y nothing reads writes it only then).
int32_t run_step(const fav_plan* p, const fav::StateRef& state, int n_streams, int frames, const float* z,
                 int z_stride, int z_offset, float* audio, int audio_stride, int audio_offset, float* ws,
                 uint32_t* status, cudaStream_t stream, int last_layer = 25, float** last_out = nullptr,
                 cudaEvent_t* events = nullptr, bool fuse = true, const StepDiag* diag = nullptr) {
  // events (optional, 27): recorded before the stem and after each layer.
  auto mark = [&](int i) {
    if (events) cudaEventRecord(events[i], stream);
  };
  auto diagnose = [&](fav::LayerArgs& l, int index) {
    if (diag && diag->layer == index) {
      l.wait_limit = diag->wait_limit;
      l.gate = diag->gate;
    }
  };
  mark(0);
  const size_t region = (size_t)n_streams * frames * kRegionFloatsPerFrame;
  float* X[2] = {ws, ws + region};
  float* S[2] = {ws + 2 * region, ws + 3 * region};
  uint16_t* planes = reinterpret_cast<uint16_t*>(ws + 4 * region);       // [2][rows][C] bf16
  uint16_t* planes_prev = reinterpret_cast<uint16_t*>(ws + 5 * region);  // row t holds time step t - 1
  // A whole step runs stage 5's residual units and the final conv as one fused
  // kernel; a step stopped inside stage 5 (layer checks) runs them one by one.
  bool tail = fuse && last_layer >= 25 && p->stages[fav::kStages - 1].c_out == fav::kTailC;
  for (int j = 0; j < 3; ++j) tail = tail && !p->stages[fav::kStages - 1].res[j].int8;
  // Stages 2-4 (256, 128 and 64 channels, bf16 units feeding a bf16
  // transposed conv) run their three residual units and the next conv's
  // planes as one fused kernel, unless the step stops inside the stage or at
  // its last unit.
  auto fused_stage = [&](int i) {
    if (!fuse || i + 1 >= fav::kStages || last_layer <= 4 * i + 4) return false;
    const StageDev& st = p->stages[i];
    if (st.c_out != 64 && st.c_out != 128 && st.c_out != 256) return false;
    if (st.c_out == 256) {
      // Stage 2's fused kernel walks a stream's tiles one after another (a
      // one-frame stream has two, the second after a warm-up tile); with
      // fewer tiles than SMs (a step of few streams, latency-bound) the
      // per-layer kernels, which run every tile at once, finish sooner.
      int rows = frames;
      for (int k = 0; k <= i; ++k) rows *= fav::kRates[k];
      if ((long long)n_streams * ((rows + fav::kTileM - 1) / fav::kTileM) < fav::stage_sm_count()) return false;
    }
    for (int j = 0; j < 3; ++j)
      if (st.res[j].int8) return false;
    return !p->stages[i + 1].int8;
  };
  auto tconv_hist = [p](int i) {
    const StageDev& st = p->stages[i];
    return fav::HistRef{1 + 4 * i, 2 * st.state_t, 1, st.c_in};
  };
  // int8 plans: the activated input of an int8 transposed conv (fp32) takes
  // the planes' region, its per-row partial maxima the shifted planes' region
  // (followed there by the int8 residual units' s8 operand and row scales).
  float* act = reinterpret_cast<float*>(planes);
  float* rowmax = reinterpret_cast<float*>(planes_prev);
  int act_parts = 0;  // partial row maxima per row of the activation feeding the next int8 conv
  // Sets the epilogue of a layer whose output feeds stage ``i``'s transposed
  // conv: split-bf16 planes, or (int8 conv) the fp32 activation and row maxima.
  auto feed_tconv = [&](fav::LayerArgs& l, int i, bool debug_y) {
    const StageDev& nx = p->stages[i];
    l.next_scale = nx.scale;
    l.next_offset = nx.offset;
    l.next_alpha = nx.alpha;
    l.next_recip = nx.recip;
    l.hist_next = tconv_hist(i);
    if (nx.int8) {
      l.epi = fav::kEpiAct | (debug_y ? fav::kEpiX : 0);
      l.out_s = act;
      l.rowmax_out = rowmax;
      l.rowmax_parts = l.n_total / l.n_tile;  // the units recount them once their kind and N tile are set
    } else {
      l.epi = fav::kEpiPlanes | (debug_y ? fav::kEpiX : 0);
      l.out_planes = planes;
      l.out_planes_prev = planes_prev;
    }
  };
  // A bf16 layer whose tiles would occupy few SMs (a step of few rows, e.g.
  // one stream's 40 ms chunk) runs 64-column N tiles read from its wider
  // weight image, so more SMs stream its weights.
  auto narrow = [](fav::LayerArgs& l, int img_nt) {
    const int m_tiles = (l.rows + fav::kTileM - 1) / fav::kTileM;
    l.n_tile = img_nt;
    l.img_nt = img_nt;
    if (l.mode != fav::kModeI8 && img_nt > 64 && l.n_total % 64 == 0 && m_tiles * (l.n_total / img_nt) < 64)
      l.n_tile = 64;
  };
  int32_t es = FAV_OK;
  cudaError_t e = cudaSuccess;
  // stem: depthwise k=7 -> 1x1 64->2048; epilogue writes stage 0's activated planes.
  {
    fav::LayerArgs a{};
    a.state = state;
    a.status = status;
    a.kind = fav::kStem;
    a.mode = fav::kModeSplit4;
    a.rows = n_streams * frames;
    a.rows_per_stream = frames;
    a.k_channels = 64;
    a.num_kblocks = 1;
    a.n_total = 2048;
    // A step of few rows (a server's one-frame chunks, one stream's latency)
    // spreads the stem over 64-column N tiles so more SMs share its epilogue.
    a.n_tile = a.rows <= 1024 ? 64 : 256;
    a.c_out = 2048;
    a.x = z;
    a.z_stride = z_stride;
    a.z_offset = z_offset;
    a.bias = p->pw_b;
    a.dw_w = p->stem_w;
    a.dw_b = p->stem_b;
    a.wimg = a.n_tile == 64 ? p->stem_img64 : p->stem_img;
    a.hist = fav::HistRef{0, 0, 6, fav::kLatentChannels};
    a.out_x = X[0];
    feed_tconv(a, 0, last_layer == 0);
    if (p->precision == FAV_PRECISION_INT8) {
      // The int8 recipe's cascade starts here: the stem runs in the oracle's operation order.
      a.dense_w = p->stem_pw;
      a.rowmax_parts = 1;
      e = fav::launch_stem_exact(a, stream);
    } else {
      diagnose(a, 0);
      e = fav::launch_gemm_layer(a, stream);
    }
    act_parts = a.rowmax_parts;
    if (e != cudaSuccess) return cuda_fail(e, "stem launch");
  }
  int layer = 0;
  mark(1);
  if (last_out) *last_out = X[0];
  if (layer == last_layer) return FAV_OK;
  int n = frames;
  for (int i = 0; i < fav::kStages; ++i) {
    const StageDev& st = p->stages[i];
    fav::LayerArgs t{};
    t.state = state;
    t.status = status;
    t.kind = fav::kTconv;
    t.mode = fav::kModeSplit;
    const bool into_tail = tail && i + 1 == fav::kStages;
    const bool into_stage = fused_stage(i);
    // Stages 2-4 with bf16 residual units (all of them in a bf16 plan, stage 4
    // in an int8 plan): this conv and units 0-1 write the next unit's
    // Snake_pre(y) in f16 (kEpiS16), which the unit's producers stage as is.
    const bool s16 = i >= 2 && i + 1 < fav::kStages && !st.res[0].int8;
    t.epi = fav::kEpiX | ((into_tail || into_stage) ? 0 : s16 ? fav::kEpiS16 : fav::kEpiS);
    t.rows = n_streams * n;
    t.rows_per_stream = n;
    t.k_channels = st.c_in;
    t.num_kblocks = 2 * st.c_in / fav::kKBlock;
    t.n_total = st.c_out * st.rate;
    t.n_tile = st.n_tile_t;
    t.n_major = t.rows > t.n_total;  // A (both taps' planes) outweighs the weights
    t.c_out = st.c_out;
    t.stride = st.rate;
    t.bias = st.tbias;
    t.next_alpha = st.res[0].pre_a;
    t.next_recip = st.res[0].pre_r;
    t.wimg = st.timg;
    t.hist = fav::HistRef{1 + 4 * i, 2 * st.state_t, 1, st.c_in};
    t.out_x = X[0];
    t.out_s = S[0];
    if (st.int8) {
      // W8A8: s8 taps of the fp32 activation, per-row scales from the row maxima, one accumulator per tap.
      t.mode = fav::kModeI8;
      t.num_kblocks = st.c_in / fav::kKBlockI8;
      t.rowmax_in = rowmax;
      t.rowmax_in_parts = act_parts;
      t.w_scale = st.tsw;
      t.w_scale2 = st.tsw + t.n_total;
      t.hist_max_slot = fav::kNumHistories + i;
    }
    narrow(t, t.n_tile);
    if (st.int8 && t.n_total / t.n_tile < 2) {
      // One N tile (stage 4): the producers quantise staged fp32 rows.
      if ((es = encode_input_map(&t.tmap, act, t.rows, st.c_in, fav::kTileM + 1)) != FAV_OK) return es;
    } else if (st.int8) {
      // Several N tiles (stages 0-3) would each quantise the same rows: quantise
      // each input row once into both s8 taps (in S[1], unused while the conv
      // runs: 2 * rows * C bytes fit the region); the engine TMA-loads them.
      uint8_t* q0 = reinterpret_cast<uint8_t*>(S[1]);
      uint8_t* q1 = q0 + (size_t)t.rows * st.c_in;
      const fav::QuantizeArgs qa{act, rowmax, act_parts, q0, q1, t.rows, n, st.c_in, state, t.hist, t.hist_max_slot};
      if ((e = fav::launch_quantize(qa, stream)) != cudaSuccess) return cuda_fail(e, "quantize launch");
      t.kind = fav::kTconvPre;
      if ((es = encode_s8_map(&t.tmap, q0, t.rows, st.c_in)) != FAV_OK) return es;
      if ((es = encode_s8_map(&t.tmap2, q1, t.rows, st.c_in)) != FAV_OK) return es;
    } else {
      if ((es = encode_plane_map(&t.tmap, planes, t.rows, st.c_in)) != FAV_OK) return es;
      if ((es = encode_plane_map(&t.tmap2, planes_prev, t.rows, st.c_in)) != FAV_OK) return es;
    }
    diagnose(t, layer + 1);
    if ((e = fav::launch_gemm_layer(t, stream)) != cudaSuccess) return cuda_fail(e, "transpose launch");
    n *= st.rate;
    if (last_out) *last_out = X[0];
    mark(++layer + 1);
    if (layer == last_layer) return FAV_OK;
    if (into_tail) {
      fav::TailArgs ta{};
      ta.rows = n_streams * n;
      ta.rows_per_stream = n;
      for (int j = 0; j < 3; ++j) {
        const auto& r = st.res[j];
        ta.unit[j] = fav::TailUnitArgs{r.pre_a, r.pre_r, r.coef, r.pw_b, r.img,
                                       fav::HistRef{2 + 4 * i + j, 2 * r.state_off, 6 * r.dilation, st.c_out}};
      }
      ta.fin_a = p->fin_a;
      ta.fin_r = p->fin_r;
      ta.fin_w = p->fin_w;
      ta.fin_b = p->fin_b;
      ta.fin_hist = fav::HistRef{25, 2 * p->state_final, 6, fav::kFinalChannels};
      ta.audio = audio;
      ta.audio_stride = audio_stride;
      ta.audio_offset = audio_offset;
      ta.state = state;
      ta.status = status;
      if ((es = encode_tail_map(&ta.xmap, X[0], ta.rows, fav::kTailBoxRows)) != FAV_OK) return es;
      if ((e = fav::launch_tail(ta, stream)) != cudaSuccess) return cuda_fail(e, "tail launch");
      // The fused kernel's time counts as stage 5's first residual unit.
      for (int l = 23; l <= 26; ++l) mark(l);
      if (last_out) *last_out = audio;
      return FAV_OK;
    }
    if (into_stage) {
      fav::StageArgs sa{};
      sa.channels = st.c_out;
      sa.rows = n_streams * n;
      sa.rows_per_stream = n;
      for (int j = 0; j < 3; ++j) {
        const auto& r = st.res[j];
        sa.unit[j] = fav::StageUnitArgs{r.pre_a, r.pre_r, r.coef, r.pw_b, r.img,
                                        fav::HistRef{2 + 4 * i + j, 2 * r.state_off, 6 * r.dilation, st.c_out}};
      }
      const StageDev& nx = p->stages[i + 1];
      sa.next_scale = nx.scale;
      sa.next_offset = nx.offset;
      sa.next_alpha = nx.alpha;
      sa.next_recip = nx.recip;
      sa.out_planes = planes;
      sa.out_planes_prev = planes_prev;
      sa.hist_next = tconv_hist(i + 1);
      sa.state = state;
      sa.status = status;
      if (diag && diag->layer >= 4 * i + 2 && diag->layer <= 4 * i + 4) {
        sa.wait_limit = diag->wait_limit;
        sa.gate = diag->gate;
      }
      sa.x = X[0];
      if ((es = encode_stage_map(&sa.xmap, X[0], sa.rows, st.c_out)) != FAV_OK) return es;
      if ((es = encode_stage_planes_map(&sa.planes_map, planes, n_streams, n, st.c_out)) != FAV_OK) return es;
      if ((es = encode_stage_planes_map(&sa.prev_map, planes_prev, n_streams, n, st.c_out)) != FAV_OK) return es;
      if ((e = fav::launch_stage(sa, stream)) != cudaSuccess) return cuda_fail(e, "stage launch");
      // The fused kernel's time counts as the stage's first residual unit.
      for (int j = 0; j < 3; ++j) mark(++layer + 1);
      continue;
    }
    // Residual unit j reads y and Snake_pre(y) from pair j % 2 and writes pair
    // (j + 1) % 2; the last unit writes the next stage's planes instead (stage 5:
    // Snake_final(y) for the final conv).
    for (int j = 0; j < 3; ++j) {
      const auto& r = st.res[j];
      const int in = j & 1, out = in ^ 1;
      fav::LayerArgs u{};
      u.state = state;
      u.status = status;
      u.kind = fav::kResidual;
      u.mode = fav::kModeF16;
      u.rows = n_streams * n;
      u.rows_per_stream = n;
      u.k_channels = st.c_out;
      u.num_kblocks = st.c_out < fav::kKBlock ? 1 : st.c_out / fav::kKBlock;
      u.n_total = st.c_out;
      u.n_tile = r.n_tile;
      u.n_major = 1;  // N tiles of one M tile share its input box in L2
      u.c_out = st.c_out;
      u.dilation = r.dilation;
      u.x = X[in];
      u.bias = r.pw_b;
      u.wimg = r.img;
      u.coef = r.coef;
      u.hist = fav::HistRef{2 + 4 * i + j, 2 * r.state_off, 6 * r.dilation, st.c_out};
      u.box_rows = fav::box_rows_for(fav::kResidual, r.dilation);
      u.raw_pitch = st.c_out < fav::kKBlock ? st.c_out : fav::kKBlock;
      if (r.int8) {
        u.mode = fav::kModeI8;
        u.num_kblocks = st.c_out / fav::kKBlockI8;
        u.w_scale = r.sw;
      }
      const bool debug_y = layer + 1 == last_layer;
      u.out_x = X[out];
      u.out_s = S[out];
      if (j < 2) {
        u.epi = fav::kEpiX | (s16 ? fav::kEpiS16 : fav::kEpiS);
        u.next_alpha = st.res[j + 1].pre_a;
        u.next_recip = st.res[j + 1].pre_r;
      } else if (i + 1 < fav::kStages) {
        feed_tconv(u, i + 1, debug_y);
      } else {
        u.epi = fav::kEpiS | (debug_y ? fav::kEpiX : 0);
        u.next_alpha = p->fin_a;
        u.next_recip = p->fin_r;
      }
      if (r.int8) {
        // W8A8: the quantising pre-pass writes the s8 A operand and its row
        // scales into the shifted planes' region (idle in int8 plans but for
        // the up to kMaxRowmaxParts partial row maxima per row the stage's
        // last unit writes at its start for the next int8 conv); the engine
        // TMA-loads it.
        uint8_t* q8 = reinterpret_cast<uint8_t*>(rowmax + (size_t)u.rows * fav::kMaxRowmaxParts);
        float* qscale = reinterpret_cast<float*>(q8 + (size_t)u.rows * st.c_out);
        const fav::QuantResidualArgs qa{S[in], q8, qscale, r.coef, u.rows, n, st.c_out, r.dilation, state, u.hist};
        if ((e = fav::launch_quantize_residual(qa, stream)) != cudaSuccess) return cuda_fail(e, "quantize launch");
        u.kind = fav::kResidualPre;
        u.row_scale = qscale;
        if ((es = encode_s8_map(&u.tmap, q8, u.rows, st.c_out)) != FAV_OK) return es;
      } else if (i <= 1) {
        // Stages 0-1 (8 and 48 rows per stream and frame, mostly history taps,
        // N split over 4 and 2 tiles): the depthwise pre-pass writes the f16 A
        // operand once, behind this layer's Snake output in S[out] (both fit:
        // 1.5 * rows * C <= the region), and the engine TMA-loads it.
        uint16_t* a_op = reinterpret_cast<uint16_t*>(S[out] + (size_t)u.rows * st.c_out);
        const fav::DepthwiseArgs dw{S[in], a_op, r.coef, u.rows, n, st.c_out, r.dilation, state, u.hist};
        if ((e = fav::launch_depthwise(dw, stream)) != cudaSuccess) return cuda_fail(e, "depthwise launch");
        u.kind = fav::kResidualPre;
        if ((es = encode_operand_map(&u.tmap, a_op, u.rows, st.c_out)) != FAV_OK) return es;
      } else if (s16) {
        u.s16 = 1;
        if ((es = encode_input_map_f16(&u.tmap, S[in], u.rows, st.c_out, u.box_rows)) != FAV_OK) return es;
      } else if ((es = encode_input_map(&u.tmap, S[in], u.rows, st.c_out, u.box_rows)) != FAV_OK) {
        return es;
      }
      narrow(u, u.n_tile);
      if (u.epi & fav::kEpiAct) {
        // One partial row maximum per N tile and epilogue column group.
        u.rowmax_parts = (u.n_total / u.n_tile) * fav::epilogue_column_groups(u.n_tile, u.kind);
        act_parts = u.rowmax_parts;
      }
      diagnose(u, layer + 1);
      if ((e = fav::launch_gemm_layer(u, stream)) != cudaSuccess) return cuda_fail(e, "residual launch");
      if (last_out) *last_out = X[out];
      mark(++layer + 1);
      if (layer == last_layer) return FAV_OK;
    }
  }
  // Stage 5's last unit (j = 2) wrote Snake_final(y) to S[1].
  fav::FinalArgs f{};
  f.rows = n_streams * n;
  f.rows_per_stream = n;
  f.x = S[1];
  f.audio = audio;
  f.audio_stride = audio_stride;
  f.audio_offset = audio_offset;
  f.w = p->fin_w;
  f.b = p->fin_b;
  f.state = state;
  f.hist = fav::HistRef{25, 2 * p->state_final, 6, fav::kFinalChannels};
  f.status = status;
  if ((e = fav::launch_final(f, stream)) != cudaSuccess) return cuda_fail(e, "final launch");
  mark(26);
  if (last_out) *last_out = audio;
  return FAV_OK;
}

// The plan's weights live on the device that was current at fav_plan_create;
// every step must run with that device current (its kernels would otherwise
// read another GPU's memory).
int32_t check_device(const fav_plan* plan) {
  int dev = -1;
  const cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev != plan->device)
    return fail(FAV_INVALID_ARGUMENT, "the plan was created on device %d but device %d is current", plan->device, dev);
  return FAV_OK;
}

bool overflow_mul(size_t a, size_t b, size_t* out) {
  if (a && b > SIZE_MAX / a) return true;
  *out = a * b;
  return false;
}

// Step workspace for fav_step_static, for callers that cannot allocate device
// memory (a real-time audio callback, a host that forbids cudaMalloc after
// start-up). It lives in this file-scope device array, so every GPU that loads
// the library holds FAV_STATIC_MAX_FRAMES * 6 * 61440 floats (22.5 MiB) until
// the process exits. Host code must not use the array's name as a device
// address; fav_step_static looks the address up once per device.
__device__ __align__(256) float g_static_workspace[(size_t)FAV_STATIC_MAX_FRAMES * kWorkspaceRegions *
                                                  kRegionFloatsPerFrame];

std::mutex g_static_mutex;
constexpr int kMaxDevices = 64;
void* g_static_address[kMaxDevices] = {};

// Device address of g_static_workspace on the current device, looked up on the
// first call per device (with that device current) and cached.
int32_t static_workspace(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(FAV_UNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_static_mutex);
  if (!g_static_address[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_workspace);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static workspace)");
    g_static_address[dev] = p;
  }
  *out = static_cast<float*>(g_static_address[dev]);
  return FAV_OK;
}

}  // namespace

extern "C" {

int32_t fav_abi_version(void) { return FAV_ABI_VERSION; }

const char* fav_last_error(void) { return g_error; }

const char* fav_status_string(int32_t s) {
  switch (s) {
    case FAV_OK: return "ok";
    case FAV_INVALID_ARGUMENT: return "invalid argument";
    case FAV_UNSUPPORTED: return "unsupported";
    case FAV_OVERLAP: return "overlapping buffers";
    case FAV_SIZE_OVERFLOW: return "size overflow";
    case FAV_DEVICE_ERROR: return "device error";
    case FAV_TIMEOUT: return "device wait timed out";
    default: return "unknown status";
  }
}

int32_t fav_host_device_pointer(void* host, void** device) {
  if (!host || !device) return fail(FAV_INVALID_ARGUMENT, "host and device must be non-null");
  const cudaError_t e = cudaHostGetDevicePointer(device, host, 0);
  if (e != cudaSuccess) {
    cudaGetLastError();  // not sticky: clear it for the caller's next call
    return cuda_fail(e, "not mapped page-locked host memory");
  }
  return FAV_OK;
}

int32_t fav_device_supported(void) {
  int dev = 0, major = 0, minor = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) return 0;
  return major == 10 && minor == 0;
}

int32_t fav_plan_create(const float* const* coefficients, int32_t count, int32_t precision, fav_plan** plan_out) {
  g_error[0] = 0;
  if (!plan_out) return fail(FAV_INVALID_ARGUMENT, "plan_out is NULL");
  *plan_out = nullptr;
  if (!coefficients || count != FAV_NUM_COEFFICIENTS)
    return fail(FAV_INVALID_ARGUMENT, "expected %d coefficient arrays", FAV_NUM_COEFFICIENTS);
  if (precision != FAV_PRECISION_BF16 && precision != FAV_PRECISION_INT8)
    return fail(FAV_UNSUPPORTED, "unsupported precision %d", precision);
  for (int i = 0; i < count; ++i) {
    if (!coefficients[i]) return fail(FAV_INVALID_ARGUMENT, "coefficient %d is NULL", i);
    const size_t nvals = expected_count(i);
    for (size_t j = 0; j < nvals; ++j)
      if (!std::isfinite(coefficients[i][j])) return fail(FAV_INVALID_ARGUMENT, "coefficient %d is not finite", i);
  }
  if (!fav_device_supported()) return fail(FAV_UNSUPPORTED, "current CUDA device is not an sm_100 (B200) GPU");
  cudaError_t e = prepare_once();
  if (e != cudaSuccess) return cuda_fail(e, "kernel attributes");
  fav_plan* plan = new (std::nothrow) fav_plan();
  if (!plan) return fail(FAV_DEVICE_ERROR, "out of host memory");
  cudaGetDevice(&plan->device);
  plan->precision = precision;
  const int32_t st = build_plan(plan, coefficients);
  if (st != FAV_OK) {
    delete plan;
    return st;
  }
  *plan_out = plan;
  return FAV_OK;
}

void fav_plan_destroy(fav_plan* plan) { delete plan; }

size_t fav_plan_bytes(const fav_plan* plan) { return plan ? plan->mem.bytes : 0; }

size_t fav_state_pool_bytes(int32_t num_slots) {
  if (num_slots <= 0) return 0;
  return (size_t)num_slots * fav::kSlotStride * sizeof(float);
}

size_t fav_step_workspace_bytes(int32_t n_streams, int32_t frames) {
  if (n_streams <= 0 || frames <= 0) return 0;
  size_t rows, bytes;
  if (overflow_mul((size_t)n_streams, (size_t)frames, &rows)) return 0;
  if (overflow_mul(rows, kWorkspaceRegions * kRegionFloatsPerFrame * sizeof(float), &bytes)) return 0;
  return bytes;
}

int32_t fav_step(const fav_plan* plan, float* state_pool, int32_t num_slots, const int32_t* slot_codes,
                 int32_t n_streams, int32_t frames, const float* latents, float* audio, void* workspace,
                 size_t workspace_bytes, uint32_t* status, void* cuda_stream) {
  g_error[0] = 0;
  if (!plan) return fail(FAV_INVALID_ARGUMENT, "plan is NULL");
  if (n_streams < 0 || frames < 0) return fail(FAV_INVALID_ARGUMENT, "negative stream or frame count");
  if (n_streams == 0 || frames == 0) return FAV_OK;
  if ((int64_t)n_streams * frames * fav::kHop > INT32_MAX)
    return fail(FAV_SIZE_OVERFLOW, "step too large: %d streams x %d frames", n_streams, frames);
  if (!latents || !audio || !workspace) return fail(FAV_INVALID_ARGUMENT, "NULL latents, audio or workspace");
  if (!state_pool || !slot_codes || num_slots < n_streams)
    return fail(FAV_INVALID_ARGUMENT, "state pool, slot codes and num_slots >= n_streams are required");
  const size_t need = fav_plan_workspace_bytes(plan, n_streams, frames);
  if (!need) return fail(FAV_SIZE_OVERFLOW, "workspace size overflow");
  if (workspace_bytes < need)
    return fail(FAV_INVALID_ARGUMENT, "workspace too small: %zu < %zu bytes", workspace_bytes, need);
  if (const int32_t d = check_device(plan)) return d;
  fav::StateRef st{state_pool, slot_codes, num_slots, 0};
  return run_step(plan, st, n_streams, frames, latents, frames, 0, audio, frames * fav::kHop, 0,
                  static_cast<float*>(workspace), status, static_cast<cudaStream_t>(cuda_stream));
}

int32_t fav_debug_step_unfused(const fav_plan* plan, float* state_pool, int32_t num_slots, const int32_t* slot_codes,
                               int32_t n_streams, int32_t frames, const float* latents, float* audio, void* workspace,
                               size_t workspace_bytes, uint32_t* status, void* cuda_stream) {
  g_error[0] = 0;
  if (!plan || n_streams <= 0 || frames <= 0 || !latents || !audio || !workspace)
    return fail(FAV_INVALID_ARGUMENT, "bad debug step arguments");
  if ((int64_t)n_streams * frames * fav::kHop > INT32_MAX)
    return fail(FAV_SIZE_OVERFLOW, "step too large: %d streams x %d frames", n_streams, frames);
  if (!state_pool || !slot_codes || num_slots < n_streams)
    return fail(FAV_INVALID_ARGUMENT, "state pool, slot codes and num_slots >= n_streams are required");
  if (workspace_bytes < fav_plan_workspace_bytes(plan, n_streams, frames))
    return fail(FAV_INVALID_ARGUMENT, "workspace too small");
  if (const int32_t d = check_device(plan)) return d;
  fav::StateRef st{state_pool, slot_codes, num_slots, 0};
  return run_step(plan, st, n_streams, frames, latents, frames, 0, audio, frames * fav::kHop, 0,
                  static_cast<float*>(workspace), status, static_cast<cudaStream_t>(cuda_stream), 25, nullptr,
                  nullptr, false);
}

int32_t fav_debug_step_gated(const fav_plan* plan, float* state_pool, int32_t num_slots, const int32_t* slot_codes,
                             int32_t n_streams, int32_t frames, const float* latents, float* audio, void* workspace,
                             size_t workspace_bytes, uint32_t* status, int32_t layer, uint32_t wait_limit,
                             const uint32_t* gate, void* cuda_stream) {
  g_error[0] = 0;
  if (!plan || n_streams <= 0 || frames <= 0 || !latents || !audio || !workspace || !status)
    return fail(FAV_INVALID_ARGUMENT, "bad gated step arguments");
  if (layer < 0 || layer > 21 || !gate || wait_limit == 0)
    return fail(FAV_INVALID_ARGUMENT, "layer must be an engine layer (0..21), gate non-NULL and wait_limit > 0");
  if (plan->precision != FAV_PRECISION_BF16)
    return fail(FAV_UNSUPPORTED, "the gated diagnostic step supports FAV_PRECISION_BF16 plans only");
  if ((int64_t)n_streams * frames * fav::kHop > INT32_MAX)
    return fail(FAV_SIZE_OVERFLOW, "step too large: %d streams x %d frames", n_streams, frames);
  if (!state_pool || !slot_codes || num_slots < n_streams)
    return fail(FAV_INVALID_ARGUMENT, "state pool, slot codes and num_slots >= n_streams are required");
  if (workspace_bytes < fav_plan_workspace_bytes(plan, n_streams, frames))
    return fail(FAV_INVALID_ARGUMENT, "workspace too small");
  if (const int32_t d = check_device(plan)) return d;
  fav::StateRef st{state_pool, slot_codes, num_slots, 0};
  const StepDiag diag{layer, wait_limit, gate};
  return run_step(plan, st, n_streams, frames, latents, frames, 0, audio, frames * fav::kHop, 0,
                  static_cast<float*>(workspace), status, static_cast<cudaStream_t>(cuda_stream), 25, nullptr,
                  nullptr, true, &diag);
}

int32_t fav_step_static(const fav_plan* plan, float* state_pool, int32_t num_slots, const int32_t* slot_codes,
                        int32_t n_streams, int32_t frames, const float* latents, float* audio, uint32_t* status,
                        void* cuda_stream) {
  g_error[0] = 0;
  if (!plan) return fail(FAV_INVALID_ARGUMENT, "plan is NULL");
  if (n_streams < 0 || frames < 0) return fail(FAV_INVALID_ARGUMENT, "negative stream or frame count");
  if (n_streams == 0 || frames == 0) return FAV_OK;
  if ((int64_t)n_streams * frames > FAV_STATIC_MAX_FRAMES)
    return fail(FAV_SIZE_OVERFLOW, "n_streams * frames = %lld exceeds the static workspace limit of %d frames",
                (long long)n_streams * frames, FAV_STATIC_MAX_FRAMES);
  if (!latents || !audio) return fail(FAV_INVALID_ARGUMENT, "NULL latents or audio");
  if (!state_pool || !slot_codes || num_slots < n_streams)
    return fail(FAV_INVALID_ARGUMENT, "state pool, slot codes and num_slots >= n_streams are required");
  if (const int32_t d = check_device(plan)) return d;
  float* ws = nullptr;
  const int32_t st = static_workspace(&ws);
  if (st != FAV_OK) return st;
  fav::StateRef ref{state_pool, slot_codes, num_slots, 0};
  return run_step(plan, ref, n_streams, frames, latents, frames, 0, audio, frames * fav::kHop, 0, ws, status,
                  static_cast<cudaStream_t>(cuda_stream));
}

size_t fav_batch_workspace_bytes(int32_t n_clips, int32_t chunk_frames) {
  const size_t act = fav_step_workspace_bytes(n_clips, chunk_frames);
  if (!act) return 0;
  return act + fav_state_pool_bytes(n_clips);
}

size_t fav_plan_workspace_bytes(const fav_plan* plan, int32_t n_streams, int32_t frames) {
  if (!plan) return 0;
  return fav_step_workspace_bytes(n_streams, frames);
}

size_t fav_plan_batch_workspace_bytes(const fav_plan* plan, int32_t n_clips, int32_t chunk_frames) {
  const size_t act = fav_plan_workspace_bytes(plan, n_clips, chunk_frames);
  if (!act) return 0;
  return act + fav_state_pool_bytes(n_clips);
}

int32_t fav_plan_precision(const fav_plan* plan) { return plan ? plan->precision : -1; }

int32_t fav_decode_batch(const fav_plan* plan, const float* latents, int32_t n_clips, int32_t frames,
                         int32_t chunk_frames, float* audio, void* workspace, size_t workspace_bytes,
                         uint32_t* status, void* cuda_stream) {
  g_error[0] = 0;
  if (!plan) return fail(FAV_INVALID_ARGUMENT, "plan is NULL");
  if (n_clips < 0 || frames < 0 || chunk_frames <= 0) return fail(FAV_INVALID_ARGUMENT, "bad clip/frame counts");
  if (n_clips == 0 || frames == 0) return FAV_OK;
  if (!latents || !audio || !workspace) return fail(FAV_INVALID_ARGUMENT, "NULL latents, audio or workspace");
  if ((int64_t)frames * fav::kHop > INT32_MAX || (int64_t)n_clips * chunk_frames * fav::kHop > INT32_MAX)
    return fail(FAV_SIZE_OVERFLOW, "clip too large");
  if (chunk_frames > frames) chunk_frames = frames;
  const size_t need = fav_plan_batch_workspace_bytes(plan, n_clips, chunk_frames);
  if (!need || workspace_bytes < need)
    return fail(FAV_INVALID_ARGUMENT, "workspace too small: %zu < %zu bytes", workspace_bytes, need);
  if (const int32_t d = check_device(plan)) return d;
  float* ws = static_cast<float*>(workspace);
  float* pool = ws + fav_plan_workspace_bytes(plan, n_clips, chunk_frames) / sizeof(float);
  cudaStream_t stream = static_cast<cudaStream_t>(cuda_stream);
  for (int t0 = 0, c = 0; t0 < frames; t0 += chunk_frames, ++c) {
    const int tc = frames - t0 < chunk_frames ? frames - t0 : chunk_frames;
    // Chunk c reads head table (c & 1) (a fresh, zero history for the first chunk) and writes the other.
    fav::StateRef st{pool, nullptr, n_clips, (c == 0 ? 2 : 0) | (c & 1)};
    const int32_t s = run_step(plan, st, n_clips, tc, latents, frames, t0, audio, frames * fav::kHop,
                               t0 * fav::kHop, ws, status, stream);
    if (s != FAV_OK) return s;
  }
  return FAV_OK;
}

int32_t fav_step_profile(const fav_plan* plan, float* state_pool, int32_t num_slots, const int32_t* slot_codes,
                         int32_t n_streams, int32_t frames, const float* latents, float* audio, void* workspace,
                         size_t workspace_bytes, uint32_t* status, float* layer_ms, void* cuda_stream) {
  g_error[0] = 0;
  if (!layer_ms) return fail(FAV_INVALID_ARGUMENT, "layer_ms is NULL");
  if (!plan || n_streams <= 0 || frames <= 0 || !latents || !audio || !workspace || !state_pool || !slot_codes ||
      num_slots < n_streams)
    return fail(FAV_INVALID_ARGUMENT, "bad profile step arguments");
  if (workspace_bytes < fav_plan_workspace_bytes(plan, n_streams, frames))
    return fail(FAV_INVALID_ARGUMENT, "workspace too small");
  if (const int32_t d = check_device(plan)) return d;
  cudaEvent_t ev[27];
  for (int i = 0; i < 27; ++i) {
    cudaError_t e = cudaEventCreate(&ev[i]);
    if (e != cudaSuccess) {
      for (int j = 0; j < i; ++j) cudaEventDestroy(ev[j]);
      return cuda_fail(e, "cudaEventCreate");
    }
  }
  fav::StateRef st{state_pool, slot_codes, num_slots, 0};
  cudaStream_t stream = static_cast<cudaStream_t>(cuda_stream);
  int32_t r = run_step(plan, st, n_streams, frames, latents, frames, 0, audio, frames * fav::kHop, 0,
                       static_cast<float*>(workspace), status, stream, 25, nullptr, ev);
  if (r == FAV_OK) {
    cudaError_t e = cudaEventSynchronize(ev[26]);
    for (int i = 0; i < 26 && e == cudaSuccess; ++i) e = cudaEventElapsedTime(&layer_ms[i], ev[i], ev[i + 1]);
    if (e != cudaSuccess) r = cuda_fail(e, "profile events");
  }
  for (int i = 0; i < 27; ++i) cudaEventDestroy(ev[i]);
  return r;
}

int32_t fav_debug_step_layers(const fav_plan* plan, float* state_pool, int32_t num_slots, const int32_t* slot_codes,
                              int32_t n_streams, int32_t frames, const float* latents, void* workspace,
                              size_t workspace_bytes, uint32_t* status, int32_t last_layer, float** layer_out,
                              void* cuda_stream) {
  g_error[0] = 0;
  if (!plan || !layer_out || last_layer < 0 || last_layer > 24 || n_streams <= 0 || frames <= 0 || !latents ||
      !workspace)
    return fail(FAV_INVALID_ARGUMENT, "bad debug step arguments");
  if (workspace_bytes < fav_plan_workspace_bytes(plan, n_streams, frames))
    return fail(FAV_INVALID_ARGUMENT, "workspace too small");
  if (state_pool && (!slot_codes || num_slots < n_streams))
    return fail(FAV_INVALID_ARGUMENT, "slot codes and num_slots >= n_streams are required with a state pool");
  if (const int32_t d = check_device(plan)) return d;
  fav::StateRef st{state_pool, state_pool ? slot_codes : nullptr, num_slots, 0};
  return run_step(plan, st, n_streams, frames, latents, frames, 0, nullptr, 0, 0, static_cast<float*>(workspace),
                  status, static_cast<cudaStream_t>(cuda_stream), last_layer, layer_out);
}

int32_t fav_test_gemm(const float* a, int32_t m, int32_t k, const float* b, int32_t n, int32_t mode, float* c,
                      void* cuda_stream) {
  g_error[0] = 0;
  if (!a || !b || !c || m <= 0 || k <= 0 || n <= 0) return fail(FAV_INVALID_ARGUMENT, "bad test GEMM arguments");
  if (k % 2) return fail(FAV_INVALID_ARGUMENT, "K must be even");
  int nt = n % 256 == 0 ? 256 : n % 128 == 0 ? 128 : n % 64 == 0 ? 64 : n % 32 == 0 ? 32 : 0;
  if (!nt) return fail(FAV_INVALID_ARGUMENT, "N must be a multiple of 32");
  cudaError_t e = prepare_once();
  if (e != cudaSuccess) return cuda_fail(e, "kernel attributes");
  if (mode < 0 || mode > 2) return fail(FAV_INVALID_ARGUMENT, "mode must be 0, 1 or 2");
  const int md = mode == 2 ? fav::kModeI8 : mode ? fav::kModeSplit : fav::kModeF16;
  std::vector<uint8_t> img;
  if (md == fav::kModeI8) {
    // Operands hold integers in [-127, 127]; B is packed as it is (no scales).
    const int kb = (k + fav::kKBlockI8 - 1) / fav::kKBlockI8;
    img.assign((size_t)(n / nt) * kb * nt * 128, 0);
    for (int row = 0; row < n; ++row)
      for (int col = 0; col < k; ++col) {
        const int tile = row / nt, r = row % nt, blk = col / fav::kKBlockI8, kk = col % fav::kKBlockI8;
        const long q = std::lround(b[(size_t)row * k + col]);
        if (q < -127 || q > 127) return fail(FAV_INVALID_ARGUMENT, "int8 test operands must be integers in [-127, 127]");
        img[((size_t)tile * kb + blk) * nt * 128 + (size_t)r * 128 + ((((kk >> 4) ^ (r & 7)) << 4) | (kk & 15))] =
            static_cast<uint8_t>(static_cast<int8_t>(q));
      }
  } else {
    auto h = pack_operand(n, k, nt, md, [b, k](int row, int col) { return b[(size_t)row * k + col]; });
    img.resize(h.size() * 2);
    std::memcpy(img.data(), h.data(), img.size());
  }
  void* dimg = nullptr;
  uint32_t* dstatus = nullptr;
  if ((e = cudaMalloc(&dimg, img.size())) != cudaSuccess) return cuda_fail(e, "cudaMalloc");
  if ((e = cudaMalloc(&dstatus, 4)) != cudaSuccess) {
    cudaFree(dimg);
    return cuda_fail(e, "cudaMalloc");
  }
  cudaMemcpy(dimg, img.data(), img.size(), cudaMemcpyHostToDevice);
  cudaMemset(dstatus, 0, 4);
  fav::LayerArgs la{};
  la.kind = fav::kTestGemm;
  la.mode = md;
  la.rows = m;
  la.rows_per_stream = m;
  la.k_channels = k;
  la.num_kblocks = md == fav::kModeI8 ? (k + fav::kKBlockI8 - 1) / fav::kKBlockI8 : (k + fav::kKBlock - 1) / fav::kKBlock;
  la.n_total = n;
  la.n_tile = nt;
  la.c_out = n;
  la.epi = fav::kEpiX;
  la.x = a;
  la.wimg = static_cast<const uint8_t*>(dimg);
  la.status = dstatus;
  cudaStream_t stream = static_cast<cudaStream_t>(cuda_stream);
  la.out_x = c;
  e = fav::launch_gemm_layer(la, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  uint32_t hs = 0;
  if (e == cudaSuccess) e = cudaMemcpy(&hs, dstatus, 4, cudaMemcpyDeviceToHost);
  cudaFree(dimg);
  cudaFree(dstatus);
  if (e != cudaSuccess) return cuda_fail(e, "test GEMM");
  if (hs) return fail(FAV_TIMEOUT, "test GEMM kernel status 0x%x", hs);
  return FAV_OK;
}

int32_t fav_test_sine(const float* x, int32_t n, float* out, void* cuda_stream) {
  g_error[0] = 0;
  if (!x || !out || n < 0) return fail(FAV_INVALID_ARGUMENT, "bad sine test arguments");
  const cudaError_t e = fav::launch_sine_test(x, n, out, static_cast<cudaStream_t>(cuda_stream));
  return e == cudaSuccess ? FAV_OK : cuda_fail(e, "sine test launch");
}

}  // extern "C"
