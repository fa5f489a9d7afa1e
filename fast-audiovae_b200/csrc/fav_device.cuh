// Device-side primitives for the sm_100a decoder kernels: mbarriers with
// bounded waits, bulk global->shared copies, tcgen05 MMA/TMEM access and the
// shared-memory operand layout (K-major, 128-byte swizzle) the MMAs read.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace fav {

// Error codes a kernel records in the status word (first error wins).
enum DeviceError : uint32_t {
  kDevOk = 0,
  kDevTimeoutProducer = 0x101,
  kDevTimeoutLoader = 0x102,
  kDevTimeoutMma = 0x103,
  kDevTimeoutEpilogue = 0x104,
  kDevBadLaunch = 0x105,
  kDevNonFinite = 0x106,  // the step produced a non-finite audio sample
  kDevTimeoutGate = 0x107,  // a diagnostic launch's gate flag was never set
};

// A wait that has not completed after this many polls is a bug; the kernel
// records the error and returns instead of spinning forever. Each poll may
// suspend the warp for up to kSuspendNs (it resumes when the phase completes),
// so a wait gives up after at most ~kWaitLimit * kSuspendNs (about 2.6 s).
constexpr uint32_t kWaitLimit = 1u << 18;
constexpr uint32_t kSuspendNs = 10000;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void record_error(uint32_t* status, uint32_t code) {
  if (status) atomicCAS(status, 0u, code);
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendNs)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase with ``parity`` to complete. Returns false (and
// records ``code``) after ``limit`` polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* status, uint32_t code,
                                          uint32_t limit = kWaitLimit) {
  for (uint32_t i = 0; i < limit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  record_error(status, code);
  return false;
}

// Bounded wait for a device flag (global memory) to become nonzero. Returns
// false (and records ``code``) after ``limit`` polls.
__device__ __forceinline__ bool flag_wait(const uint32_t* flag, uint32_t* status, uint32_t code, uint32_t limit) {
  for (uint32_t i = 0; i < limit; ++i) {
    uint32_t v;
    asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (v) return true;
    __nanosleep(64);
  }
  record_error(status, code);
  return false;
}

// ----------------------------------------------------------- bulk copies
// 1-D bulk copy global -> own shared memory, completion counted on ``bar``.
// Source and destination 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Bulk prefetch of a global range into L2 (no shared memory involved).
// Address 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// 2-D TMA tile load (no multicast) of the box at coordinates (x = innermost,
// y) into own shared memory, completion counted on ``bar``. Out-of-range
// coordinates read as zero. ``map`` must live in param/const/global space.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// 4-D TMA tile store of the box at coordinates (x = innermost, y, z, w) from
// own shared memory, in the issuing thread's bulk async-group. Rows outside
// the tensor are not written; x must be 16-byte aligned and every coordinate
// non-negative.
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int x, int y, int z, int w) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(src))
               : "memory");
}
// Closes the issuing thread's current bulk async-group.
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until every bulk group of this thread has finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Waits until every bulk group of this thread has completed (writes visible).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Programmatic dependent launch. A kernel launched with the programmatic
// stream serialization attribute may start while the previous kernel in the
// stream is still draining: it waits here, before touching any memory an
// earlier kernel writes or reads, until that kernel has completed and its
// writes are visible, then lets the next kernel in the stream launch (whose
// blocks take SMs only as this kernel's blocks finish). Both are no-ops in a
// kernel launched the ordinary way.
__device__ __forceinline__ void grid_dependency_sync() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Make generic-proxy shared-memory writes visible to the async proxy (MMA).
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void named_barrier(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
// Named barrier that returns the AND of ``pred`` over all participating threads.
__device__ __forceinline__ bool named_barrier_and(uint32_t id, uint32_t threads, bool pred) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %3, 0;\n\tbar.red.and.pred p, %1, %2, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(out)
      : "r"(id), "r"(threads), "r"((uint32_t)pred)
      : "memory");
  return out != 0;
}

// --------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (f16 or bf16 operands, fp32 accumulate).
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, kind::i8 (signed 8-bit operands, s32 accumulate).
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on ``bar`` when all previously issued MMAs of this thread finish.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
// 32 lanes x 16 consecutive fp32 columns of the accumulator, issued without
// waiting: the registers are valid only after tmem_wait_ld on the same array,
// which names them as operands so no use can be scheduled ahead of the wait.
__device__ __forceinline__ void tmem_ld16_async(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15])
               :
               : "memory");
}

// 32 lanes x 16 consecutive fp32 columns from registers into the accumulator
// memory, then a wait until the stores have completed (so a thread that syncs
// with others afterwards publishes them, with the tcgen05 thread-sync fences).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// ------------------------------------------------------------ descriptors
// Instruction descriptor, kind::i8: s32 accumulator, signed 8-bit K-major A and B. M = 128.
__host__ __device__ constexpr uint32_t instr_desc_i8(uint32_t n) {
  return (2u << 4)              // D format s32
         | (1u << 7)            // A format s8
         | (1u << 10)           // B format s8
         | ((n >> 3) << 17)     // N / 8
         | ((128u >> 4) << 24); // M / 16
}
// Instruction descriptor, kind::f16: fp32 accumulator, K-major A and B.
// fmt: 0 = f16, 1 = bf16. M = 128.
__host__ __device__ constexpr uint32_t instr_desc_f16(uint32_t fmt, uint32_t n) {
  return (1u << 4)              // D format f32
         | (fmt << 7)           // A format
         | (fmt << 10)          // B format
         | ((n >> 3) << 17)     // N / 8
         | ((128u >> 4) << 24); // M / 16
}
// Shared-memory matrix descriptor for a K-major operand tile stored as rows of
// 128 bytes (64 sixteen-bit elements) with the 128-byte swizzle; 8-row groups
// are 1024 bytes apart. ``addr`` is the tile (or K-step) start.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  return (uint64_t)((addr & 0x3FFFFu) >> 4)  // start address
         | ((uint64_t)1 << 16)               // leading byte offset (unused with swizzle)
         | ((uint64_t)(1024 >> 4) << 32)     // stride byte offset: 8 rows
         | ((uint64_t)1 << 46)               // descriptor version (sm100)
         | ((uint64_t)2 << 61);              // SWIZZLE_128B
}
// Byte offset of 16-bit element (row, k) inside such a tile (k < 64).
__host__ __device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t k) {
  const uint32_t chunk = (k >> 3) ^ (row & 7u);
  return row * 128u + (chunk << 4) + ((k & 7u) << 1);
}

// --------------------------------------------------------------- numerics
// Packed fp32 pairs (the sm_100 f32x2 instructions: two lanes per issue slot).
// Each lane rounds to nearest exactly as the scalar operation does. The
// assembler may fuse a packed multiply whose result feeds a packed add into
// one packed fused multiply-add (a single rounding), even with the rounding
// mode explicit, so these are used only where no product feeds an add: the
// bf16 path's Snake and depthwise chains. The int8 path's fixed operation
// order keeps scalar __fmul_rn / __fadd_rn.
__device__ __forceinline__ uint64_t f2pack(float2 v) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(v.x), "f"(v.y));
  return r;
}
__device__ __forceinline__ float2 f2unpack(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ float2 f2mul(float2 a, float2 b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2pack(a)), "l"(f2pack(b)));
  return f2unpack(d);
}
__device__ __forceinline__ float2 f2add(float2 a, float2 b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2pack(a)), "l"(f2pack(b)));
  return f2unpack(d);
}
__device__ __forceinline__ float2 f2fma(float2 a, float2 b, float2 c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(f2pack(a)), "l"(f2pack(b)), "l"(f2pack(c)));
  return f2unpack(d);
}

// Snake with the stored reciprocal: x + r * sin(a*x)^2.
__device__ __forceinline__ float snake(float x, float a, float r) {
  const float s = __sinf(a * x);
  return fmaf(r, s * s, x);
}
// Sine in a fixed sequence of IEEE fp32 operations (no fused multiply-add),
// the same sequence as the int8 oracle's ``sin_cw``: Cody-Waite argument
// reduction (Cody & Waite, Software Manual for the Elementary Functions, 1980)
// with pi/2 = P1 + P2 + P3 (P1, P2 of 15 significant bits, so k*P1 and k*P2 are
// exact for |k| < 2^9), then Taylor polynomials of degree 11 (sine) and 12
// (cosine) on [-pi/4, pi/4] by Horner's rule. The constants are 2/pi, the
// parts of pi/2 and +-1/n! rounded to fp32. Within ~1.3 ulp of sin for the
// arguments Snake sees.
__device__ __forceinline__ float sin_cw(float x) {
  const float k = rintf(__fmul_rn(x, 0x1.45f306p-1f));
  const float r = __fsub_rn(__fsub_rn(__fsub_rn(x, __fmul_rn(k, 0x1.921cp+0f)), __fmul_rn(k, 0x1.daap-15f)),
                            __fmul_rn(k, 0x1.10b46p-30f));
  const float r2 = __fmul_rn(r, r);
  float ps = __fmul_rn(r2, -0x1.ae6456p-26f);  // -1/11!
  ps = __fmul_rn(r2, __fadd_rn(ps, 0x1.71de3ap-19f));   // 1/9!
  ps = __fmul_rn(r2, __fadd_rn(ps, -0x1.a01a02p-13f));  // -1/7!
  ps = __fmul_rn(r2, __fadd_rn(ps, 0x1.111112p-7f));    // 1/5!
  ps = __fmul_rn(r2, __fadd_rn(ps, -0x1.555556p-3f));   // -1/3!
  const float sin_r = __fadd_rn(r, __fmul_rn(r, ps));
  float pc = __fmul_rn(r2, 0x1.1eed8ep-29f);   // 1/12!
  pc = __fmul_rn(r2, __fadd_rn(pc, -0x1.27e4fcp-22f));  // -1/10!
  pc = __fmul_rn(r2, __fadd_rn(pc, 0x1.a01a02p-16f));   // 1/8!
  pc = __fmul_rn(r2, __fadd_rn(pc, -0x1.6c16c2p-10f));  // -1/6!
  pc = __fmul_rn(r2, __fadd_rn(pc, 0x1.555556p-5f));    // 1/4!
  pc = __fmul_rn(r2, __fadd_rn(pc, -0x1p-1f));          // -1/2!
  const float cos_r = __fadd_rn(1.f, pc);
  const int q = static_cast<int>(k) & 3;
  return q == 0 ? sin_r : q == 1 ? cos_r : q == 2 ? -sin_r : -cos_r;
}
// Snake in the int8 path's fixed operation order (mps_decoder.py:44-50:
// scaled = alpha*x; s = sin(scaled); y = x + r*(s*s), each step rounded). A
// quantised cascade turns any difference before a quantisation step into
// whole-step rounding flips downstream, so the int8 path and its oracle share it.
__device__ __forceinline__ float snake_exact(float x, float a, float r) {
  const float s = sin_cw(__fmul_rn(a, x));
  return __fadd_rn(x, __fmul_rn(r, __fmul_rn(s, s)));
}
// Two lanes of snake: x + r * sin(a*x)^2 with the hardware sine; the
// products and the fused multiply-add as packed fp32 operations (the same
// roundings as snake).
__device__ __forceinline__ float2 snake2(float2 x, float2 a, float2 r) {
  const float2 ax = f2mul(a, x);
  const float2 s = make_float2(__sinf(ax.x), __sinf(ax.y));
  return f2fma(r, f2mul(s, s), x);
}

// The W8A8 recipe's symmetric quantisation (precision.cpp:82-92 of the
// reference): scale = max|v| / 127 in fp32 (1 for an all-zero vector, max|v|
// itself when the quotient underflows to zero); q = clamp(v / scale, -127, 127)
// rounded half to even. Both divisions are IEEE round-to-nearest.
__device__ __forceinline__ float quant_scale(float mx) {
  if (mx == 0.f) return 1.f;
  const float s = __fdiv_rn(mx, 127.f);
  return s > 0.f ? s : mx;
}
__device__ __forceinline__ uint32_t quant_byte(float v, float scale) {
  const float q = fminf(fmaxf(__fdiv_rn(v, scale), -127.f), 127.f);
  return static_cast<uint32_t>(__float2int_rn(q)) & 0xffu;
}
// Four quantised values packed little-endian (v.x in the lowest byte).
__device__ __forceinline__ uint32_t quant4(float4 v, float scale) {
  return quant_byte(v.x, scale) | (quant_byte(v.y, scale) << 8) | (quant_byte(v.z, scale) << 16) |
         (quant_byte(v.w, scale) << 24);
}

__device__ __forceinline__ uint32_t pack_bf16(float lo_elem, float hi_elem) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo_elem, hi_elem);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ uint32_t pack_f16(float lo_elem, float hi_elem) {
  __half2 v = __floats2half2_rn(lo_elem, hi_elem);
  return *reinterpret_cast<uint32_t*>(&v);
}
// Split two fp32 values into bf16 (hi, lo) pairs with v ~= hi + lo.
__device__ __forceinline__ void split_bf16(float v0, float v1, uint32_t& hi, uint32_t& lo) {
  hi = pack_bf16(v0, v1);
  const float h0 = __uint_as_float(hi << 16), h1 = __uint_as_float(hi & 0xffff0000u);
  lo = pack_bf16(v0 - h0, v1 - h1);
}

}  // namespace fav
