// Device helpers shared by the DeepSeek-V4.1 decode kernels (sm_100a).
//
// Numeric conventions: every "bf16-valued" quantity is rounded with __float2bfloat16_rn;
// FP8 is e4m3fn, encoded with satfinite round-to-nearest-even after an explicit clamp;
// E8M0 codes are biased exponents (value 2^(code - 127)). The scalar rules mirror the
// CPU oracle bit for bit where a stage's output must be bit-exact (KV records, routing).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace dsv41 {

constexpr int kWarp = 32;
constexpr float kFp8Max = 448.0f;
constexpr float kFltMin = 1.17549435082228750797e-38f;
constexpr float kRmsEps = 1e-20f;  // rms_norm_eps of V4

// ------------------------------------------------------------------ scalars
__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
__device__ __forceinline__ float bf2f(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float bfbits2f(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }
__device__ __forceinline__ uint16_t f2bfbits(float x) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  return (uint32_t)f2bfbits(lo) | ((uint32_t)f2bfbits(hi) << 16);
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  return (uint32_t)__half_as_ushort(__float2half_rn(lo)) | ((uint32_t)__half_as_ushort(__float2half_rn(hi)) << 16);
}
// bf16x2 bits -> f16x2 bits (exact for magnitudes in fp16's normal range).
__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t v) {
  return pack_f16x2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
}

// e4m3fn byte of x clamped to +-448 (round to nearest even).
__device__ __forceinline__ uint8_t e4m3_byte(float x) {
  x = fminf(fmaxf(x, -kFp8Max), kFp8Max);
  return (uint8_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
}
__device__ __forceinline__ float e4m3_float(uint8_t b) {
  __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)b, __NV_E4M3);
  return __half2float(__half(h));
}

// Biased exponent of the smallest power of two >= v (v >= 0).
__device__ __forceinline__ int code_ceil(float v) {
  uint32_t b = __float_as_uint(v);
  return (int)((b >> 23) & 0xFF) + ((b & 0x7FFFFF) != 0);
}
// 2^(127 - code) as the bit pattern (254 - code) << 23 (code 254 gives 0).
__device__ __forceinline__ float mx_mul(int code) { return __uint_as_float((uint32_t)(254 - code) << 23); }
// 2^(code - 127), exact for every code 0..254.
__device__ __forceinline__ float pow2c(int code) {
  return code ? __uint_as_float((uint32_t)code << 23) : __uint_as_float(0x400000u);
}

// vLLM's MXFP8 scale code: clamp(code_ceil(RN(max(amax, FLT_MIN) / 448)), 0, 254).
__device__ __forceinline__ int mx_code_vllm(float amax) {
  int c = code_ceil(__fdiv_rn(fmaxf(amax, kFltMin), kFp8Max));
  return min(max(c, 0), 254);
}
// aiter's routed-expert code: clamp(code_ceil(max(amax, 1e-10) * RN(1/448)), 1, 254).
__device__ __forceinline__ int mx_code_aiter(float amax) {
  int c = code_ceil(__fmul_rn(fmaxf(amax, 1e-10f), 1.0f / 448.0f));
  return min(max(c, 1), 254);
}

// ------------------------------------------------------------------ warp reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
  return v;
}
// v[q] = the sum over k < kslices of src[k kstride + q] (q < 8), added in k order from 0.f; the
// loads of 4 slices (two 16-byte loads each) are in flight together, where a loop of scalar
// loads a value would wait out one memory latency a slice. src 16-byte aligned, kstride a
// multiple of 4 floats.
__device__ __forceinline__ void sum_slices8(const float* src, size_t kstride, int kslices, float (&v)[8]) {
#pragma unroll
  for (int q = 0; q < 8; ++q) v[q] = 0.f;
  int k = 0;
  for (; k + 4 <= kslices; k += 4) {
    float4 u[4][2];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4* p = reinterpret_cast<const float4*>(src + (size_t)(k + i) * kstride);
      u[i][0] = p[0];
      u[i][1] = p[1];
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[0] += u[i][0].x; v[1] += u[i][0].y; v[2] += u[i][0].z; v[3] += u[i][0].w;
      v[4] += u[i][1].x; v[5] += u[i][1].y; v[6] += u[i][1].z; v[7] += u[i][1].w;
    }
  }
  for (; k < kslices; ++k) {
    const float4* p = reinterpret_cast<const float4*>(src + (size_t)k * kstride);
    const float4 a = p[0], b = p[1];
    v[0] += a.x; v[1] += a.y; v[2] += a.z; v[3] += a.w;
    v[4] += b.x; v[5] += b.y; v[6] += b.z; v[7] += b.w;
  }
}
// 32 sums over the warp at once: lane l ends with the warp's sum of v[l] (v is consumed). Each
// step halves the values a lane holds and exchanges the other half with the xor partner, so
// value j meets the same partners in the same order (16, 8, 4, 2, 1) as warp_sum(v[j]) and
// gives the same bits, in 31 shuffles over 5 dependent steps instead of 160 over 5 x 32.
__device__ __forceinline__ float warp_transpose_sum(float (&v)[32], int lane) {
#pragma unroll
  for (int step = 16; step >= 1; step >>= 1) {
    const bool upper = (lane & step) != 0;
#pragma unroll
    for (int i = 0; i < step; ++i) {
      const float send = upper ? v[i] : v[i + step];
      const float keep = upper ? v[i + step] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, step);
    }
  }
  return v[0];
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, d));
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, d));
  return v;
}

// ------------------------------------------------------------------ memory
// Streaming 16-byte load of data read once (weights): no L1 allocation.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint4 ldg16(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// Asynchronous global -> shared copies (no register staging); completion by commit groups.
__device__ __forceinline__ void cp_async16_stream(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint4 lds16(uint32_t addr) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(addr));
  return r;
}
__device__ __forceinline__ uint2 lds8(uint32_t addr) {
  uint2 r;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "r"(addr));
  return r;
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x2(uint32_t (&r)[2], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x2_trans(uint32_t (&r)[2], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(addr));
}

// ------------------------------------------------------------------ tensor-core MMA
// D += A(16x16, row) * B(16x8, col), fp32 accumulate.
__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_f16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                       uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Four e4m3 bytes w = (b0, b1, b2, b3) as two bf16x2 registers (b0, b2) and (b1, b3), each
// value scaled by 2^-120: the e4m3 magnitude bits shifted into bf16's exponent/mantissa
// field. Exact for every code, subnormals included (they become bf16 subnormals).
__device__ __forceinline__ void e4m3x4_bf16(uint32_t w, uint32_t& lo, uint32_t& hi) {
  lo = ((w << 4) & 0x07F007F0u) | ((w << 8) & 0x80008000u);
  hi = ((w >> 4) & 0x07F007F0u) | (w & 0x80008000u);
}

// Two E2M1 nibbles (low nibble first) as an f16x2 register (exact).
__device__ __forceinline__ uint32_t e2m1x2_f16(uint32_t byte) {
  uint32_t r;
  asm("{ .reg .b8 t; cvt.u8.u32 t, %1; cvt.rn.f16x2.e2m1x2 %0, t; }" : "=r"(r) : "r"(byte));
  return r;
}
// Two e4m3 bytes (low byte first) as an f16x2 register (exact).
__device__ __forceinline__ uint32_t e4m3x2_f16(uint32_t two) {
  uint32_t r;
  asm("{ .reg .b16 t; cvt.u16.u32 t, %1; cvt.rn.f16x2.e4m3x2 %0, t; }" : "=r"(r) : "r"(two));
  return r;
}

__device__ __forceinline__ uint32_t hmul2_bits(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Four e4m3 bytes of w (byte 0 lowest) -> two f16x2 words {b0, b1}, {b2, b3}, each times the f16x2
// factor s2 (both halves the same power of two, 2^8 x the wanted scale), by integer ops and one f16
// multiply a word: an e4m3 byte s.eeee.mmm placed as the f16 bits s.0eeee.mmm0000000 is its value
// times 2^-8 exactly, normal and subnormal alike (e4m3 bias 7, f16 bias 15: exponent fields that
// differ by 8; subnormal mantissas alike), so the multiply by s2 rounds the exact product once --
// the bits cvt.rn.f16x2.e4m3x2 and a multiply by the scale give. (e4m3 NaN, 0x7f / 0xff, becomes a
// finite value: the KV records never hold it.)
__device__ __forceinline__ void e4m3x4_f16x2_scaled(uint32_t w, uint32_t s2, uint32_t& lo, uint32_t& hi) {
  uint32_t z0, z1;
  asm("prmt.b32 %0, %1, 0, 0x1404;" : "=r"(z0) : "r"(w));  // {0, b0, 0, b1}
  asm("prmt.b32 %0, %1, 0, 0x3424;" : "=r"(z1) : "r"(w));  // {0, b2, 0, b3}
  lo = hmul2_bits(((z0 >> 1) & 0x3F803F80u) | (z0 & 0x80008000u), s2);
  hi = hmul2_bits(((z1 >> 1) & 0x3F803F80u) | (z1 & 0x80008000u), s2);
}
// The f16x2 factor of e4m3x4_f16x2_scaled for an E8M0 scale code: 2^8 x 2^(code - 127), a
// normal f16 for codes 105 .. 134.
__device__ __forceinline__ bool e4m3_f16_scale_ok(int code) { return code >= 105 && code <= 134; }
__device__ __forceinline__ uint32_t e4m3_f16_scale(int code) {
  const uint32_t s1 = (uint32_t)(code - 104) << 10;
  return s1 | (s1 << 16);
}
__device__ __forceinline__ float2 e4m3x2_float2(uint32_t two) {
  const uint32_t h = e4m3x2_f16(two);
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}
__device__ __forceinline__ float2 e2m1x2_float2(uint32_t byte) {
  const uint32_t h = e2m1x2_f16(byte);
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}

// ------------------------------------------------------------------ PDL
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;"); }

__host__ __device__ __forceinline__ int cdiv(int a, int b) { return (a + b - 1) / b; }

// A RoPE table row for position p: clamped into the table's rows (rows = 0: unchecked), so a
// position past the table reads its last row instead of memory past it.
__device__ __forceinline__ int64_t rope_row(int64_t p, int64_t rows) {
  return rows > 0 ? min(max(p, (int64_t)0), rows - 1) : p;
}

// Raise a kernel's dynamic shared-memory limit once per (kernel, device) -- not on every
// launch, so launches captured into a CUDA graph make no attribute calls after the first.
cudaError_t ensure_smem(const void* kernel, int bytes);

}  // namespace dsv41
