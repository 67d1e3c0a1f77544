// Warp-level bf16 tensor-core helpers (m16n8k16, fp32 accumulate) and ldmatrix fragment loaders
// for row-major shared-memory tiles, plus cp.async staging.
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

namespace cqb {
namespace ws {

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid = true) {
  // zero-fills the 16 bytes when !valid (src-size 0)
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src),
               "r"(valid ? 16 : 0));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t* r, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"((uint32_t)__cvta_generic_to_shared(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t* r, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"((uint32_t)__cvta_generic_to_shared(p)));
}

__device__ __forceinline__ void mma16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// A (16x16) from row-major [m][k].
__device__ __forceinline__ void frag_a(uint32_t* r, const __nv_bfloat16* base, int m0, int k0, int ld, int lane) {
  ldsm_x4(r, base + (m0 + (lane & 15)) * ld + k0 + (lane >> 4) * 8);
}
// A = X^T, X row-major [k][m].
__device__ __forceinline__ void frag_at(uint32_t* r, const __nv_bfloat16* base, int m0, int k0, int ld, int lane) {
  const int k = k0 + (lane & 7) + ((lane >> 4) << 3);
  const int m = m0 + ((lane >> 3) & 1) * 8;
  ldsm_x4_t(r, base + k * ld + m);
}
// Two B fragments (n-tiles n0, n0+8) of B row-major [k][n]:  r = {b0(n0), b1(n0), b0(n0+8), b1(n0+8)}.
__device__ __forceinline__ void frag_b2(uint32_t* r, const __nv_bfloat16* base, int k0, int n0, int ld, int lane) {
  const int k = k0 + (lane & 7) + ((lane >> 3) & 1) * 8;
  const int n = n0 + (lane >> 4) * 8;
  ldsm_x4_t(r, base + k * ld + n);
}
// Two B fragments of B = X^T with X row-major [n][k] (e.g. keys x dims for S = Q K^T).
__device__ __forceinline__ void frag_bt2(uint32_t* r, const __nv_bfloat16* base, int k0, int n0, int ld, int lane) {
  const int n = n0 + (lane & 7) + (lane >> 4) * 8;
  const int k = k0 + ((lane >> 3) & 1) * 8;
  ldsm_x4(r, base + n * ld + k);
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Accumulator tiles (n-tiles 2i, 2i+1 of a 16-row strip) -> A fragment for the next product over k.
__device__ __forceinline__ void acc_to_a(uint32_t* a, const float* c0, const float* c1) {
  a[0] = pack_bf16(c0[0], c0[1]);
  a[1] = pack_bf16(c0[2], c0[3]);
  a[2] = pack_bf16(c1[0], c1[1]);
  a[3] = pack_bf16(c1[2], c1[3]);
}

}  // namespace ws
}  // namespace cqb
