// bt_async.h -- asynchronous global->shared copies (cp.async) shared by the
// row kernels.
#pragma once
#include <stdint.h>

namespace bt {

__device__ __forceinline__ int phase4(const void* p) { return (int)(((uintptr_t)p >> 2) & 3); }

// 16-byte copy; both addresses 16-byte aligned.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem_dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem_src) : "memory");
}
// 8-byte copy; both addresses 8-byte aligned.
__device__ __forceinline__ void cp_async8(void* smem_dst, const void* gmem_src) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem_dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(s), "l"(gmem_src) : "memory");
}
// 4-byte copy; both addresses 4-byte aligned.
__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gmem_src) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem_dst);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
// Waits until at most N of this thread's committed copy groups are pending.
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
}

// Starts copying n floats g[0..n) into b[0..n) (b shares g's 16-byte phase)
// with the `lanes` threads whose index (0..lanes-1) is `t`: 16-byte copies
// for the aligned interior, 4-byte copies for the at most six edge elements,
// so no thread waits on a load here.
__device__ __forceinline__ void stage_floats_async(float* b, const float* g, int n, int t, int lanes) {
  int head = (4 - phase4(g)) & 3;
  if (head > n) head = n;
  const int nvec = (n - head) >> 2;
  for (int q = t; q < nvec; q += lanes) cp_async16(b + head + 4 * q, g + head + 4 * q);
  const int tail0 = head + 4 * nvec;
  const int nedge = head + (n - tail0);
  for (int e = t; e < nedge; e += lanes) {
    const int i = e < head ? e : tail0 + (e - head);
    cp_async4(b + i, g + i);
  }
}

}  // namespace bt
