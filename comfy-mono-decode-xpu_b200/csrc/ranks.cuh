// 64-bit ranks of bf16 logits for exact top-k / argmax (larger = better), shared by the top-k kernels (topk.cu) and
// the lm_head pick (lmhead.cu). The tie orders are the reference's (csrc/fast_topk.sycl:22-40), which reproduce
// torch's on its device, so they are kept as the reference defines them:
//   top-k   high half: the bf16 radix key (NaN on top, -0 below +0); low half: ~(the XPU topk gather key)
//           (i >> 15) << 15 | ((i & 8191) >> 3) << 5 | ((i & 32767) >> 13) << 3 | (i & 7)
//   argmax  high half: the float order key (NaN largest, -0 == +0); low half: ~i (smallest index on ties)
// Ranks of distinct indices differ, so a set of candidates has one exact order whatever the merge order.
#pragma once
#include "common.cuh"

namespace mono {

constexpr int kTkK = 8;  // largest k

__device__ __forceinline__ uint64_t rank_topk(uint16_t bits, uint32_t i) {
    const uint32_t mask = (bits & 0x8000u) ? 0xFFFFu : 0x8000u;
    const bool nan = (bits & 0x7FFFu) > 0x7F80u;
    const uint32_t conv = nan ? 0xFFFFu : ((bits ^ mask) & 0xFFFFu);
    const uint32_t it = i >> 15, off = i & 32767u;
    const uint32_t g = (it << 15) | (((off & 8191u) >> 3) << 5) | ((off >> 13) << 3) | (off & 7u);
    return (uint64_t(conv) << 32) | uint64_t(0xFFFFFFFFu - g);
}
__device__ __forceinline__ uint64_t rank_argmax(uint16_t bits, uint32_t i) {
    const bool nan = (bits & 0x7FFFu) > 0x7F80u;
    uint32_t key;
    if (nan) {
        key = 0xFFFFFFFFu;
    } else {
        const uint16_t b = (bits & 0x7FFFu) == 0 ? 0 : bits;
        key = (b & 0x8000u) ? uint32_t(0x7FFFu - (b & 0x7FFFu)) : uint32_t(0x8000u + b);
    }
    return (uint64_t(key) << 32) | uint64_t(0xFFFFFFFFu - i);
}
__device__ __forceinline__ uint32_t topk_index(uint64_t r) {
    const uint32_t g = 0xFFFFFFFFu - uint32_t(r);
    return ((g >> 15) << 15) | (((g >> 3) & 3u) << 13) | (((g >> 5) & 1023u) << 3) | (g & 7u);
}
// insert r into the descending list top[0 .. k) (register array: every index below is a compile-time one)
__device__ __forceinline__ void insert_rank(uint64_t (&top)[kTkK], uint64_t r, int k) {
    uint64_t tail = top[0];
#pragma unroll
    for (int q = 1; q < kTkK; ++q)
        if (q == k - 1) tail = top[q];
    if (r <= tail) return;
    int p = k - 1;
#pragma unroll
    for (int q = kTkK - 1; q > 0; --q)
        if (q <= p && top[q - 1] < r) {
            top[q] = top[q - 1];
            p = q - 1;
        }
    // p is the first slot whose predecessor is >= r (or 0)
#pragma unroll
    for (int q = 0; q < kTkK; ++q)
        if (q == p) top[q] = r;
}
// merge the sorted (descending) lists at a and b, keep the k best at a
__device__ __forceinline__ void merge_lists(uint64_t* lst, int a, int b, int k) {
    uint64_t out[kTkK];
    int i = 0, j = 0;
#pragma unroll
    for (int o = 0; o < kTkK; ++o) {
        if (o < k) {
            const uint64_t x = lst[a + i], y = lst[b + j];
            if (x >= y) {
                out[o] = x;
                ++i;
            } else {
                out[o] = y;
                ++j;
            }
        }
    }
#pragma unroll
    for (int o = 0; o < kTkK; ++o)
        if (o < k) lst[a + o] = out[o];
}


}  // namespace mono
