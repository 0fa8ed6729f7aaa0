// Exact top-k (k <= 8) and argmax over bf16 logit rows (the role of csrc/fast_topk.sycl:22-176; used by the
// greedy verify / draft picks). Every element gets a 64-bit rank, larger = better:
//   top-k   high half: the bf16 radix key (NaN on top, -0 below +0); low half: ~(the XPU topk gather key)
//           (i >> 15) << 15 | ((i & 8191) >> 3) << 5 | ((i & 32767) >> 13) << 3 | (i & 7), so ties come out in
//           the order of the reference's torch topk
//   argmax  high half: the float order key (NaN largest, -0 == +0); low half: ~i (smallest index on ties)
// Kernel 1, CTA = (row, slice of 128): each thread reads its elements 8 at a time (16-byte loads, all of them
// issued before the first is ranked) and keeps its k best ranks sorted in registers, the CTA merges the 256 lists
// pairwise in shared memory and writes its list (and argmax best) to the workspace. Kernel 2, CTA = row: merges
// the slices' lists and inverts the ranks to indices. Integer work: bit-exact.
#include "launch.h"

namespace mono {

constexpr int kTkK = 8, kTkThreads = 256, kTkSlices = 128;

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
__device__ __forceinline__ void insert_rank(uint64_t (&top)[kTkK], uint64_t r, int k) {
    if (r <= top[k - 1]) return;
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

__global__ void __launch_bounds__(kTkThreads) topk_partial_kernel(const TopkArgs A) {
    __shared__ uint64_t lst[kTkThreads * kTkK];
    __shared__ uint64_t amb[kTkThreads / 32];
    const int t = threadIdx.x, slice = blockIdx.x, row = blockIdx.y;
    // slices of a multiple of 8 elements, so 16-byte pieces never straddle two slices
    const int64_t per = ((A.V + kTkSlices - 1) / kTkSlices + 7) / 8 * 8, c0 = slice * per,
                  c1 = c0 + per < A.V ? c0 + per : A.V;
    const uint16_t* x = A.x + size_t(row) * A.V;
    uint64_t top[kTkK];
#pragma unroll
    for (int j = 0; j < kTkK; ++j) top[j] = 0;
    uint64_t best = 0;
    auto take = [&](uint16_t b, uint32_t i) {
        insert_rank(top, A.argmax_order ? rank_argmax(b, i) : rank_topk(b, i), A.k);
        if (A.with_argmax) best = max(best, rank_argmax(b, i));
    };
    const bool vec = (A.V & 7) == 0 && (reinterpret_cast<uintptr_t>(A.x) & 15) == 0;
    if (vec) {
        constexpr int kMaxPieces = 4;  // pieces per thread loaded together
        for (int64_t base = c0 / 8 + t; base * 8 < c1; base += int64_t(kTkThreads) * kMaxPieces) {
            uint4 v[kMaxPieces];
#pragma unroll
            for (int p = 0; p < kMaxPieces; ++p)
                if ((base + int64_t(kTkThreads) * p) * 8 < c1) v[p] = __ldg(reinterpret_cast<const uint4*>(x) + base + kTkThreads * p);
#pragma unroll
            for (int p = 0; p < kMaxPieces; ++p) {
                const int64_t e0 = (base + int64_t(kTkThreads) * p) * 8;
                if (e0 < c1) {
                    const uint32_t u[4] = {v[p].x, v[p].y, v[p].z, v[p].w};
#pragma unroll
                    for (int e = 0; e < 8; ++e) take(uint16_t((e & 1) ? (u[e >> 1] >> 16) : (u[e >> 1] & 0xFFFFu)), uint32_t(e0 + e));
                }
            }
        }
    } else {
        for (int64_t i = c0 + t; i < c1; i += kTkThreads) take(x[i], uint32_t(i));
    }
#pragma unroll
    for (int j = 0; j < kTkK; ++j) lst[t * kTkK + j] = top[j];
    if (A.with_argmax) {
#pragma unroll
        for (int o = 16; o; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
        if ((t & 31) == 0) amb[t >> 5] = best;
    }
    __syncthreads();
    for (int n = kTkThreads / 2; n >= 1; n >>= 1) {
        if (t < n) merge_lists(lst, t * kTkK, (t + n) * kTkK, A.k);
        __syncthreads();
    }
    uint64_t* part = A.ws + (size_t(row) * kTkSlices + slice) * (kTkK + 1);
    if (t < kTkK) part[t] = lst[t];
    if (t == 0) {
        uint64_t b = 0;
        for (int w = 0; w < kTkThreads / 32; ++w) b = max(b, amb[w]);
        part[kTkK] = A.with_argmax ? b : 0;
    }
}

__global__ void __launch_bounds__(kTkSlices) topk_final_kernel(const TopkArgs A) {
    __shared__ uint64_t lst[kTkSlices * kTkK];
    __shared__ uint64_t amb[kTkSlices / 32];
    const int t = threadIdx.x, row = blockIdx.x;
    const uint64_t* part = A.ws + size_t(row) * kTkSlices * (kTkK + 1);
#pragma unroll
    for (int j = 0; j < kTkK; ++j) lst[t * kTkK + j] = part[t * (kTkK + 1) + j];
    uint64_t best = A.with_argmax ? part[t * (kTkK + 1) + kTkK] : 0;
#pragma unroll
    for (int o = 16; o; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
    if ((t & 31) == 0) amb[t >> 5] = best;
    __syncthreads();
    for (int n = kTkSlices / 2; n >= 1; n >>= 1) {
        if (t < n) merge_lists(lst, t * kTkK, (t + n) * kTkK, A.k);
        __syncthreads();
    }
    if (t < A.k) {
        const uint64_t r = lst[t];
        const uint32_t i = A.argmax_order ? 0xFFFFFFFFu - uint32_t(r) : topk_index(r);
        A.indices[size_t(row) * A.k + t] = int64_t(i);
        A.values[size_t(row) * A.k + t] = A.x[size_t(row) * A.V + i];
    }
    if (t == 0 && A.with_argmax) {
        uint64_t b = 0;
        for (int w = 0; w < kTkSlices / 32; ++w) b = max(b, amb[w]);
        A.argmax[row] = int64_t(0xFFFFFFFFu - uint32_t(b));
    }
}

size_t topk_workspace_bytes(int64_t rows) { return size_t(rows) * kTkSlices * (kTkK + 1) * 8; }

int launch_topk(const TopkArgs& A, cudaStream_t stream) {
    topk_partial_kernel<<<dim3(kTkSlices, A.rows), kTkThreads, 0, stream>>>(A);
    CUDA_TRY(cudaGetLastError());
    topk_final_kernel<<<A.rows, kTkSlices, 0, stream>>>(A);
    CUDA_TRY(cudaGetLastError());
    return MONO_OK;
}

}  // namespace mono
