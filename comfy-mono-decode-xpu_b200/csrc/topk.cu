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
#include "ranks.cuh"

namespace mono {

constexpr int kTkThreads = 256, kTkSlices = 128;

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
