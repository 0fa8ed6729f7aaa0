// Exact top-k (k <= 64) of a few long rows: the verify step's sampling filter (the role of the reference's
// topk_rows, csrc/topk_rows.sycl:2-17). The result is torch.topk of the rows' fp32 values: per row the k
// largest by the radix key (the fp32 bits with the sign flipped: -0 below +0, no NaN case), sorted descending,
// ties in one of two orders. Each element gets a unique 64-bit rank (larger = earlier in the output):
//   key = bits ^ (sign ? 0xFFFFFFFF : 0x80000000);   rank = key << 32 | (0xFFFFFFFF - g)
//   gather order (ORD 0, the reference platform's torch topk, csrc/topk_rows.sycl:34-42):
//     off = i % 32768;  g = (i / 32768) << 15 | ((off % 4096) / 4) << 5 | (off / 4096) << 2 | off % 4
//   index order (ORD 1): g = i, equal values by ascending index -- torch's CUDA topk order for k >= 33 (and k = 1)
//     as measured on B200 over tie-heavy rows (for 2 <= k <= 32 its order among equal values is its small
//     sorting network's, which no fixed rule reproduces)
// Kernel 1, CTA = (row, slice): each warp keeps the 64 best ranks of its elements sorted in registers (lane l
// holds entries l and 32 + l); an element enters only if it beats the list's last entry, by a warp-wide
// insertion (a ballot counts the entries above it, the rest shift by one lane), or, when 4 or more lanes hold a
// candidate, by a bitonic merge of the whole batch (measured faster than buffering candidates across batches).
// The CTA merges its warps' lists in a tree and writes one list per slice. Kernel 2, one CTA per row: each warp merges a share of the
// slices' lists, the warps' lists meet in a tree, and the first k entries become indices and fp32 values.
// Integer work: bit-exact.
#include <mutex>

#include "launch.h"

namespace mono {

constexpr int kTrK = 64, kTrWarps = 8, kTrThreads = kTrWarps * 32, kTrMaxSlices = 64, kTrMaxRows = 16;

template <int ORD>
__device__ __forceinline__ uint64_t tr_rank(uint32_t bits, uint32_t i) {
    const uint32_t key = bits ^ ((bits & 0x80000000u) ? 0xFFFFFFFFu : 0x80000000u);
    const uint32_t off = i & 32767u;
    const uint32_t g = ORD ? i : ((i >> 15) << 15) | (((off & 4095u) >> 2) << 5) | ((off >> 12) << 2) | (off & 3u);
    return (uint64_t(key) << 32) | uint64_t(0xFFFFFFFFu - g);
}
template <int ORD>
__device__ __forceinline__ uint32_t tr_index(uint64_t r) {
    const uint32_t g = 0xFFFFFFFFu - uint32_t(r);
    return ORD ? g : ((g >> 15) << 15) | (((g >> 2) & 7u) << 12) | (((g >> 5) & 1023u) << 2) | (g & 3u);
}

// The warp's sorted list: L[l] = a (lane l), L[32 + l] = b (lane l), descending.
struct WarpList {
    uint64_t a, b;
    __device__ uint64_t last() const { return __shfl_sync(0xffffffffu, b, 31); }
    // insert rank c (the same on every lane, known to beat last())
    __device__ void insert(uint64_t c, int lane) {
        const int p = __popc(__ballot_sync(0xffffffffu, a > c)) + __popc(__ballot_sync(0xffffffffu, b > c));
        const uint64_t a_up = __shfl_up_sync(0xffffffffu, a, 1), b_up = __shfl_up_sync(0xffffffffu, b, 1);
        const uint64_t a31 = __shfl_sync(0xffffffffu, a, 31);
        const uint64_t na = lane < p ? a : (lane == p ? c : a_up);
        const uint64_t nb = 32 + lane < p ? b : (32 + lane == p ? c : (lane == 0 ? a31 : b_up));
        a = na;
        b = nb;
    }
    // 32 values across the lanes, one per lane, sorted descending (bitonic network)
    __device__ static uint64_t sort32(uint64_t v, int lane) {
#pragma unroll
        for (int k = 2; k <= 32; k <<= 1)
#pragma unroll
            for (int j = k >> 1; j > 0; j >>= 1) {
                const uint64_t p = __shfl_xor_sync(0xffffffffu, v, j);
                const bool keep_max = ((lane & k) == 0) == ((lane & j) == 0);
                v = keep_max ? (v > p ? v : p) : (v < p ? v : p);
            }
        return v;
    }
    // a bitonic sequence of 32 across the lanes, sorted descending
    __device__ static uint64_t merge32(uint64_t v, int lane) {
#pragma unroll
        for (int j = 16; j > 0; j >>= 1) {
            const uint64_t p = __shfl_xor_sync(0xffffffffu, v, j);
            v = (lane & j) == 0 ? (v > p ? v : p) : (v < p ? v : p);
        }
        return v;
    }
    // merge one candidate per lane (0 = none): the new 64 best of A u B u C are A u top32(B u C) (every entry
    // of A beats all of B and at least as many entries of C as it loses to), re-sorted into A, B
    __device__ void merge_batch(uint64_t c, int lane) {
        c = sort32(c, lane);
        const uint64_t cr = __shfl_sync(0xffffffffu, c, 31 - lane);
        const uint64_t d = merge32(b > cr ? b : cr, lane);  // top 32 of B u C
        const uint64_t dr = __shfl_sync(0xffffffffu, d, 31 - lane);
        const uint64_t hi = a > dr ? a : dr, lo = a > dr ? dr : a;
        a = merge32(hi, lane);
        b = merge32(lo, lane);
    }
    // offer one rank per lane
    __device__ void offer(uint64_t r, bool valid, int lane) {
        uint64_t t = last();
        unsigned mask = __ballot_sync(0xffffffffu, valid && r > t);
        if (__popc(mask) >= 4) {  // many candidates: one merge instead of one insertion each
            merge_batch(valid && r > t ? r : 0ull, lane);
            return;
        }
        while (mask) {
            const int j = __ffs(mask) - 1;
            mask &= mask - 1;
            const uint64_t c = __shfl_sync(0xffffffffu, r, j);
            if (c > t) {
                insert(c, lane);
                t = last();
            }
        }
    }
};

template <bool BF16>
__device__ __forceinline__ uint32_t tr_bits_at(const void* x, size_t i) {
    if constexpr (BF16) return uint32_t(__ldg(static_cast<const uint16_t*>(x) + i)) << 16;
    else return __ldg(static_cast<const uint32_t*>(x) + i);
}

template <bool BF16, int ORD>
__global__ void __launch_bounds__(kTrThreads) topk_rows_partial(const void* x, int64_t N, int slices, uint64_t* ws) {
    __shared__ uint64_t lists[kTrWarps][kTrK];
    const int row = blockIdx.y, slice = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t per = (N + slices - 1) / slices, c0 = slice * per, c1 = c0 + per < N ? c0 + per : N;
    const size_t base = size_t(row) * N;
    WarpList L{0, 0};
    // 4 batches of 32 elements per warp per iteration; the next iteration's loads are issued before this one's
    // elements are offered
    const int64_t step = int64_t(kTrWarps) * 128;
    uint32_t bits[4], next[4];
    int64_t b0 = c0 + int64_t(warp) * 128;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int64_t i = b0 + u * 32 + lane;
        next[u] = i < c1 ? tr_bits_at<BF16>(x, base + i) : 0u;
    }
    for (; b0 < c1; b0 += step) {
#pragma unroll
        for (int u = 0; u < 4; ++u) bits[u] = next[u];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t i = b0 + step + u * 32 + lane;
            next[u] = i < c1 ? tr_bits_at<BF16>(x, base + i) : 0u;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t i = b0 + u * 32 + lane;
            L.offer(tr_rank<ORD>(bits[u], uint32_t(i)), i < c1, lane);
        }
    }
    lists[warp][lane] = L.a;
    lists[warp][32 + lane] = L.b;
    // tree merge: at level d, warp w (a multiple of 2d) takes in warp w + d's list
    for (int d = 1; d < kTrWarps; d *= 2) {
        __syncthreads();
        if (warp % (2 * d) == 0) {
            uint64_t t = L.last();
            for (int j = 0; j < kTrK; ++j) {
                const uint64_t c = lists[warp + d][j];
                if (c <= t) break;  // each list is sorted: the rest cannot enter
                L.insert(c, lane);
                t = L.last();
            }
            lists[warp][lane] = L.a;
            lists[warp][32 + lane] = L.b;
        }
    }
    if (warp == 0) {
        uint64_t* out = ws + (size_t(row) * slices + slice) * kTrK;
        out[lane] = L.a;
        out[32 + lane] = L.b;
    }
}

template <bool BF16, int ORD>
__global__ void __launch_bounds__(kTrThreads) topk_rows_final(const void* x, int64_t N, int slices, int k,
                                                              const uint64_t* ws, float* values, int64_t* indices) {
    __shared__ uint64_t lists[kTrWarps][kTrK];
    const int row = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t* lst = ws + size_t(row) * slices * kTrK;
    // warp w merges slices w, w + 8, ..., then the warps' lists meet in a tree
    WarpList L{0, 0};
    for (int s = warp; s < slices; s += kTrWarps) {
        uint64_t t = L.last();
        for (int j = 0; j < kTrK; ++j) {
            const uint64_t c = lst[size_t(s) * kTrK + j];
            if (c <= t) break;
            L.insert(c, lane);
            t = L.last();
        }
    }
    lists[warp][lane] = L.a;
    lists[warp][32 + lane] = L.b;
    for (int d = 1; d < kTrWarps; d *= 2) {
        __syncthreads();
        if (warp % (2 * d) == 0) {
            uint64_t t = L.last();
            for (int j = 0; j < kTrK; ++j) {
                const uint64_t c = lists[warp + d][j];
                if (c <= t) break;
                L.insert(c, lane);
                t = L.last();
            }
            lists[warp][lane] = L.a;
            lists[warp][32 + lane] = L.b;
        }
    }
    if (warp == 0) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int o = lane + 32 * h;
            if (o < k) {
                const uint32_t i = tr_index<ORD>(h ? L.b : L.a);
                indices[size_t(row) * k + o] = int64_t(i);
                values[size_t(row) * k + o] = __uint_as_float(tr_bits_at<BF16>(x, size_t(row) * N + i));
            }
        }
    }
}

static int topk_rows_slices(int64_t rows, int64_t N) {
    int s = int((2 * int64_t(sm_count()) + rows - 1) / rows);  // about two CTAs per SM over all rows
    s = s < 1 ? 1 : (s > kTrMaxSlices ? kTrMaxSlices : s);
    while (s > 1 && (N + s - 1) / s < kTrK) --s;  // every slice holds at least k elements
    return s;
}

template <bool BF16, int ORD>
int launch_topk_rows(const void* x, int64_t rows, int64_t N, int64_t k, float* values, int64_t* indices,
                            uint64_t* ws, cudaStream_t s) {
    const int slices = topk_rows_slices(rows, N);
    topk_rows_partial<BF16, ORD><<<dim3(slices, unsigned(rows)), kTrThreads, 0, s>>>(x, N, slices, ws);
    CUDA_TRY(cudaGetLastError());
    topk_rows_final<BF16, ORD><<<unsigned(rows), kTrThreads, 0, s>>>(x, N, slices, int(k), ws, values, indices);
    CUDA_TRY(cudaGetLastError());
    return MONO_OK;
}

}  // namespace mono

using namespace mono;

extern "C" {

size_t mono_topk_rows_workspace(int64_t rows, int64_t N) {
    if (rows < 1 || N < 1) return 0;
    return size_t(rows) * topk_rows_slices(rows, N) * kTrK * sizeof(uint64_t);
}

int mono_topk_rows(const void* x, int flags, int64_t rows, int64_t N, int64_t k, float* values, int64_t* indices,
                   void* workspace, size_t workspace_bytes, mono_stream_t stream) {
    MONO_CHECK(x && values && indices && workspace, "null operand");
    MONO_CHECK(rows >= 1 && rows <= kTrMaxRows, "1 <= rows <= %d", kTrMaxRows);
    MONO_CHECK(k >= 1 && k <= kTrK && N >= kTrK && N < (int64_t(1) << 31), "1 <= k <= 64, 64 <= N < 2^31");
    MONO_CHECK(workspace_bytes >= mono_topk_rows_workspace(rows, N) && aligned(workspace, 8),
               "workspace (mono_topk_rows_workspace)");
    MONO_CHECK((flags & ~(MONO_TOPK_BF16 | MONO_TOPK_INDEX_ORDER)) == 0, "flags: MONO_TOPK_BF16 | MONO_TOPK_INDEX_ORDER");
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    uint64_t* ws = static_cast<uint64_t*>(workspace);
    switch (flags) {
        case 0: return launch_topk_rows<false, 0>(x, rows, N, k, values, indices, ws, s);
        case MONO_TOPK_BF16: return launch_topk_rows<true, 0>(x, rows, N, k, values, indices, ws, s);
        case MONO_TOPK_INDEX_ORDER: return launch_topk_rows<false, 1>(x, rows, N, k, values, indices, ws, s);
        default: return launch_topk_rows<true, 1>(x, rows, N, k, values, indices, ws, s);
    }
}

}  // extern "C"
