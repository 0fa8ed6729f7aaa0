// W4A8 weight preparation: the tile-major repack and the REF pair table; the device error word.
#include <cstdio>
#include <mutex>

#include "abi_internal.h"
#include "engine.cuh"

namespace mono {

__device__ int g_device_error = 0;  // declared in common.cuh

// ---- tile-major repack ------------------------------------------------------------------------------
// q:  row-major [N][K/2] bytes -> [N/16][K/128][2][32][16]: 16-byte piece (half h, lane 4 g + t) of the
//     (tile, group) block is row 16 tile + g + 8 h, bytes [64 group + 16 t, +16). GPTQ nibbles v + 8 are
//     stored as two's complement (XOR 8) so the GEMV unpacks them with one mask.
__global__ void repack_q_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int N, int K,
                                uint32_t xor_mask) {
    const int G = K >> 7;
    const int64_t pieces = int64_t(N / 16) * G * 64;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < pieces; i += int64_t(gridDim.x) * blockDim.x) {
        const int piece = int(i & 63);
        const int64_t blk = i >> 6;  // tile * G + group
        const int tile = int(blk / G), grp = int(blk - int64_t(tile) * G);
        const int h = piece >> 5, lane = piece & 31, g = lane >> 2, t = lane & 3;
        const int row = tile * 16 + g + 8 * h;
        uint4 v = *reinterpret_cast<const uint4*>(src + int64_t(row) * (K / 2) + grp * 64 + t * 16);
        v.x ^= xor_mask; v.y ^= xor_mask; v.z ^= xor_mask; v.w ^= xor_mask;
        *reinterpret_cast<uint4*>(dst + i * 16) = v;
    }
}

// scales: GPTQ fp16 [N][K/128] -> [N/16][K/256][16][2]; REF fp8 [N][K/16] -> [N/16][K/256][16][16]
__global__ void repack_s_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int N, int K, int fmt) {
    const int pairs = K >> 8;                 // 256-wide group pairs per row
    const int eb = fmt == FMT_GPTQ ? 4 : 16;  // bytes per (row, pair)
    const int64_t items = int64_t(N) * pairs;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < items; i += int64_t(gridDim.x) * blockDim.x) {
        const int row = int(i / pairs), pr = int(i - int64_t(row) * pairs);
        const uint8_t* s = src + int64_t(row) * pairs * eb + int64_t(pr) * eb;
        uint8_t* d = dst + ((int64_t(row >> 4) * pairs + pr) * 16 + (row & 15)) * eb;
        for (int b = 0; b < eb; ++b) d[b] = s[b];
    }
}

// REF pair table: entry (s << 8 | byte) = int8 grid values of the byte's low and high code at FP8 scale s,
// by the reference decode (w4a8_decode.sycl:35-45): r = rint(cb[code] * scale); isnan(r) ? 0 : clamp.
__device__ __forceinline__ uint32_t ref_grid(float c, float scale) {
    const float r = rintf(__fmul_rn(c, scale));
    if (isnan(r)) return 0;
    return uint32_t(int(fminf(fmaxf(r, -127.f), 127.f))) & 0xFF;
}
__global__ void pair_table_kernel(const float* __restrict__ cb, uint16_t* __restrict__ tab) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= 65536) return;
    const int byte = i & 255;
    const float scale = fp8e4m3_to_f32(uint8_t(i >> 8));
    const float lo = cb ? cb[byte & 15] : float((byte & 15) - 8), hi = cb ? cb[byte >> 4] : float((byte >> 4) - 8);
    tab[i] = uint16_t(ref_grid(lo, scale) | (ref_grid(hi, scale) << 8));
}

int launch_repack(int fmt, const void* q, const void* s, int N, int K, void* qt, void* st, cudaStream_t stream) {
    const int64_t pieces = int64_t(N / 16) * (K / 128) * 64;
    const int blocks = int((pieces + 255) / 256 < 4096 ? (pieces + 255) / 256 : 4096);
    repack_q_kernel<<<blocks, 256, 0, stream>>>(static_cast<const uint8_t*>(q), static_cast<uint8_t*>(qt), N, K,
                                                fmt == FMT_GPTQ ? 0x88888888u : 0u);
    CUDA_TRY(cudaGetLastError());
    const int64_t items = int64_t(N) * (K / 256);
    const int sblocks = int((items + 255) / 256 < 4096 ? (items + 255) / 256 : 4096);
    repack_s_kernel<<<sblocks, 256, 0, stream>>>(static_cast<const uint8_t*>(s), static_cast<uint8_t*>(st), N, K, fmt);
    CUDA_TRY(cudaGetLastError());
    return MONO_OK;
}

int launch_pair_table(const float* codebook, uint16_t* tab, cudaStream_t stream) {
    pair_table_kernel<<<256, 256, 0, stream>>>(codebook, tab);
    CUDA_TRY(cudaGetLastError());
    return MONO_OK;
}

}  // namespace mono
