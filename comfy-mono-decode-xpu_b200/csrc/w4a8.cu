// W4A8 weight preparation: the tile-major repack and the REF pair table; the device error word.
#include <cstdio>
#include <mutex>

#include "launch.h"

namespace mono {

__device__ int g_device_error = 0;                   // declared in common.cuh
__device__ unsigned long long* g_trace = nullptr;  // declared in common.cuh

// ---- tile-major repack ------------------------------------------------------------------------------
// Row-major [N][K/2] weights + scales -> one buffer of items [N/16][K/1024][8192 weight bytes | SB scale
// bytes]: piece (group gi, half h, lane 4 g + t) of an item's weights is row 16 tile + g + 8 h, bytes
// [64 (8 chunk + gi) + 16 t, +16) of that row; the scales follow as [16 rows][8 groups] fp16 (GPTQ) or
// [16 rows][8 groups x 8] fp8 (REF). GPTQ nibbles v + 8 are stored as two's complement (XOR 8) so the
// engine unpacks them with one mask.
__global__ void repack_kernel(const uint8_t* __restrict__ q, const uint8_t* __restrict__ s, uint8_t* __restrict__ dst,
                              int N, int K, int fmt) {
    const int C = K >> 10;
    const int sb = fmt == FMT_GPTQ ? Fmt<FMT_GPTQ>::SB : Fmt<FMT_REF>::SB;
    const int per_unit = (kStageW + sb) >> 4;  // 16-byte pieces per item
    const int64_t pieces = int64_t(N >> 4) * C * per_unit;
    const uint32_t xm = fmt == FMT_GPTQ ? 0x88888888u : 0u;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < pieces; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t unit = i / per_unit;
        const int p = int(i - unit * per_unit);
        const int tile = int(unit / C), chunk = int(unit - int64_t(tile) * C);
        uint4 v;
        if (p < 512) {
            const int gi = p >> 6, r = p & 63, h = r >> 5, lane = r & 31, g = lane >> 2, t = lane & 3;
            const int row = tile * 16 + g + 8 * h;
            v = *reinterpret_cast<const uint4*>(q + int64_t(row) * (K >> 1) + (chunk * 8 + gi) * 64 + t * 16);
            v.x ^= xm; v.y ^= xm; v.z ^= xm; v.w ^= xm;
        } else if (fmt == FMT_GPTQ) {
            const int row = tile * 16 + (p - 512);
            v = *reinterpret_cast<const uint4*>(s + (int64_t(row) * (K >> 7) + chunk * 8) * 2);
        } else {
            const int r = p - 512, row = tile * 16 + (r >> 2), part = r & 3;
            v = *reinterpret_cast<const uint4*>(s + int64_t(row) * (K >> 4) + chunk * 64 + part * 16);
        }
        *reinterpret_cast<uint4*>(dst + i * 16) = v;
    }
}

size_t tiled_bytes(int fmt, int64_t N, int64_t K) {
    const int sb = fmt == FMT_GPTQ ? Fmt<FMT_GPTQ>::SB : Fmt<FMT_REF>::SB;
    return size_t(N / 16) * size_t(K / 1024) * size_t(kStageW + sb);
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

int launch_repack(int fmt, const void* q, const void* s, int N, int K, void* out, cudaStream_t stream) {
    const int64_t pieces = int64_t(tiled_bytes(fmt, N, K) / 16);
    const int blocks = int((pieces + 255) / 256 < 8192 ? (pieces + 255) / 256 : 8192);
    repack_kernel<<<blocks, 256, 0, stream>>>(static_cast<const uint8_t*>(q), static_cast<const uint8_t*>(s),
                                              static_cast<uint8_t*>(out), N, K, fmt);
    CUDA_TRY(cudaGetLastError());
    return MONO_OK;
}

int launch_pair_table(const float* codebook, uint16_t* tab, cudaStream_t stream) {
    pair_table_kernel<<<256, 256, 0, stream>>>(codebook, tab);
    CUDA_TRY(cudaGetLastError());
    return MONO_OK;
}

}  // namespace mono
