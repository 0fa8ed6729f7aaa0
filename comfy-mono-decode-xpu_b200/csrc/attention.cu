// Full-attention decode layer pieces: per-head Q/K RMSNorm + partial RoPE + KV cache append, and tree decode
// attention split along the context.
//
// qk_norm_rope_kv (the role of csrc/rope_kv.sycl:120-245): one warp per (row, head); lane l holds head
// elements 8l .. 8l + 7. RMSNorm with this build's pinned order (lane sums of squares in element order, xor
// butterfly 16 8 4 2 1, r = 1 / sqrt(total / 256 + eps), bf16((x * r) * w)); then split-half RoPE on the
// first rd lanes from the normalized bf16 values, each product rounded to fp32 on its own and the sum rounded
// once to bf16 (csrc/rope_kv.sycl:7-9, :46-52). k and v rows are written to the caches at position[s]
// (positions outside [0, cap) are skipped and recorded in the device error word).
//
// Tree attention (the role of csrc/attn_dpas.sycl:269-342): q rows of one kv head (groups x S <= 32) attend
// the committed prefix [0, L) of the bf16 cache plus the tree rows their mask admits.
//   Kernel 1, CTA = (kv head, context chunk): 64-token tiles of K and V staged in shared memory, S = Q K^T and
//   O += P V on the tensor cores (mma.sync m16n8k16 bf16, fp32 accumulation; P rounded to bf16 for P V), an
//   online softmax per row; the chunk's unnormalized O, running max and sum go to the workspace.
//   Kernel 2, CTA = (q head, row): merge of the active chunks and of the admitted tree rows (fp32 scores over
//   the head dimension), one bf16 rounding of the output.
// Chunks follow the actual length L read on the device: per = max(ceil(L / chunks), 64) tokens rounded up to
// the tile, active = ceil(L / per); CTAs past the last active chunk exit.
#include <cmath>
#include <mutex>

#include "launch.h"

namespace mono {

constexpr int kHD = 256;

// ---- qk_norm_rope_kv ---------------------------------------------------------------------------------


__global__ void __launch_bounds__(32) qk_norm_rope_kv_kernel(const NormRopeArgs A) {
    __shared__ __align__(16) uint16_t nrm[kHD];
    const int lane = threadIdx.x;
    const int s = blockIdx.x / (A.Hq + 2 * A.Hk), h = blockIdx.x % (A.Hq + 2 * A.Hk);
    const int64_t p = A.pos[s];
    const bool pos_ok = p >= 0 && p < A.cap;
    if (!pos_ok && lane == 0) set_device_error(DEV_BAD_POSITION);
    if (h >= A.Hq + A.Hk) {  // v: cache write only
        const int hv = h - A.Hq - A.Hk;
        if (pos_ok)
            reinterpret_cast<uint4*>(A.vc + (size_t(hv) * A.cap + p) * kHD)[lane] =
                reinterpret_cast<const uint4*>(A.v + size_t(s) * A.vs + size_t(hv) * kHD)[lane];
        return;
    }
    const bool isq = h < A.Hq;
    const int hh = isq ? h : h - A.Hq;
    const uint16_t* src = isq ? A.q + size_t(s) * A.qs + size_t(hh) * A.qh : A.k + size_t(s) * A.ks + size_t(hh) * kHD;
    const uint16_t* w = isq ? A.wq : A.wk;
    const uint4 xv = reinterpret_cast<const uint4*>(src)[lane];
    const uint4 wv = reinterpret_cast<const uint4*>(w)[lane];
    const uint32_t xu[4] = {xv.x, xv.y, xv.z, xv.w}, wu[4] = {wv.x, wv.y, wv.z, wv.w};
    float x[8];
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        x[e] = __uint_as_float((e & 1) ? (xu[e >> 1] & 0xFFFF0000u) : (xu[e >> 1] << 16));
        ss = __fadd_rn(ss, __fmul_rn(x[e], x[e]));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    const float r = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, float(kHD)), isq ? A.epsq : A.epsk)));
    uint32_t nu[4] = {0, 0, 0, 0};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const float wf = __uint_as_float((e & 1) ? (wu[e >> 1] & 0xFFFF0000u) : (wu[e >> 1] << 16));
        nu[e >> 1] |= uint32_t(f32_to_bf16_bits(__fmul_rn(__fmul_rn(x[e], r), wf))) << (16 * (e & 1));
    }
    reinterpret_cast<uint4*>(nrm)[lane] = make_uint4(nu[0], nu[1], nu[2], nu[3]);
    __syncwarp();
    const int half = A.rd >> 1;
    uint32_t ou[4] = {0, 0, 0, 0};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const int d = lane * 8 + e;
        uint16_t res = nrm[d];
        if (d < A.rd) {
            const int j = d < half ? d : d - half;
            const float* f = A.freqs + (size_t(s) * half + j) * 4;  // [[f00, f01], [f10, f11]]
            const float lo = bf16_bits_to_f32(nrm[j]), hi = bf16_bits_to_f32(nrm[j + half]);
            const float o = d < half ? __fadd_rn(__fmul_rn(lo, f[0]), __fmul_rn(hi, f[1]))
                                     : __fadd_rn(__fmul_rn(hi, f[3]), __fmul_rn(lo, f[2]));
            res = f32_to_bf16_bits(o);
        }
        ou[e >> 1] |= uint32_t(res) << (16 * (e & 1));
    }
    const uint4 out = make_uint4(ou[0], ou[1], ou[2], ou[3]);
    if (isq) {
        reinterpret_cast<uint4*>(A.oq + (size_t(hh) * A.S + s) * kHD)[lane] = out;
    } else {
        reinterpret_cast<uint4*>(A.ok + (size_t(hh) * A.S + s) * kHD)[lane] = out;
        if (pos_ok) reinterpret_cast<uint4*>(A.kc + (size_t(hh) * A.cap + p) * kHD)[lane] = out;
    }
}

int launch_qk_norm_rope_kv(const NormRopeArgs& A, cudaStream_t stream) {
    qk_norm_rope_kv_kernel<<<A.S * (A.Hq + 2 * A.Hk), 32, 0, stream>>>(A);
    CUDA_TRY(cudaGetLastError());
    return MONO_OK;
}

// ---- tree attention ------------------------------------------------------------------------------------

constexpr int kAttTile = 64;              // tokens per K / V tile
constexpr int kAttRows = 32;              // q rows per kv head (groups x S), padded
constexpr int kQPitch = kHD + 8;          // bf16 elements per staged row (16-byte skew: conflict-free ldmatrix)
constexpr int kPPitch = kAttTile + 8;
constexpr int kAttThreads = 128;


__device__ __forceinline__ void attn_chunking(int L, int chunks, int& per, int& active) {
    per = (L + chunks - 1) / chunks;
    per = per < kAttTile ? kAttTile : per;
    per = (per + kAttTile - 1) / kAttTile * kAttTile;
    active = L > 0 ? (L + per - 1) / per : 0;
}
__device__ __forceinline__ int clamp_len(int raw, int cap) { return raw < 0 ? 0 : (raw > cap ? cap : raw); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__global__ void __launch_bounds__(kAttThreads) attn_partial_kernel(const AttnArgs A) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint16_t* Qs = reinterpret_cast<uint16_t*>(smem);               // [32][kQPitch]
    uint16_t* Ks = Qs + kAttRows * kQPitch;                         // [64][kQPitch]
    uint16_t* Vs = Ks + kAttTile * kQPitch;                         // [64][kQPitch]
    uint16_t* Ps = Vs + kAttTile * kQPitch;                         // [32][kPPitch]
    float* red = reinterpret_cast<float*>(Ps + kAttRows * kPPitch);  // [4 warps][32 rows]
    const int chunk = blockIdx.x, kh = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int L = clamp_len(A.seqlen[0], A.cap);
    int per, active;
    attn_chunking(L, A.chunks, per, active);
    if (chunk >= active) return;
    const int groups = A.H / A.Hk, R = groups * A.S;
    const int t0 = chunk * per, t1 = (t0 + per < L) ? t0 + per : L;
    // Q rows r = gi * S + s of q head kh * groups + gi; rows >= R are zero
    for (int i = tid; i < kAttRows * (kHD / 8); i += kAttThreads) {
        const int r = i / (kHD / 8), c = i % (kHD / 8);
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < R) {
            const int gi = r / A.S, s = r % A.S;
            v = reinterpret_cast<const uint4*>(A.q + (size_t(kh * groups + gi) * A.S + s) * kHD)[c];
        }
        reinterpret_cast<uint4*>(Qs + r * kQPitch)[c] = v;
    }
    float O[2][8][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) O[mt][nt][i] = 0.f;
    // running max / sum of the rows this thread's fragments touch: rows g, g + 8 (m-tile 0), g + 16, g + 24
    float mrun[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY}, lrun[4] = {0.f, 0.f, 0.f, 0.f};
    const uint16_t* kbase = A.kc + size_t(kh) * A.cap * kHD;
    const uint16_t* vbase = A.vc + size_t(kh) * A.cap * kHD;
    for (int tt = t0; tt < t1; tt += kAttTile) {
        const int nvalid = (t1 - tt) < kAttTile ? (t1 - tt) : kAttTile;
        __syncthreads();  // the previous tile's K / V / P reads are done
        for (int i = tid; i < kAttTile * (kHD / 8); i += kAttThreads) {
            const int r = i / (kHD / 8), c = i % (kHD / 8);
            if (r < nvalid) {
                cp_async16(Ks + r * kQPitch + c * 8, kbase + size_t(tt + r) * kHD + c * 8);
                cp_async16(Vs + r * kQPitch + c * 8, vbase + size_t(tt + r) * kHD + c * 8);
            } else {
                reinterpret_cast<uint4*>(Ks + r * kQPitch)[c] = make_uint4(0, 0, 0, 0);
                reinterpret_cast<uint4*>(Vs + r * kQPitch)[c] = make_uint4(0, 0, 0, 0);
            }
        }
        cp_async_commit();
        cp_async_wait<0>();
        __syncthreads();
        // S = Q K^T for tokens [16 warp, 16 warp + 16) of the tile, all 32 rows
        float Sc[2][2][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int i = 0; i < 4; ++i) Sc[mt][nt][i] = 0.f;
#pragma unroll 4
        for (int kk = 0; kk < kHD; kk += 16) {
            uint32_t b[4];  // n-tile 0: b[0], b[1]; n-tile 1: b[2], b[3]
            ldsm_x4(b, Ks + (warp * 16 + (lane & 7) + 8 * (lane >> 4)) * kQPitch + kk + 8 * ((lane >> 3) & 1));
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
                uint32_t a[4];
                ldsm_x4(a, Qs + (mt * 16 + (lane & 7) + 8 * ((lane >> 3) & 1)) * kQPitch + kk + 8 * (lane >> 4));
                mma_bf16(Sc[mt][0], a, b[0], b[1]);
                mma_bf16(Sc[mt][1], a, b[2], b[3]);
            }
        }
        // scale, mask the tokens past the chunk, per-row tile maxima across the 4 warps
        float tmax[4];
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) tmax[rr] = -INFINITY;
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int col = warp * 16 + nt * 8 + 2 * t + (i & 1);
                    float v = Sc[mt][nt][i] * 0.0625f;
                    if (col >= nvalid) v = -INFINITY;
                    Sc[mt][nt][i] = v;
                    const int rr = mt * 2 + (i >> 1);
                    tmax[rr] = fmaxf(tmax[rr], v);
                }
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
            tmax[rr] = fmaxf(tmax[rr], __shfl_xor_sync(0xffffffffu, tmax[rr], 1));
            tmax[rr] = fmaxf(tmax[rr], __shfl_xor_sync(0xffffffffu, tmax[rr], 2));
            if (t == 0) red[warp * 32 + (rr >> 1) * 16 + (rr & 1) * 8 + g] = tmax[rr];
        }
        __syncthreads();
        float mnew[4], scale_old[4];
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
            const int row = (rr >> 1) * 16 + (rr & 1) * 8 + g;
            float m = mrun[rr];
            for (int w = 0; w < 4; ++w) m = fmaxf(m, red[w * 32 + row]);
            mnew[rr] = m;
            scale_old[rr] = mrun[rr] == -INFINITY ? 0.f : expf(mrun[rr] - m);
            mrun[rr] = m;
        }
        // P = exp(S - m) (bf16 into shared memory); this warp's share of the row sums
        float psum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
                uint32_t pk[2];
#pragma unroll
                for (int hi = 0; hi < 2; ++hi) {
                    const int rr = mt * 2 + hi;
                    const float p0 = Sc[mt][nt][2 * hi] == -INFINITY ? 0.f : expf(Sc[mt][nt][2 * hi] - mnew[rr]);
                    const float p1 = Sc[mt][nt][2 * hi + 1] == -INFINITY ? 0.f : expf(Sc[mt][nt][2 * hi + 1] - mnew[rr]);
                    const uint16_t b0 = f32_to_bf16_bits(p0), b1 = f32_to_bf16_bits(p1);
                    psum[rr] += bf16_bits_to_f32(b0) + bf16_bits_to_f32(b1);
                    pk[hi] = uint32_t(b0) | (uint32_t(b1) << 16);
                }
                const int col = warp * 16 + nt * 8 + 2 * t;
                *reinterpret_cast<uint32_t*>(Ps + (mt * 16 + g) * kPPitch + col) = pk[0];
                *reinterpret_cast<uint32_t*>(Ps + (mt * 16 + 8 + g) * kPPitch + col) = pk[1];
            }
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
            psum[rr] += __shfl_xor_sync(0xffffffffu, psum[rr], 1);
            psum[rr] += __shfl_xor_sync(0xffffffffu, psum[rr], 2);
        }
        __syncthreads();  // every warp has read red (maxima) and written its P columns
        if (t == 0)
#pragma unroll
            for (int rr = 0; rr < 4; ++rr) red[warp * 32 + (rr >> 1) * 16 + (rr & 1) * 8 + g] = psum[rr];
        // rescale O and add P V for dims [64 warp, 64 warp + 64)
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
                O[mt][nt][0] *= scale_old[mt * 2];
                O[mt][nt][1] *= scale_old[mt * 2];
                O[mt][nt][2] *= scale_old[mt * 2 + 1];
                O[mt][nt][3] *= scale_old[mt * 2 + 1];
            }
#pragma unroll
        for (int kk = 0; kk < kAttTile; kk += 16) {
            uint32_t a[2][4];
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
                ldsm_x4(a[mt], Ps + (mt * 16 + (lane & 7) + 8 * ((lane >> 3) & 1)) * kPPitch + kk + 8 * (lane >> 4));
#pragma unroll
            for (int np = 0; np < 4; ++np) {  // pairs of 8-dim n-tiles
                uint32_t b[4];
                ldsm_x4_t(b, Vs + (kk + (lane & 7) + 8 * ((lane >> 3) & 1)) * kQPitch + warp * 64 + np * 16 + 8 * (lane >> 4));
#pragma unroll
                for (int mt = 0; mt < 2; ++mt) {
                    mma_bf16(O[mt][2 * np], a[mt], b[0], b[1]);
                    mma_bf16(O[mt][2 * np + 1], a[mt], b[2], b[3]);
                }
            }
        }
        __syncthreads();
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
            const int row = (rr >> 1) * 16 + (rr & 1) * 8 + g;
            float sum = 0.f;
            for (int w = 0; w < 4; ++w) sum += red[w * 32 + row];
            lrun[rr] = lrun[rr] * scale_old[rr] + sum;
        }
    }
    // the chunk's unnormalized O, max and sum
    const size_t unit = size_t(kh) * A.chunks + chunk;
    float* po = A.part + unit * kAttRows * kHD;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            const int col = warp * 64 + nt * 8 + 2 * t;
            *reinterpret_cast<float2*>(po + (mt * 16 + g) * kHD + col) = make_float2(O[mt][nt][0], O[mt][nt][1]);
            *reinterpret_cast<float2*>(po + (mt * 16 + 8 + g) * kHD + col) = make_float2(O[mt][nt][2], O[mt][nt][3]);
        }
    if (warp == 0 && t == 0)
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
            const int row = (rr >> 1) * 16 + (rr & 1) * 8 + g;
            A.ml[(unit * kAttRows + row) * 2] = mrun[rr];
            A.ml[(unit * kAttRows + row) * 2 + 1] = lrun[rr];
        }
}

// CTA = (q head h, row s), thread = head dim d.
__global__ void __launch_bounds__(kHD) attn_merge_kernel(const AttnArgs A) {
    __shared__ float red[kHD / 32];
    const int d = threadIdx.x, h = blockIdx.x / A.S, s = blockIdx.x % A.S;
    const int groups = A.H / A.Hk, kh = h / groups, r = (h % groups) * A.S + s;
    const int L = clamp_len(A.seqlen[0], A.cap);
    int per, active;
    attn_chunking(L, A.chunks, per, active);
    float M = -INFINITY;
    for (int c = 0; c < active; ++c) M = fmaxf(M, A.ml[((size_t(kh) * A.chunks + c) * kAttRows + r) * 2]);
    float acc = 0.f, sum = 0.f;
    for (int c = 0; c < active; ++c) {
        const size_t u = (size_t(kh) * A.chunks + c) * kAttRows + r;
        const float w = expf(A.ml[u * 2] - M);
        sum += A.ml[u * 2 + 1] * w;
        acc += A.part[u * kHD + d] * w;
    }
    if (A.mask != nullptr) {
        const int mk = A.mask[s];
        const float qd = bf16_bits_to_f32(A.q[(size_t(h) * A.S + s) * kHD + d]);
        for (int tr = 0; tr < A.S; ++tr) {
            if (!((mk >> tr) & 1)) continue;
            float v = qd * bf16_bits_to_f32(A.xk[(size_t(kh) * A.S + tr) * kHD + d]);
#pragma unroll
            for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            __syncthreads();
            if ((d & 31) == 0) red[d >> 5] = v;
            __syncthreads();
            float sc = 0.f;
#pragma unroll
            for (int w = 0; w < kHD / 32; ++w) sc += red[w];
            sc *= 0.0625f;
            const float M2 = fmaxf(M, sc);
            const float fp = M == -INFINITY ? 0.f : expf(M - M2), ft = expf(sc - M2);
            acc = acc * fp + ft * bf16_bits_to_f32(A.xv[(size_t(kh) * A.S + tr) * kHD + d]);
            sum = sum * fp + ft;
            M = M2;
        }
    }
    A.out[(size_t(s) * A.H + h) * kHD + d] = f32_to_bf16_bits(sum > 0.f ? acc / sum : 0.f);
}

size_t attn_smem_bytes() {
    return size_t(kAttRows + 2 * kAttTile) * kQPitch * 2 + size_t(kAttRows) * kPPitch * 2 + 4 * 32 * 4;
}
int attn_chunks(int Hk, int cap, int sms) {
    // about two CTAs per SM at the longest context the cache holds, at least one tile per chunk
    int chunks = (2 * sms + Hk - 1) / Hk;
    const int tiles = (cap + kAttTile - 1) / kAttTile;
    return chunks < tiles ? chunks : (tiles > 0 ? tiles : 1);
}
size_t attn_workspace_bytes(int Hk, int cap, int sms) {
    const size_t chunks = attn_chunks(Hk, cap, sms);
    return size_t(Hk) * chunks * kAttRows * (kHD + 2) * 4;
}

int launch_tree_attention(AttnArgs A, void* ws, cudaStream_t stream) {
    A.chunks = attn_chunks(A.Hk, A.cap, sm_count());
    A.part = static_cast<float*>(ws);
    A.ml = A.part + size_t(A.Hk) * A.chunks * kAttRows * kHD;
    const size_t smem = attn_smem_bytes();
    static std::once_flag once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(once, [&] {
        attr_err = cudaFuncSetAttribute(attn_partial_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    });
    CUDA_TRY(attr_err);
    attn_partial_kernel<<<dim3(A.chunks, A.Hk), kAttThreads, smem, stream>>>(A);
    CUDA_TRY(cudaGetLastError());
    attn_merge_kernel<<<A.H * A.S, kHD, 0, stream>>>(A);
    CUDA_TRY(cudaGetLastError());
    return MONO_OK;
}

}  // namespace mono
