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
// the committed prefix [0, L) of the bf16 cache plus the tree rows their mask admits. One launch:
//   CTA = (kv head, context chunk), chunks in clusters of 8 CTAs: 64-token tiles of K and V staged in shared
//   memory, S = Q K^T and O += P V on the tensor cores (mma.sync m16n8k16 bf16, fp32 accumulation; P rounded to
//   bf16 for P V), an online softmax per row; the chunk's unnormalized O, running max and sum stay in the CTA's
//   shared memory.
//   Cluster merge: after a cluster barrier, warp w of cluster rank j merges row 4 j + w over the 8 chunks of
//   the cluster, reading the peers' shared memory (rank order; fp32).
//   Cross-cluster merge (only when the context spans more than one cluster): each cluster writes its merged
//   rows to the workspace; per (kv head, rank) the last arriving CTA merges the clusters in cluster order.
//   The merged row then takes the admitted tree rows (fp32 scores over the head dimension) and is rounded
//   once to bf16.
// Chunks follow the actual length L read on the device: per = max(ceil(L / chunks), 64) tokens rounded up to
// the tile, active = ceil(L / per); clusters past the last active chunk exit at once, inactive chunks of a
// live cluster contribute an empty partial.
#include <cooperative_groups.h>

#include <cmath>
#include <mutex>

#include "launch.h"

namespace mono {

namespace cg = cooperative_groups;

constexpr int kHD = 256;

// ---- qk_norm_rope_kv ---------------------------------------------------------------------------------


__global__ void __launch_bounds__(32) qk_norm_rope_kv_kernel(const NormRopeArgs A) {
    __shared__ __align__(16) uint16_t nrm[kHD];
    pdl_launch_dependents();  // an ordinary launch (its inputs are complete): the attention may launch at once
    const int lane = threadIdx.x;
    const int s = blockIdx.x / (A.Hq + 2 * A.Hk), h = blockIdx.x % (A.Hq + 2 * A.Hk);
    // batched streams: rows [b R, (b + 1) R) are stream b's, its caches are kv heads [b Hk, (b + 1) Hk)
    const int R = A.S / A.streams, b = s / R, sr = s % R;
    const int64_t p = A.pos[s];
    const bool pos_ok = p >= 0 && p < A.cap;
    if (!pos_ok && lane == 0) set_device_error(DEV_BAD_POSITION);
    if (h >= A.Hq + A.Hk) {  // v: cache write only
        const int hv = h - A.Hq - A.Hk;
        if (pos_ok)
            reinterpret_cast<uint4*>(A.vc + (size_t(b * A.Hk + hv) * A.cap + p) * kHD)[lane] =
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
        reinterpret_cast<uint4*>(A.oq + (size_t(b * A.Hq + hh) * R + sr) * kHD)[lane] = out;
    } else {
        reinterpret_cast<uint4*>(A.ok + (size_t(b * A.Hk + hh) * R + sr) * kHD)[lane] = out;
        if (pos_ok) reinterpret_cast<uint4*>(A.kc + (size_t(b * A.Hk + hh) * A.cap + p) * kHD)[lane] = out;
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
constexpr int kAttCluster = 8;            // chunk CTAs per cluster; 4 warps x 8 CTAs = the 32 rows
constexpr int kOPitch = kHD + 8;          // fp32 elements per row of a CTA's partial O in shared memory

__device__ __forceinline__ void cluster_arrive_release() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
// the shared::cluster address of p (this CTA's shared memory) in cluster CTA `rank`, and loads from it
__device__ __forceinline__ uint32_t cluster_addr(const void* p, int rank) {
    uint32_t a;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
    return a;
}
__device__ __forceinline__ float4 ld_cluster_v4(uint32_t a) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ float2 ld_cluster_v2(uint32_t a) {
    float2 v;
    asm volatile("ld.shared::cluster.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ void prefetch_l2(const void* p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

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

__device__ __forceinline__ void unpack8(const uint4 v, float (&f)[8]) {
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        f[2 * j] = __uint_as_float(u[j] << 16);
        f[2 * j + 1] = __uint_as_float(u[j] & 0xFFFF0000u);
    }
}

// The tree value row t of kv head kh (of all streams' heads), as strided by the caller.
__device__ __forceinline__ const uint16_t* attn_xv_row(const AttnArgs& A, int kh, int t) {
    const int hs = A.Hk / A.streams;
    return A.xv + size_t(kh / hs) * A.xv_bs + size_t(kh % hs) * A.xv_hs + size_t(t) * A.xv_rs;
}

// One warp finishes row r of kv head kh (q head kh * groups + r / S, tree row r % S); lane l holds dims
// [8 l, 8 l + 8) of the merged prefix (acc unnormalized, running max M, sum). The admitted tree rows follow in
// row order (score = q . xk / 16 over the head dimension: lane sums in dim order, xor butterfly 16 .. 1), then
// out = bf16(acc / sum).
__device__ __forceinline__ void attn_finish_row(const AttnArgs& A, int kh, int r, int lane, float (&acc)[8], float M,
                                                float sum) {
    const int groups = A.H / A.Hk, h = kh * groups + r / A.S, s = r % A.S;
    if (A.mask != nullptr) {
        const int mk = A.mask[s];
        float qf[8];
        unpack8(reinterpret_cast<const uint4*>(A.q + (size_t(h) * A.S + s) * kHD)[lane], qf);
        uint4 kx[8], vx[8];
#pragma unroll
        for (int tr = 0; tr < 8; ++tr)
            if (tr < A.S) {  // every tree row, not only the admitted ones: no wait on the mask word
                kx[tr] = reinterpret_cast<const uint4*>(A.xk + (size_t(kh) * A.S + tr) * kHD)[lane];
                vx[tr] = reinterpret_cast<const uint4*>(attn_xv_row(A, kh, tr))[lane];
            }
#pragma unroll
        for (int tr = 0; tr < 8; ++tr) {
            if (!(tr < A.S && ((mk >> tr) & 1))) continue;
            float kf[8], vf[8];
            unpack8(kx[tr], kf);
            unpack8(vx[tr], vf);
            float v = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j) v += qf[j] * kf[j];
#pragma unroll
            for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            const float sc = v * 0.0625f;
            const float M2 = fmaxf(M, sc);
            const float fp = M == -INFINITY ? 0.f : expf(M - M2), ft = expf(sc - M2);
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] = acc[j] * fp + ft * vf[j];
            sum = sum * fp + ft;
            M = M2;
        }
    }
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float lo = sum > 0.f ? acc[2 * j] / sum : 0.f, hi = sum > 0.f ? acc[2 * j + 1] / sum : 0.f;
        o[j] = uint32_t(f32_to_bf16_bits(lo)) | (uint32_t(f32_to_bf16_bits(hi)) << 16);
    }
    const int Hs = A.H / A.streams, b = h / Hs;  // stream b's output rows [b S, (b + 1) S) of Hs heads
    reinterpret_cast<uint4*>(A.out + ((size_t(b) * A.S + s) * Hs + h % Hs) * kHD)[lane] =
        make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void __cluster_dims__(kAttCluster, 1, 1) __launch_bounds__(kAttThreads) attn_kernel(const AttnArgs A) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint16_t* Qs = reinterpret_cast<uint16_t*>(smem);               // [32][kQPitch]
    uint16_t* Ks = Qs + kAttRows * kQPitch;                         // [64][kQPitch]
    uint16_t* Vs = Ks + kAttTile * kQPitch;                         // [64][kQPitch]
    uint16_t* Ps = Vs + kAttTile * kQPitch;                         // [32][kPPitch]
    float* red = reinterpret_cast<float*>(Ps + kAttRows * kPPitch);  // [4 warps][32 rows]
    const int chunk = blockIdx.x, kh = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int L = clamp_len(A.seqlen[kh / (A.Hk / A.streams)], A.cap);
    int per, active;
    attn_chunking(L, A.chunks, per, active);
    const int parts = active > 0 ? active : 1;  // L = 0: cluster 0 still writes the tree rows' outputs
    const int live = (parts + kAttCluster - 1) / kAttCluster, cg0 = chunk / kAttCluster;
    if (cg0 >= live) return;  // the whole cluster: no chunk of it has work
    const int groups = A.H / A.Hk, R = groups * A.S;
    const int t0 = chunk * per, t1 = (t0 + per < L) ? t0 + per : L;
    const uint16_t* kbase = A.kc + size_t(kh) * A.cap * kHD;
    const uint16_t* vbase = A.vc + size_t(kh) * A.cap * kHD;
    // Before the dependency wait (a launch with programmatic dependency on the Q / K norm + KV write): the chunk's
    // first K / V tile when the preceding kernel cannot have written it. That kernel writes this call's rows at
    // their positions: past the prefix with a tree mask, the prefix's last S tokens for the draft row.
    const int fresh = A.mask != nullptr ? L : L - A.S;
    const bool early = chunk < active && t0 < t1 && t0 + ((t1 - t0) < kAttTile ? (t1 - t0) : kAttTile) <= fresh;
    auto load_tile = [&](int tt, int nvalid) {
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
    };
    if (early) load_tile(t0, (t1 - t0) < kAttTile ? (t1 - t0) : kAttTile);
    pdl_wait();
    pdl_launch_dependents();  // after the wait: a dependent's early loads never see this kernel's inputs change
    {  // the rows a merging warp finishes (q row, tree rows' k and v: 128-byte lines) into L2 ahead of use
        const int r = (chunk % kAttCluster) * 4 + warp;
        if (r < R && A.mask != nullptr) {
            const int h = kh * groups + r / A.S, s = r % A.S;
            const int lines = 4 * (1 + 2 * A.S);
            for (int i = lane; i < lines; i += 32) {
                const int row = i >> 2, part = (i & 3) * 64;
                const uint16_t* base = row == 0      ? A.q + (size_t(h) * A.S + s) * kHD
                                       : row <= A.S ? A.xk + (size_t(kh) * A.S + (row - 1)) * kHD
                                                    : attn_xv_row(A, kh, row - 1 - A.S);
                prefetch_l2(base + part);
            }
        }
    }
    // Q rows r = gi * S + s of q head kh * groups + gi, rows >= R zero (the copies join the first tile's group)
    for (int i = tid; chunk < active && i < kAttRows * (kHD / 8); i += kAttThreads) {
        const int r = i / (kHD / 8), c = i % (kHD / 8);
        if (r < R)
            cp_async16(Qs + r * kQPitch + c * 8, A.q + (size_t(kh * groups + r / A.S) * A.S + r % A.S) * kHD + c * 8);
        else
            reinterpret_cast<uint4*>(Qs + r * kQPitch)[c] = make_uint4(0, 0, 0, 0);
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
    for (int tt = t0; tt < t1; tt += kAttTile) {
        const int nvalid = (t1 - tt) < kAttTile ? (t1 - tt) : kAttTile;
        __syncthreads();  // the previous tile's K / V / P reads are done
        if (!(early && tt == t0)) load_tile(tt, nvalid);
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
    // the chunk's unnormalized O, max and sum into this CTA's shared memory, over the K / V tiles (every warp
    // is past its last P V read)
    float* Op = reinterpret_cast<float*>(Ks);  // [32][kOPitch]
    float* Ml = Op + kAttRows * kOPitch;       // [32][2]
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            const int col = warp * 64 + nt * 8 + 2 * t;
            *reinterpret_cast<float2*>(Op + (mt * 16 + g) * kOPitch + col) = make_float2(O[mt][nt][0], O[mt][nt][1]);
            *reinterpret_cast<float2*>(Op + (mt * 16 + 8 + g) * kOPitch + col) = make_float2(O[mt][nt][2], O[mt][nt][3]);
        }
    if (warp == 0 && t == 0)
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
            const int row = (rr >> 1) * 16 + (rr & 1) * 8 + g;
            Ml[row * 2] = mrun[rr];
            Ml[row * 2 + 1] = lrun[rr];
        }
    cluster_arrive_release();
    cluster_wait_acquire();  // every chunk's partial of the cluster is written
    // cluster merge: warp w of cluster rank j takes row r = 4 j + w; lane l dims [8 l, 8 l + 8)
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = int(cluster.block_rank()), r = rank * 4 + warp;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float M = -INFINITY, sum = 0.f;
    if (r < R) {
        float mc[kAttCluster], lc[kAttCluster];
        float4 oc[kAttCluster][2];
#pragma unroll
        for (int c = 0; c < kAttCluster; ++c) {
            const float2 ml2 = ld_cluster_v2(cluster_addr(Ml + r * 2, c));
            const uint32_t oa = cluster_addr(Op + r * kOPitch + 8 * lane, c);
            mc[c] = ml2.x;
            lc[c] = ml2.y;
            oc[c][0] = ld_cluster_v4(oa);
            oc[c][1] = ld_cluster_v4(oa + 16);
        }
#pragma unroll
        for (int c = 0; c < kAttCluster; ++c) M = fmaxf(M, mc[c]);
#pragma unroll
        for (int c = 0; c < kAttCluster; ++c) {
            const float w = mc[c] == -INFINITY ? 0.f : expf(mc[c] - M);
            sum += lc[c] * w;
            const float o8[8] = {oc[c][0].x, oc[c][0].y, oc[c][0].z, oc[c][0].w,
                                 oc[c][1].x, oc[c][1].y, oc[c][1].z, oc[c][1].w};
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] += o8[j] * w;
        }
    }
    cluster_arrive_release();  // this CTA is done with the peers' shared memory
    if (live == 1) {
        if (r < R) attn_finish_row(A, kh, r, lane, acc, M, sum);
    } else {
        // cross-cluster merge: clusters write their merged rows; per (kv head, rank) the last arriving CTA merges
        // the live clusters in cluster order
        __shared__ int last;
        const size_t G = size_t(A.chunks / kAttCluster);
        if (r < R) {
            const size_t u = (size_t(kh) * G + cg0) * kAttRows + r;
            float4* gp = reinterpret_cast<float4*>(A.part + u * kHD) + 2 * lane;
            gp[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
            gp[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
            if (lane == 0) {
                A.ml[u * 2] = M;
                A.ml[u * 2 + 1] = sum;
            }
        }
        __syncthreads();
        if (tid == 0) {
            // acq_rel: releases the CTA's rows (ordered before by the barrier) and, for the last arrival, acquires
            // every other cluster's
            unsigned* cnt = A.count + kh * kAttCluster + rank;
            const unsigned prev = atom_add_acq_rel_gpu(cnt, 1u);
            last = prev == unsigned(live - 1);
            if (last) *cnt = 0u;  // every live cluster has arrived: zero for the next launch
        }
        __syncthreads();
        if (last && r < R) {
            // lane c holds cluster c's (max, sum) (live <= 32 clusters: attn_chunks); the rows
            // are loaded four clusters at a time, merged in cluster order
            const size_t u0 = size_t(kh) * G * kAttRows + r;
            float mc = -INFINITY, lc = 0.f;
            if (lane < live) {
                mc = __ldcg(A.ml + (u0 + size_t(lane) * kAttRows) * 2);
                lc = __ldcg(A.ml + (u0 + size_t(lane) * kAttRows) * 2 + 1);
            }
            M = mc;
#pragma unroll
            for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
            const float wl = mc == -INFINITY ? 0.f : expf(mc - M);
            sum = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] = 0.f;
            for (int c0 = 0; c0 < live; c0 += 4) {
                float4 a[4], b[4];
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    if (c0 + q < live) {
                        const float4* gp = reinterpret_cast<const float4*>(A.part + (u0 + size_t(c0 + q) * kAttRows) * kHD) + 2 * lane;
                        a[q] = __ldcg(gp);
                        b[q] = __ldcg(gp + 1);
                    }
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float w = __shfl_sync(0xffffffffu, wl, (c0 + q) & 31);
                    const float l = __shfl_sync(0xffffffffu, lc, (c0 + q) & 31);
                    if (c0 + q >= live) continue;
                    sum += l * w;
                    const float o8[8] = {a[q].x, a[q].y, a[q].z, a[q].w, b[q].x, b[q].y, b[q].z, b[q].w};
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc[j] += o8[j] * w;
                }
            }
            attn_finish_row(A, kh, r, lane, acc, M, sum);
        }
    }
    cluster_wait_acquire();  // the peers are done with this CTA's shared memory
}

size_t attn_smem_bytes() {
    return size_t(kAttRows + 2 * kAttTile) * kQPitch * 2 + size_t(kAttRows) * kPPitch * 2 + 4 * 32 * 4;
}
static_assert(size_t(kAttRows) * kOPitch * 4 + kAttRows * 2 * 4 <= size_t(2 * kAttTile) * kQPitch * 2,
              "the partial O fits over the K / V tiles");
int attn_chunks(int Hk, int cap, int sms) {
    // about two CTAs per SM at the longest context the cache holds, at least one tile per chunk, whole clusters
    int chunks = (2 * sms + Hk - 1) / Hk;
    const int tiles = (cap + kAttTile - 1) / kAttTile;
    if (tiles < chunks) chunks = tiles > 0 ? tiles : 1;
    if (chunks > 32 * kAttCluster) chunks = 32 * kAttCluster;  // the cross-cluster merge holds one cluster per lane
    return (chunks + kAttCluster - 1) / kAttCluster * kAttCluster;
}
// chunks follow one stream's kv heads: a batched stream is split exactly as it would be alone
size_t attn_workspace_bytes(int Hk, int streams, int cap, int sms) {
    const size_t clusters = attn_chunks(Hk / streams, cap, sms) / kAttCluster;
    return size_t(Hk) * clusters * kAttRows * (kHD + 2) * 4 + size_t(Hk) * kAttCluster * 4;
}

int launch_tree_attention(AttnArgs A, void* ws, cudaStream_t stream) {
    A.chunks = attn_chunks(A.Hk / A.streams, A.cap, sm_count());
    const size_t G = size_t(A.chunks / kAttCluster);
    A.part = static_cast<float*>(ws);
    A.ml = A.part + size_t(A.Hk) * G * kAttRows * kHD;
    A.count = reinterpret_cast<unsigned*>(A.ml + size_t(A.Hk) * G * kAttRows * 2);
    MONO_CHECK(G <= 32, "at most 32 clusters of context chunks per kv head (got %d)", int(G));
    const size_t smem = attn_smem_bytes();
    static std::once_flag once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(once, [&] {
        attr_err = cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    });
    CUDA_TRY(attr_err);
    // programmatic dependency on the preceding kernel (the Q / K norm + KV write): griddepcontrol.wait inside
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(A.chunks, A.Hk);
    cfg.blockDim = dim3(kAttThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CUDA_TRY(cudaLaunchKernelEx(&cfg, attn_kernel, A));
    return MONO_OK;
}

}  // namespace mono
