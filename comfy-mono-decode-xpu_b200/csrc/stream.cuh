// Producer/consumer form of the W4A8 stream engine: PW producer warps per CTA keep a ring of S item
// stages full, CW consumer warps compute the items in the order they were requested.
//
// Why this shape (measured on B200): a thread that issues 8 KB bulk copies back to back is held for each
// copy, so one issuing thread per SM streams at most ~32 GB/s (4.7 TB/s over 148 SMs) and a few warps
// issuing side by side are needed for the HBM rate (4 issuing warps: 6.6 TB/s); and a warp that both
// computes and refills its own ring waits behind every request issued before its refill (warps with a
// second item finished 2-3 us after the last byte had landed). Here the producers only issue, consumer
// warp w takes items w, w + CW, w + 2 CW, ... of the CTA's request order, and producer warp p issues
// items p, p + PW, ..., so work follows the arrival order of the data.
//
// S is a multiple of CW and of PW, so every slot is always filled by the same producer and consumed by the
// same consumer warp, one use after the other. This is what makes the parity waits exact: an mbarrier only tells the parity
// of its current phase, and a warp that waited for a slot's use u + 1 while use u had not landed yet
// would see the older phase of the same parity as complete.
//
// Items of a CTA: for every phase of the program, the CTA's 16-row tiles T = b + k * gridDim.x (b = blockIdx.x, or
// gridDim.x - 1 - blockIdx.x for a phase marked `rev`: CTAs with more tiles in one phase get fewer in the next,
// and the ring carries the difference across the grid barrier), and per tile its subtiles (gate | up of a
// paired phase) and 1024-wide chunks:
//     i = base(phase) + (k * subs + sub) * C + chunk.
// Ring slot s = i % S; the producer waits for empty[s] (phase (i / S - 1) & 1) before reusing it, the
// consumer waits for full[s] (phase (i / S) & 1). Item partials (engine.cuh compute_item) go to shared
// memory at [(k * subs + sub) * C + chunk]; after a phase the consumers sum them in chunk order, so the
// arithmetic is exactly that of the per-warp form.
#pragma once
#include "engine.cuh"

namespace mono {

constexpr int kConsumerBar = 15;  // named barrier of the consumer warps

// Warp configurations of the cooperative stream kernels, deepest ring first: the launchers take the first whose
// ring fits next to the partials and the staged activations. S is a multiple of CW and PW.
struct StreamConfig {
    int CW, PW, S;
};
// The last, shallow ring leaves room for 32 staged activation rows (4 batched decode streams).
constexpr int kStreamConfigs = 4;
constexpr StreamConfig kStreamConfig[kStreamConfigs] = {{10, 2, 20}, {8, 4, 16}, {12, 4, 12}, {8, 4, 8}};
constexpr size_t kStreamSmemLimit = 227 * 1024 - 512;  // dynamic bytes, leaving room for the static ones

// Barrier of the CW consumer warps (the producer warp is warp CW, the last one).
template <int CW>
__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync %0, %1;" ::"n"(kConsumerBar), "n"(CW * 32) : "memory");
}

// Consumer barrier that also ANDs a per-thread flag over the consumer threads.
template <int CW>
__device__ __forceinline__ bool consumer_sync_and(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(uint32_t(v)), "n"(kConsumerBar), "n"(CW * 32)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ int phase_subs(const PhaseDesc& p) { return p.paired ? 2 : 1; }
// this CTA's position in the phase's round robin
__device__ __forceinline__ int cta_slot(const PhaseDesc& p) {
    return p.rev ? int(gridDim.x) - 1 - int(blockIdx.x) : int(blockIdx.x);
}
__device__ __forceinline__ int cta_tiles(const PhaseDesc& p) {
    const int nt = phase_tiles(p), b = cta_slot(p), G = int(gridDim.x);
    return b < nt ? (nt - 1 - b) / G + 1 : 0;
}
// global tile of this CTA's k-th tile of the phase
__device__ __forceinline__ int cta_tile(const PhaseDesc& p, int k) { return cta_slot(p) + k * int(gridDim.x); }
__device__ __forceinline__ int cta_items(const PhaseDesc& p) { return cta_tiles(p) * phase_subs(p) * (p.K >> 10); }
__device__ __forceinline__ int cta_base(const Program& P, int ph) {
    int b = 0;
    for (int q = 0; q < ph; ++q) b += cta_items(P.ph[q]);
    return b;
}
__device__ __forceinline__ int cta_total(const Program& P) { return cta_base(P, P.nph); }

// Issue the copy of item (tile T, sub, c) of phase p into `stage`, completing on `full`. TILED: lane 0, one bulk
// copy (the full barrier counts 1 arrival + the bytes). ROW: every lane gathers its 16-byte pieces with
// cp.async and arrives once when they land (the full barrier counts 32 arrivals).
template <int FMT, int LAYOUT>
__device__ __forceinline__ void issue_tile_item(const PhaseDesc& p, int T, int sub, int c, uint8_t* stage, uint64_t* full,
                                                int lane) {
    constexpr int SB = Fmt<FMT>::SB;
    int mat, lt;
    resolve(p, T, sub, mat, lt);
    const MatDesc& w = p.m[mat];
    if constexpr (LAYOUT == LAYOUT_TILED) {
        if (lane == 0) {
            mbar_arrive_expect_tx(full, kStageW + SB);
            bulk_g2s_hint(stage, w.q + (size_t(lt) * (p.K >> 10) + c) * (kStageW + SB), kStageW + SB, full,
                          l2_evict_first_policy());
        }
    } else {
        const int g = lane >> 2, t = lane & 3;
        const size_t rowb = size_t(p.K) >> 1;
        const uint8_t* r0 = w.q + size_t(lt * 16 + g) * rowb + size_t(c) * 512 + t * 16;
        const uint8_t* r1 = r0 + 8 * rowb;
#pragma unroll
        for (int gi = 0; gi < 8; ++gi) {
            cp_async16(stage + gi * 1024 + lane * 16, r0 + gi * 64);
            cp_async16(stage + gi * 1024 + 512 + lane * 16, r1 + gi * 64);
        }
        if constexpr (FMT == FMT_GPTQ) {
            if (lane < 16) cp_async16(stage + kStageW + lane * 16, w.s + (size_t(lt * 16 + lane) * (p.K >> 7) + c * 8) * 2);
        } else {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int piece = lane + 32 * h, row = piece >> 2, part = piece & 3;
                cp_async16(stage + kStageW + row * 64 + part * 16, w.s + size_t(lt * 16 + row) * (p.K >> 4) + c * 64 + part * 16);
            }
        }
        asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(full)) : "memory");
    }
}

// The same for the k-th round-robin tile of this CTA (T = blockIdx.x + k * gridDim.x).
template <int FMT, int LAYOUT>
__device__ __forceinline__ void issue_item(const PhaseDesc& p, int k, int sub, int c, uint8_t* stage, uint64_t* full,
                                           int lane) {
    issue_tile_item<FMT, LAYOUT>(p, cta_tile(p, k), sub, c, stage, full, lane);
}

// Ask the L2 to fetch item (k, sub, c) of phase p (TILED layout: one contiguous block) ahead of its copy.
template <int FMT>
__device__ __forceinline__ void prefetch_item_l2(const PhaseDesc& p, int k, int sub, int c) {
    constexpr int SB = Fmt<FMT>::SB;
    const int T = int(blockIdx.x) + k * int(gridDim.x);
    int mat, lt;
    resolve(p, T, sub, mat, lt);
    const uint8_t* src = p.m[mat].q + (size_t(lt) * (p.K >> 10) + c) * (kStageW + SB);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(kStageW + SB) : "memory");
}

// Incremental walk over a CTA's items across the phases of a program, in request order (no divisions per
// step): the current item is (phase ph, tile T, subtile sub, chunk c); `left` items of the phase remain after it.
struct ItemWalk {
    int ph, T, sub, c, left, subs, C, tstep;
    bool done;
    // position at the n-th item of phase ph for this CTA; false if the phase has fewer
    __device__ bool enter(const Program& P, int n) {
        const PhaseDesc& p = P.ph[ph];
        const int cnt = cta_items(p);
        if (n >= cnt) return false;
        subs = phase_subs(p);
        C = p.K >> 10;
        const int per = subs * C, k = n / per, r = n - k * per;
        T = cta_tile(p, k);
        tstep = int(gridDim.x);
        sub = r / C;
        c = r - sub * C;
        left = cnt - 1 - n;
        return true;
    }
    __device__ void start(const Program& P, int i) {
        done = false;
        for (ph = 0; ph < P.nph; ++ph) {
            if (enter(P, i)) return;
            i -= cta_items(P.ph[ph]);
        }
        done = true;
    }
    __device__ void step(const Program& P) {
        if (left == 0) {
            while (++ph < P.nph)
                if (enter(P, 0)) return;
            done = true;
            return;
        }
        --left;
        if (++c < C) return;
        c = 0;
        if (++sub < subs) return;
        sub = 0;
        T += tstep;
    }
};

// Producer warp p (of PW): items p, p + PW, ..., slot i % S. Returns false if a wait gave up (then it
// stops issuing; the consumers' own bounded waits end the kernel). Before returning, it waits (bounded)
// for the last copy of each of its slots, so no copy lands in shared memory after the CTA has exited.
template <int FMT, int LAYOUT, int PW>
__device__ __forceinline__ bool produce_all(const Program& P, uint8_t* ring, uint64_t* full, uint64_t* empty, int S,
                                            int p, int lane) {
    bool ok = true;
    int i = p;
    ItemWalk w;
    w.start(P, i);
    for (; !w.done && ok; i += PW) {
        const int s = i % S;
        if (i >= S) ok = __all_sync(0xffffffffu, mbar_wait(&empty[s], ((i / S) - 1) & 1));
        if (!ok) break;
        issue_tile_item<FMT, LAYOUT>(P.ph[w.ph], w.T, w.sub, w.c, ring + size_t(s) * stage_bytes<FMT>(), &full[s], lane);
        for (int q = 0; q < PW && !w.done; ++q) w.step(P);
    }
    // items p, p + PW, ..., i - PW were issued: wait for the last use of each of this producer's S / PW slots
    const int issued = (i - p) / PW, keep = S / PW < issued ? S / PW : issued;
    for (int j = 0; j < keep; ++j) {
        const int it = i - PW * (j + 1);
        mbar_wait(&full[it % S], (it / S) & 1);
    }
    return ok;
}

// Consumer side: the items [first, first + count) of phase p (count < 0: to the end of the phase) that consumer
// warp `cw` (of CW) computes, each partial stored at part[item - first] (item = (k * subs + sub) * C + chunk).
// base0 = the CTA's request index of the phase's first item. S must be a multiple of CW. Returns false if a
// wait gave up.
template <int FMT, int LAYOUT, int MT, int CW>
__device__ __forceinline__ bool consume_items(const PhaseDesc& p, int base0, const uint16_t* pair_tab, int M,
                                              const XSrc& xs, uint8_t* ring, uint64_t* full, uint64_t* empty, int S,
                                              uint32_t* part, int cw, int lane, int first = 0, int count = -1) {
    const int nph = cta_items(p), C = p.K >> 10;
    const int base = base0 + first, n = count < 0 || first + count > nph ? nph - first : count;
    bool ok = true;
    int i = base + ((cw - base % CW) + CW) % CW;
    for (; i < base + n && ok; i += CW) {
        const int s = i % S, li = i - base0;
        ok = mbar_wait(&full[s], (i / S) & 1);
        if (!ok) break;
        uint32_t R[MT][4];
        const uint8_t* stage = ring + size_t(s) * stage_bytes<FMT>();
        if (xs.smem)
            compute_item<FMT, LAYOUT, MT, 2>(stage, pair_tab, xs, M, li % C, lane, R);
        else if (xs.cg)
            compute_item<FMT, LAYOUT, MT, 3>(stage, pair_tab, xs, M, li % C, lane, R);
        else if (xs.perm)
            compute_item<FMT, LAYOUT, MT, 1>(stage, pair_tab, xs, M, li % C, lane, R);
        else
            compute_item<FMT, LAYOUT, MT, 0>(stage, pair_tab, xs, M, li % C, lane, R);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        store_partial<MT>(part, li - first, lane, R);
    }
    return ok;
}

template <int FMT, int LAYOUT, int MT, int CW>
__device__ __forceinline__ bool consume_phase(const Program& P, int ph, const XSrc& xs, uint8_t* ring, uint64_t* full,
                                              uint64_t* empty, int S, uint32_t* part, int cw, int lane, int first = 0,
                                              int count = -1) {
    return consume_items<FMT, LAYOUT, MT, CW>(P.ph[ph], cta_base(P, ph), P.pair_tab, P.M, xs, ring, full, empty, S, part,
                                              cw, lane, first, count);
}

// Vector staging of an activation block x [M][K] (rows contiguous) by the consumer threads into shared
// memory (pitch K + 16), permuted unless x is permuted already: batches of NB (8 or 16) pieces of 16 bytes per
// thread, every load of a batch in flight before any store. Ends with a consumer barrier.
// sc (optional): the M row scales, copied to sc_dst[M] in the same round trip as the first batch.
template <int CW, int NB = 8>
__device__ __forceinline__ void stage_x_consumers(const int8_t* x, int M, int K, bool xperm, int8_t* xsm,
                                                  const float* sc = nullptr, float* sc_dst = nullptr) {
    const int T = CW * 32, words = K >> 4, total = M * words;
    const uint4* src = reinterpret_cast<const uint4*>(x);
    const bool own_sc = sc != nullptr && int(threadIdx.x) < M;
    float scv = 0.f;
    if (own_sc) scv = __ldcg(sc + threadIdx.x);
    // (every CTA walks the block in the same order: staggered start offsets per CTA measured slower)
    for (int base = threadIdx.x; base < total; base += NB * T) {
        uint4 v[NB];
#pragma unroll
        for (int j = 0; j < NB; ++j)
            if (base + j * T < total) v[j] = __ldcg(src + base + j * T);
#pragma unroll
        for (int j = 0; j < NB; ++j) {
            const int i = base + j * T;
            if (i < total) {
                const int m = i / words, c = i - m * words;
                reinterpret_cast<uint4*>(xsm + size_t(m) * (K + 16))[c] = xperm ? v[j] : perm16(v[j]);
            }
        }
    }
    if (own_sc) sc_dst[threadIdx.x] = scv;
    consumer_sync<CW>();
}

// Shared-memory plan of a stream kernel (bytes, each part 128-byte aligned): ring stages, full and empty
// barriers, partials, staged activations, scratch.
struct StreamPlan {
    size_t ring, bars, part, x, scratch, total;
    int S;
    __host__ __device__ StreamPlan(int fmt_stage_bytes, int slots, size_t part_bytes, size_t x_bytes, size_t scratch_bytes) {
        S = slots;
        auto al = [](size_t b) { return (b + 127) / 128 * 128; };
        ring = size_t(slots) * fmt_stage_bytes;
        bars = al(size_t(slots) * 16);
        part = al(part_bytes);
        x = al(x_bytes);
        scratch = al(scratch_bytes);
        total = ring + bars + part + x + scratch;
    }
};

}  // namespace mono
