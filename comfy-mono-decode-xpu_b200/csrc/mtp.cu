// Device-side bookkeeping of the MTP decode loop (the role of csrc/mtp_loop.sycl:29-196): the host queues the
// next step without reading anything back.
//   prep_draft   MTP KV positions / seqlen of draft k and the draft's rope row
//   prep_verify  attention positions / seqlen, verify rope positions, ctl parity and tree program
//   accept       the greedy accept walk (continue along the child whose draft token is the token the verify
//                chose; warp-parallel over a node's children), the result row [n, commit[8], row, on_chain,
//                nranks, ranks[7], pos, kept], the counters st (st[0] committed length, st[1] MTP KV length), ctl
//                (pending, slots), the next token and hidden row, and the attention KV slot moves of an off-chain
//                path (vector copies)
// st int64 [4]; ctl int32 [2 + 3 * 8] = [pending, parity, accepted[8], parent[8], prog[8]].
#include "launch.h"

namespace mono {

constexpr int kSlots = 8, kRanks = 7;

// CTA b: stream b of a batch (st, freqs, mpos, mseq offset by b times their strides; one stream: strides 0)
__global__ void __launch_bounds__(256) mtp_prep_draft_kernel(const int64_t* st, int64_t k, const float* ftab, int64_t n,
                                                             int64_t cap, float* freqs, int64_t* mpos, int np,
                                                             int32_t* mseq, int64_t st_stride, int64_t freqs_stride,
                                                             int64_t mpos_stride, int64_t mseq_stride) {
    pdl_launch_dependents();  // an ordinary launch: its inputs are complete; the next kernel may start
    const int t = threadIdx.x;
    const int64_t b = blockIdx.x;
    st += b * st_stride;
    freqs += b * freqs_stride;
    mpos += b * mpos_stride;
    mseq += b * mseq_stride;
    const int64_t p = st[0] + k, m = st[1] + k;
    const int64_t row = p < cap ? (p < 0 ? 0 : p) : cap - 1;
    for (int64_t i = t; i < n; i += 256) freqs[i] = ftab[row * n + i];
    if (t < np) mpos[t] = m + t;
    if (t == 0) mseq[0] = int32_t(m + 1);
}

// CTA b: stream b of a batch (st, apos, aseq, vpos, ctl offset by b times their strides; one stream: strides 0)
__global__ void __launch_bounds__(64) mtp_prep_verify_kernel(const int64_t* st, int64_t* apos, int np, int32_t* aseq,
                                                             int64_t* vpos, const int64_t* tree_pos, int rows,
                                                             int32_t* ctl, const int32_t* tree_ctl, int parity,
                                                             int64_t rope_offset, int64_t st_stride,
                                                             int64_t apos_stride, int64_t aseq_stride,
                                                             int64_t vpos_stride, int64_t ctl_stride) {
    pdl_launch_dependents();  // an ordinary launch: its inputs are complete; the next kernel may start
    const int t = threadIdx.x;
    const int64_t b = blockIdx.x;
    st += b * st_stride;
    apos += b * apos_stride;
    aseq += b * aseq_stride;
    vpos += b * vpos_stride;
    ctl += b * ctl_stride;
    const int64_t pos = st[0];
    if (t < np) apos[t] = pos + t;
    if (t == 0) aseq[0] = int32_t(pos);
    if (t < rows) vpos[t] = tree_pos[t] + pos + rope_offset;
    if (t == 0) ctl[1] = parity;
    if (t < 2 * kSlots) ctl[2 + kSlots + t] = tree_ctl[t];
}

struct AcceptArgs {
    int64_t* st;
    const int64_t* toks;      // [rows] the verify's token at each row
    const int64_t* drafts;    // [rows] each row's draft token
    const int64_t* cand;      // [7 x 7] draft candidates per chain node, or null
    const int32_t* children;  // [8][8], -1 ends a row's list
    const uint16_t* x;        // [rows][H] hidden rows
    uint16_t* h_out;          // [H]
    int64_t* next_tok;
    int32_t* ctl;
    const int64_t* kv_ptrs;   // [nkv] bf16 caches [heads][cap][head_dim]
    int64_t* result;          // [32]
    int64_t H, nkv, heads, cap, head_dim;
    int rows, depth;
};

// The accept step, in three parts:
//   walk     warp 0: at node `cur`, lane j < 8 reads child j of cur and tests its draft token against the verify's
//            token at cur; the first passing child (a ballot, lowest lane) is the next node. A child index that is
//            not after its parent or not below `rows` ends the walk and records DEV_BAD_TREE (a malformed table
//            would otherwise repeat rows or move a KV slot before it is read). Then lanes write the result row,
//            counters, ctl and next token in parallel: result = [n, commit[8], row, on_chain, nranks, ranks[7], pos,
//            kept] (csrc/mtp_loop.sycl:143 layout).
//   hidden   every thread copies 16-byte pieces of the chosen row's hidden state.
//   KV       an off-chain path: accepted row path[k] moves to slot pos + k (FixedKVState.commit_path), one 16-byte
//            piece of one (cache, head) row per thread, k ascending with a barrier between (path[k] >= k, so a slot is
//            read before a later move could write it).
__global__ void __launch_bounds__(256) mtp_accept_kernel(const AcceptArgs A) {
    __shared__ int path[kSlots];
    __shared__ int meta[4];  // len, row, on_chain
    __shared__ int64_t base;
    const int t = threadIdx.x, lane = t & 31;
    if (t < 32) {
        int len = 1, cur = 0;
        if (lane == 0) path[0] = 0;
        bool bad = false;
        while (len < A.rows) {
            const int c = lane < kSlots ? A.children[cur * kSlots + lane] : -1;
            // children end at the first -1: lanes past it do not count
            const unsigned ends = ~__ballot_sync(0xffffffffu, c >= 0) & ((1u << kSlots) - 1u);
            const int first_end = ends ? __ffs(ends) - 1 : kSlots;  // lanes below it are listed children
            const bool listed = lane < first_end && c >= 0;
            const bool valid = !listed || (c > cur && c < A.rows);
            if (__any_sync(0xffffffffu, !valid)) {
                bad = true;
                break;
            }
            const unsigned hit = __ballot_sync(0xffffffffu, listed && A.drafts[listed ? c : 0] == A.toks[cur]);
            if (hit == 0u) break;
            const int next = __shfl_sync(0xffffffffu, c, __ffs(hit) - 1);
            if (lane == 0) path[len] = next;
            ++len;
            cur = next;
        }
        if (bad && lane == 0) set_device_error(DEV_BAD_TREE);
        __syncwarp();
        const int row = cur;
        const bool on_chain = row == len - 1;
        const int keep = on_chain ? len : len - 1;
        const int kept = keep < A.depth ? keep : A.depth;
        const int64_t pos = A.st[0];
        int64_t* rp = A.result;
        // rank of the verify token among a chain node's candidates (auto-tree statistics), lanes = path entries
        int r = kRanks;
        const int node = lane < len ? path[lane] : 0;
        const bool ranked = A.cand != nullptr && lane < len && node < A.depth;
        if (ranked)
            for (int q = 0; q < kRanks; ++q)
                if (A.cand[node * kRanks + q] == A.toks[node]) {
                    r = q;
                    break;
                }
        // ranks are recorded for the path's leading run of chain nodes (the walk's order)
        const unsigned rk = __ballot_sync(0xffffffffu, ranked);
        const int nr = __ffs(~rk) - 1;
        if (lane <= kSlots)
            rp[lane] = lane == 0 ? len : (lane < len ? A.drafts[path[lane]] : (lane == len ? A.toks[row] : -1));
        if (lane < kRanks) rp[12 + lane] = lane < nr ? r : 0;
        if (lane < kSlots) A.ctl[2 + lane] = lane < len ? path[lane] : lane;
        if (lane == 0) {
            rp[9] = row;
            rp[10] = on_chain;
            rp[11] = nr;
            rp[19] = pos;
            rp[20] = kept;
            A.st[0] = pos + len;
            A.st[1] = A.st[1] + kept;
            A.ctl[0] = len;
            A.next_tok[0] = A.toks[row];
            meta[0] = len;
            meta[1] = row;
            meta[2] = on_chain;
            base = pos;
        }
    }
    __syncthreads();
    const int len = meta[0], row = meta[1];
    // the chosen row's hidden state (16-byte pieces when the sizes allow, else elements)
    if ((A.H & 7) == 0 && (reinterpret_cast<uintptr_t>(A.x) & 15) == 0 && (reinterpret_cast<uintptr_t>(A.h_out) & 15) == 0) {
        const uint4* src = reinterpret_cast<const uint4*>(A.x + int64_t(row) * A.H);
        uint4* dst = reinterpret_cast<uint4*>(A.h_out);
        for (int64_t i = t; i < A.H / 8; i += blockDim.x) dst[i] = src[i];
    } else {
        for (int64_t i = t; i < A.H; i += blockDim.x) A.h_out[i] = A.x[int64_t(row) * A.H + i];
    }
    if (meta[2]) return;  // on the chain: every accepted row already sits at its slot
    // pieces of 8 elements (a 16-byte copy when the cache row is 16-byte aligned, else 8 element copies)
    const int64_t per_row = (A.head_dim + 7) / 8, pieces = A.nkv * A.heads * per_row;
    for (int k = 1; k < len; ++k) {
        const int src_row = path[k];
        if (src_row != k) {
            const int64_t dst = (base + k) % A.cap, src = (base + src_row) % A.cap;
            for (int64_t i = t; i < pieces; i += blockDim.x) {
                const int64_t which = i / (A.heads * per_row), rem = i - which * A.heads * per_row;
                const int64_t h = rem / per_row, e0 = (rem - h * per_row) * 8;
                uint16_t* cache = reinterpret_cast<uint16_t*>(A.kv_ptrs[which]);
                uint16_t* d = cache + (h * A.cap + dst) * A.head_dim + e0;
                const uint16_t* s0 = cache + (h * A.cap + src) * A.head_dim + e0;
                if (e0 + 8 <= A.head_dim && ((reinterpret_cast<uintptr_t>(d) | reinterpret_cast<uintptr_t>(s0)) & 15) == 0)
                    *reinterpret_cast<uint4*>(d) = *reinterpret_cast<const uint4*>(s0);
                else
                    for (int64_t e = 0; e < 8 && e0 + e < A.head_dim; ++e) d[e] = s0[e];
            }
        }
        __syncthreads();
    }
}

}  // namespace mono

using namespace mono;

extern "C" {

int mono_mtp_prep_draft(const int64_t* st, int64_t k, const float* ftab, int64_t row_elems, int64_t cap, float* freqs,
                        int64_t* mpos, int64_t np, int32_t* mseq, mono_stream_t stream) {
    MONO_CHECK(st && ftab && freqs && mpos && mseq, "null operand");
    MONO_CHECK(row_elems >= 1 && cap >= 1 && np >= 0 && np <= 256 && k >= 0, "sizes");
    mtp_prep_draft_kernel<<<1, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(st, k, ftab, row_elems, cap, freqs, mpos,
                                                                                  int(np), mseq, 0, 0, 0, 0);
    CUDA_TRY(cudaGetLastError());
    return MONO_OK;
}

int mono_mtp_prep_draft_streams(const int64_t* st, int64_t st_stride, int64_t k, const float* ftab, int64_t row_elems,
                                int64_t cap, float* freqs, int64_t freqs_stride, int64_t* mpos, int64_t mpos_stride,
                                int64_t np, int32_t* mseq, int64_t mseq_stride, int64_t streams, mono_stream_t stream) {
    MONO_CHECK(st && ftab && freqs && mpos && mseq, "null operand");
    MONO_CHECK(row_elems >= 1 && cap >= 1 && np >= 0 && np <= 256 && k >= 0, "sizes");
    MONO_CHECK(streams >= 1 && streams <= 65535 && st_stride >= 2 && freqs_stride >= row_elems && mpos_stride >= np &&
                   mseq_stride >= 1,
               "1 <= streams; per-stream strides cover each stream's words");
    mtp_prep_draft_kernel<<<unsigned(streams), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        st, k, ftab, row_elems, cap, freqs, mpos, int(np), mseq, st_stride, freqs_stride, mpos_stride, mseq_stride);
    CUDA_TRY(cudaGetLastError());
    return MONO_OK;
}

int mono_mtp_prep_verify(const int64_t* st, int64_t* apos, int64_t np, int32_t* aseq, int64_t* vpos,
                         const int64_t* tree_pos, int64_t rows, int32_t* ctl, const int32_t* tree_ctl, int64_t parity,
                         int64_t rope_offset, mono_stream_t stream) {
    MONO_CHECK(st && apos && aseq && vpos && tree_pos && ctl && tree_ctl, "null operand");
    MONO_CHECK(rows >= 1 && rows <= kSlots && np >= 0 && np <= 64, "rows <= 8, positions <= 64");
    mtp_prep_verify_kernel<<<1, 64, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        st, apos, int(np), aseq, vpos, tree_pos, int(rows), ctl, tree_ctl, int(parity), rope_offset, 0, 0, 0, 0, 0);
    CUDA_TRY(cudaGetLastError());
    return MONO_OK;
}

int mono_mtp_prep_verify_streams(const int64_t* st, int64_t st_stride, int64_t* apos, int64_t apos_stride, int64_t np,
                                 int32_t* aseq, int64_t aseq_stride, int64_t* vpos, int64_t vpos_stride,
                                 const int64_t* tree_pos, int64_t rows, int32_t* ctl, int64_t ctl_stride,
                                 const int32_t* tree_ctl, int64_t parity, int64_t rope_offset, int64_t streams,
                                 mono_stream_t stream) {
    MONO_CHECK(st && apos && aseq && vpos && tree_pos && ctl && tree_ctl, "null operand");
    MONO_CHECK(rows >= 1 && rows <= kSlots && np >= 0 && np <= 64, "rows <= 8, positions <= 64");
    MONO_CHECK(streams >= 1 && streams <= 65535 && st_stride >= 2 && apos_stride >= np && aseq_stride >= 1 &&
                   vpos_stride >= rows && ctl_stride >= 2 + 3 * kSlots,
               "1 <= streams; per-stream strides cover each stream's words");
    mtp_prep_verify_kernel<<<unsigned(streams), 64, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        st, apos, int(np), aseq, vpos, tree_pos, int(rows), ctl, tree_ctl, int(parity), rope_offset, st_stride,
        apos_stride, aseq_stride, vpos_stride, ctl_stride);
    CUDA_TRY(cudaGetLastError());
    return MONO_OK;
}

int mono_mtp_accept(int64_t* st, const int64_t* toks, const int64_t* drafts, const int64_t* cand,
                    const int32_t* children, int64_t rows, int64_t depth, const void* x, int64_t H, int64_t* next_tok,
                    void* h_out, int32_t* ctl, const int64_t* kv_ptrs, int64_t nkv, int64_t heads, int64_t cap,
                    int64_t head_dim, int64_t* result, mono_stream_t stream) {
    MONO_CHECK(st && toks && drafts && children && x && next_tok && h_out && ctl && result, "null operand");
    MONO_CHECK(rows >= 1 && rows <= kSlots && depth >= 0 && depth < rows, "1 <= rows <= 8, 0 <= depth < rows");
    MONO_CHECK(H >= 1 && nkv >= 0 && (nkv == 0 || (kv_ptrs && heads >= 1 && cap >= 1 && head_dim >= 1)), "sizes");
    AcceptArgs A{};
    A.st = st;
    A.toks = toks;
    A.drafts = drafts;
    A.cand = cand;
    A.children = children;
    A.x = static_cast<const uint16_t*>(x);
    A.h_out = static_cast<uint16_t*>(h_out);
    A.next_tok = next_tok;
    A.ctl = ctl;
    A.kv_ptrs = kv_ptrs;
    A.result = result;
    A.H = H;
    A.nkv = nkv;
    A.heads = heads;
    A.cap = cap;
    A.head_dim = head_dim;
    A.rows = int(rows);
    A.depth = int(depth);
    mtp_accept_kernel<<<1, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(A);
    CUDA_TRY(cudaGetLastError());
    return MONO_OK;
}

}  // extern "C"
