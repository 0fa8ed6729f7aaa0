// Device-side bookkeeping of the MTP decode loop (the role of csrc/mtp_loop.sycl:29-196): the host queues the
// next step without reading anything back.
//   prep_draft   MTP KV positions / seqlen of draft k and the draft's rope row
//   prep_verify  attention positions / seqlen, verify rope positions, ctl parity and tree program
//   accept       the greedy accept walk (continue along the child whose draft token is the token the verify
//                chose), the result row [n, commit[8], row, on_chain, nranks, ranks[7], pos, kept], the
//                counters st (st[0] committed length, st[1] MTP KV length), ctl (pending, slots), the next
//                token and hidden row, and the attention KV slot moves of an off-chain path
// st int64 [4]; ctl int32 [2 + 3 * 8] = [pending, parity, accepted[8], parent[8], prog[8]].
#include "launch.h"

namespace mono {

constexpr int kSlots = 8, kRanks = 7;

__global__ void __launch_bounds__(256) mtp_prep_draft_kernel(const int64_t* st, int64_t k, const float* ftab, int64_t n,
                                                             int64_t cap, float* freqs, int64_t* mpos, int np,
                                                             int32_t* mseq) {
    const int t = threadIdx.x;
    const int64_t p = st[0] + k, m = st[1] + k;
    const int64_t row = p < cap ? (p < 0 ? 0 : p) : cap - 1;
    for (int64_t i = t; i < n; i += 256) freqs[i] = ftab[row * n + i];
    if (t < np) mpos[t] = m + t;
    if (t == 0) mseq[0] = int32_t(m + 1);
}

__global__ void __launch_bounds__(64) mtp_prep_verify_kernel(const int64_t* st, int64_t* apos, int np, int32_t* aseq,
                                                             int64_t* vpos, const int64_t* tree_pos, int rows,
                                                             int32_t* ctl, const int32_t* tree_ctl, int parity,
                                                             int64_t rope_offset) {
    const int t = threadIdx.x;
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

__global__ void __launch_bounds__(1024) mtp_accept_kernel(const AcceptArgs A) {
    __shared__ int sh[kSlots + 4];
    __shared__ int64_t base;
    const int t = threadIdx.x;
    if (t == 0) {
        int path[kSlots], len = 1;
        path[0] = 0;
        while (len < A.rows) {
            const int cur = path[len - 1];
            int next = -1;
            for (int j = 0; j < kSlots; ++j) {
                const int c = A.children[cur * kSlots + j];
                if (c < 0 || c >= A.rows) break;
                if (A.drafts[c] == A.toks[cur]) {
                    next = c;
                    break;
                }
            }
            if (next < 0) break;
            path[len++] = next;
        }
        const int row = path[len - 1];
        const bool on_chain = row == len - 1;
        const int keep = on_chain ? len : len - 1;
        const int kept = keep < A.depth ? keep : A.depth;
        const int64_t pos = A.st[0];
        int64_t* rp = A.result;
        rp[0] = len;
        for (int i = 1; i < len; ++i) rp[i] = A.drafts[path[i]];
        rp[len] = A.toks[row];
        for (int i = len + 1; i <= kSlots; ++i) rp[i] = -1;
        rp[9] = row;
        rp[10] = on_chain;
        int nr = 0;
        if (A.cand != nullptr)
            for (int i = 0; i < len && path[i] < A.depth; ++i) {
                const int node = path[i];
                int r = kRanks;
                for (int q = 0; q < kRanks; ++q)
                    if (A.cand[node * kRanks + q] == A.toks[node]) {
                        r = q;
                        break;
                    }
                rp[12 + nr++] = r;
            }
        rp[11] = nr;
        for (int i = 12 + nr; i < 19; ++i) rp[i] = 0;
        rp[19] = pos;
        rp[20] = kept;
        A.st[0] = pos + len;
        A.st[1] = A.st[1] + kept;
        A.ctl[0] = len;
        for (int i = 0; i < kSlots; ++i) A.ctl[2 + i] = i < len ? path[i] : i;
        A.next_tok[0] = A.toks[row];
        for (int i = 0; i < kSlots; ++i) sh[i] = i < len ? path[i] : i;
        sh[kSlots] = len;
        sh[kSlots + 1] = row;
        sh[kSlots + 2] = on_chain;
        base = pos;
    }
    __syncthreads();
    const int len = sh[kSlots], row = sh[kSlots + 1];
    for (int64_t i = t; i < A.H; i += blockDim.x) A.h_out[i] = A.x[int64_t(row) * A.H + i];
    if (!sh[kSlots + 2]) {
        // accepted row path[k] becomes slot base + k, in ascending k (a row never sits above its depth, so no
        // later source is overwritten first)
        const int64_t slot = A.heads * A.head_dim;
        for (int k = 1; k < len; ++k) {
            const int r = sh[k];
            if (r != k) {
                const int64_t dst = (base + k) % A.cap, src = (base + r) % A.cap;
                for (int64_t e = t; e < A.nkv * slot; e += blockDim.x) {
                    const int64_t which = e / slot, w = e % slot, h = w / A.head_dim, d = w % A.head_dim;
                    uint16_t* p = reinterpret_cast<uint16_t*>(A.kv_ptrs[which]);
                    p[(h * A.cap + dst) * A.head_dim + d] = p[(h * A.cap + src) * A.head_dim + d];
                }
            }
            __syncthreads();
        }
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
                                                                                  int(np), mseq);
    CUDA_TRY(cudaGetLastError());
    return MONO_OK;
}

int mono_mtp_prep_verify(const int64_t* st, int64_t* apos, int64_t np, int32_t* aseq, int64_t* vpos,
                         const int64_t* tree_pos, int64_t rows, int32_t* ctl, const int32_t* tree_ctl, int64_t parity,
                         int64_t rope_offset, mono_stream_t stream) {
    MONO_CHECK(st && apos && aseq && vpos && tree_pos && ctl && tree_ctl, "null operand");
    MONO_CHECK(rows >= 1 && rows <= kSlots && np >= 0 && np <= 64, "rows <= 8, positions <= 64");
    mtp_prep_verify_kernel<<<1, 64, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        st, apos, int(np), aseq, vpos, tree_pos, int(rows), ctl, tree_ctl, int(parity), rope_offset);
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
    mtp_accept_kernel<<<1, 1024, 0, reinterpret_cast<cudaStream_t>(stream)>>>(A);
    CUDA_TRY(cudaGetLastError());
    return MONO_OK;
}

}  // extern "C"
