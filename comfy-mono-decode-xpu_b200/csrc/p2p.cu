// One-shot all-reduce (sum) of bf16 rows between two GPUs over NVLink peer memory (the tensor-parallel variant's
// residual sum: [M, 4096] bf16 after every row-sharded projection).
//
// Each rank owns a receive area in its own memory (two buffers, by call parity) and an array of per-CTA arrival
// counters; the peer's are mapped into this process (CUDA IPC). CTA b of a call: stores its chunk of the local
// input into the peer's receive buffer (plain 16-byte stores over NVLink), fences at system scope, adds 1 to the
// peer's counter b (release); waits until its own counter b reaches the call number (acquire, bounded); then
// writes out = bf16(float(local) + float(received)) for its chunk. Addition is commutative, so both ranks get the
// same bits. The call number comes from a per-CTA count in this rank's memory, so the kernel needs no host scalar
// and replays in CUDA graphs. The two buffers alternate: a rank in call i + 1 has seen the peer's call-i data, so
// the peer has finished call i - 1 (kernel order on each stream) and its buffer i + 1 mod 2 is free.
// Plain loads and stores only (no TMA). Waits give up after 1 s of %globaltimer and set the error word.
#include <cstring>

#include "launch.h"

namespace mono {

constexpr int kArThreads = 256, kArCtas = 16;

__device__ __forceinline__ void red_release_sys_add(unsigned* p, unsigned v) {
    asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_relaxed_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

struct Ar2Args {
    const uint16_t* in;   // [n] bf16, this rank's partial
    uint16_t* out;        // [n] bf16 (may be in)
    uint16_t* peer_recv;  // the peer's receive area: 2 x cap bf16
    const uint16_t* my_recv;
    unsigned* peer_arrive;  // the peer's counters [kArCtas]
    const unsigned* my_arrive;
    unsigned* my_calls;     // this rank's call count per CTA [kArCtas]
    int64_t n, cap;
};

__global__ void __launch_bounds__(kArThreads) allreduce2_kernel(const Ar2Args A) {
    __shared__ unsigned call;
    __shared__ int ok;
    const int b = blockIdx.x;
    if (threadIdx.x == 0) call = A.my_calls[b];
    __syncthreads();
    const size_t buf = size_t(call & 1u) * size_t(A.cap);
    // the CTA's chunk in 16-byte pieces (n % 8 == 0)
    const int64_t pieces = A.n >> 3, per = (pieces + gridDim.x - 1) / gridDim.x;
    const int64_t p0 = int64_t(b) * per, p1 = p0 + per < pieces ? p0 + per : pieces;
    const uint4* in4 = reinterpret_cast<const uint4*>(A.in);
    uint4* dst4 = reinterpret_cast<uint4*>(A.peer_recv + buf);
    for (int64_t p = p0 + threadIdx.x; p < p1; p += blockDim.x) dst4[p] = __ldcg(in4 + p);
    __syncthreads();
    if (threadIdx.x == 0) {
        // the release orders the CTA's chunk stores (seen by this thread through the barrier above) before the
        // arrival, at system scope
        red_release_sys_add(A.peer_arrive + b, 1u);
        const unsigned want = call + 1u;
        bool good = true;
        if (ld_relaxed_sys(A.my_arrive + b) < want) {
            const unsigned long long t0 = globaltimer();
            for (uint32_t i = 1;; ++i) {
                if (ld_relaxed_sys(A.my_arrive + b) >= want) break;
                if ((i & 255) == 0 && globaltimer() - t0 > kWaitLimitNs) {
                    set_device_error(DEV_PEER_TIMEOUT);
                    good = false;
                    break;
                }
            }
        }
        asm volatile("fence.acq_rel.sys;" ::: "memory");  // the peer's chunk after its arrival
        ok = good;
        A.my_calls[b] = want;
    }
    __syncthreads();
    if (!ok) return;
    const uint4* rcv4 = reinterpret_cast<const uint4*>(A.my_recv + buf);
    uint4* out4 = reinterpret_cast<uint4*>(A.out);
    for (int64_t p = p0 + threadIdx.x; p < p1; p += blockDim.x) {
        const uint4 a = __ldcg(in4 + p), r = __ldcg(rcv4 + p);
        const uint32_t ua[4] = {a.x, a.y, a.z, a.w}, ur[4] = {r.x, r.y, r.z, r.w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float lo = __fadd_rn(__uint_as_float(ua[j] << 16), __uint_as_float(ur[j] << 16));
            const float hi = __fadd_rn(__uint_as_float(ua[j] & 0xFFFF0000u), __uint_as_float(ur[j] & 0xFFFF0000u));
            o[j] = uint32_t(f32_to_bf16_bits(lo)) | (uint32_t(f32_to_bf16_bits(hi)) << 16);
        }
        out4[p] = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

}  // namespace mono

using namespace mono;

extern "C" {

size_t mono_allreduce2_area_bytes(int64_t cap) {
    // two receive buffers of cap bf16 values, then the arrival counters (256-byte aligned)
    return (size_t(2) * cap * 2 + 255) / 256 * 256 + 256;
}

int mono_p2p_area_alloc(size_t bytes, void** ptr_out) {
    MONO_CHECK(ptr_out && bytes > 0 && bytes <= (size_t(1) << 30), "0 < bytes <= 1 GiB");
    void* p = nullptr;
    CUDA_TRY(cudaMalloc(&p, bytes));  // its own allocation: an IPC handle names the whole of it
    const cudaError_t e = cudaMemset(p, 0, bytes);
    if (e != cudaSuccess) {
        cudaFree(p);
        return fail(MONO_ECUDA, "cudaMemset: %s", cudaGetErrorString(e));
    }
    *ptr_out = p;
    return MONO_OK;
}

int mono_p2p_area_free(void* ptr) {
    MONO_CHECK(ptr, "null pointer");
    CUDA_TRY(cudaFree(ptr));
    return MONO_OK;
}

int mono_ipc_handle(void* ptr, void* handle_out, size_t handle_bytes) {
    MONO_CHECK(ptr && handle_out && handle_bytes >= sizeof(cudaIpcMemHandle_t), "pointer and a 64-byte handle buffer");
    cudaIpcMemHandle_t h;
    CUDA_TRY(cudaIpcGetMemHandle(&h, ptr));
    memcpy(handle_out, &h, sizeof(h));
    return MONO_OK;
}

int mono_ipc_open(const void* handle, size_t handle_bytes, void** ptr_out) {
    MONO_CHECK(handle && ptr_out && handle_bytes >= sizeof(cudaIpcMemHandle_t), "a 64-byte handle and an output");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    CUDA_TRY(cudaIpcOpenMemHandle(ptr_out, h, cudaIpcMemLazyEnablePeerAccess));
    return MONO_OK;
}

int mono_ipc_close(void* ptr) {
    MONO_CHECK(ptr, "null pointer");
    CUDA_TRY(cudaIpcCloseMemHandle(ptr));
    return MONO_OK;
}

int mono_allreduce2_bf16(const void* in, void* out, int64_t n, void* my_area, void* peer_area, int64_t cap,
                         unsigned* my_calls, mono_stream_t stream) {
    MONO_CHECK(in && out && my_area && peer_area && my_calls, "null operand");
    MONO_CHECK(n >= 8 && n % 8 == 0 && n <= cap, "8 <= n <= cap, n % 8 == 0");
    MONO_CHECK(aligned(in, 16) && aligned(out, 16) && aligned(my_area, 256) && aligned(peer_area, 256),
               "16-byte aligned rows, 256-byte aligned areas");
    const size_t bufs = (size_t(2) * cap * 2 + 255) / 256 * 256;
    Ar2Args A{};
    A.in = static_cast<const uint16_t*>(in);
    A.out = static_cast<uint16_t*>(out);
    A.peer_recv = static_cast<uint16_t*>(peer_area);
    A.my_recv = static_cast<const uint16_t*>(my_area);
    A.peer_arrive = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(peer_area) + bufs);
    A.my_arrive = reinterpret_cast<const unsigned*>(static_cast<const uint8_t*>(my_area) + bufs);
    A.my_calls = my_calls;
    A.n = n;
    A.cap = cap;
    allreduce2_kernel<<<kArCtas, kArThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(A);
    CUDA_TRY(cudaGetLastError());
    return MONO_OK;
}

}  // extern "C"
