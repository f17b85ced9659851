// Cross-GPU exchange and merge of KV-sharded partials over peer memory (NVLink), in one
// kernel: no NCCL all-gather, no gathered copy.
//
// Each rank owns one exchange region (cudaMalloc'd, shared with the other ranks through
// CUDA IPC handles and mapped into their address spaces):
//   [0, 256)              control: epoch (u32 @0), done (u32 @4), error (i32 @12, read by
//                         dvattn_workspace_status like every workspace's error word),
//                         flags[kMaxRanks] (u32 @64: flags[j] = last call rank j signalled)
//   [256, 256 + P)        slot 0: packed partial (rows x Ev f32 outputs, then rows f32 LSEs)
//   [256 + P, 256 + 2P)   slot 1
// The attention call of each rank writes its partial (f32 output + natural-log LSE) into
// one slot of its own region.  dvattn_lse_merge_peers on every rank then:
//   1. signals "my partial of this call is complete" by storing the call number into its
//      flag on every rank (st.release.sys),
//   2. waits (bounded, 2 s) until every rank's flag in its own region reached the call
//      number (ld.acquire.sys),
//   3. merges all ranks' partials of that slot, read straight from their regions over
//      NVLink, with the log-sum-exp combination of the reference's split-KV reduce
//      (src/kernels/paged_kernel_v21.cuh:347-363).
// The call number lives in the region (epoch); the block that finishes last advances it,
// so the kernel can be captured in a CUDA graph and replayed.  A rank's next attention
// call may overwrite its slot while slower ranks still read it, so consecutive calls
// alternate slots: a rank is at most one call ahead of the others (its next merge waits
// for their signals), so it never writes the slot they read.
// Plain loads and stores only: no TMA and no multicast touch peer memory.
#include <cstring>

#include "decode.cuh"

namespace dvb {

constexpr int kMaxPeerRanks = 8;
constexpr size_t kPeerCtl = 256;

struct PeerArgs {
    int world, rank, slot, Ev;
    long long rows;
    char* region[kMaxPeerRanks];
    void* out;
    float* lse_out;
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__host__ __device__ __forceinline__ size_t peer_slot_bytes(long long rows, int Ev) {
    const size_t b = (size_t)rows * ((size_t)Ev + 1) * sizeof(float);
    return (b + 255) & ~size_t(255);
}

template <class T>
__global__ void __launch_bounds__(256) lse_merge_peers_kernel(PeerArgs a) {
    __shared__ int s_abort;
    // Launched as a programmatic dependent of the attention call's last kernel: the blocks
    // are resident when it finishes and signal at once.  (No launch_dependents here: what
    // follows may read this kernel's output.)
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int tid = threadIdx.x, lane = tid & 31;
    char* own = a.region[a.rank];
    uint32_t* ctl = reinterpret_cast<uint32_t*>(own);
    const uint32_t e = *reinterpret_cast<volatile uint32_t*>(ctl) + 1;  // this call's number
    if (blockIdx.x == 0 && tid < a.world) {
        // The partial was written by the kernels before this one on the stream, so it is in
        // this GPU's L2, where the peers' loads over NVLink are served from; the release store
        // orders the signal after it.  One block signals; the grid is small enough (<= 148
        // blocks) to be resident at once, so no block waits on another's scheduling.
        __threadfence();
        st_release_sys(reinterpret_cast<uint32_t*>(a.region[tid] + 64) + a.rank, e);
    }
    if (tid == 0) {
        int ok = 1;
        const unsigned long long t0 = global_ns();
        for (int j = 0; j < a.world && ok; ++j) {
            const uint32_t* f = reinterpret_cast<const uint32_t*>(own + 64) + j;
            while ((int)(ld_acquire_sys(f) - e) < 0) {
                if (global_ns() - t0 > kWaitNs) {
                    ok = 0;
                    atomicOr(reinterpret_cast<int*>(own + 12), 1);
                    break;
                }
            }
        }
        s_abort = !ok;
    }
    __syncthreads();
    const size_t slot_off = kPeerCtl + (size_t)a.slot * peer_slot_bytes(a.rows, a.Ev);
    const long long rows = a.rows;
    const int Ev = a.Ev;
    for (long long row = blockIdx.x * 8ll + (tid >> 5); row < rows; row += gridDim.x * 8ll) {
        T* orow = static_cast<T*>(a.out) + row * Ev;
        if (s_abort) {  // some rank never signalled: this call's outputs are invalid
            const float nan = __int_as_float(0x7fc00000);
            for (int c = lane; c < Ev; c += 32) orow[c] = Elem<T>::from_f(nan);
            if (a.lse_out && lane == 0) a.lse_out[row] = nan;
            continue;
        }
        // every part's LSE and (for Ev <= 128) its columns in one round of loads
        float l[kMaxPeerRanks];
        float4 v0[kMaxPeerRanks];
        float mx = neg_inf();
#pragma unroll
        for (int j = 0; j < kMaxPeerRanks; ++j) {
            l[j] = neg_inf();
            v0[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (j < a.world) {
                const float* part = reinterpret_cast<const float*>(a.region[j] + slot_off);
                l[j] = part[rows * Ev + row];
                if (4 * lane < Ev) v0[j] = *reinterpret_cast<const float4*>(part + row * Ev + 4 * lane);
            }
        }
#pragma unroll
        for (int j = 0; j < kMaxPeerRanks; ++j) mx = fmaxf(mx, l[j]);
        float den = 0.f;
#pragma unroll
        for (int j = 0; j < kMaxPeerRanks; ++j) {
            l[j] = (j < a.world && l[j] != neg_inf()) ? fast_exp2((l[j] - mx) * kLog2e) : 0.f;
            den += l[j];
        }
        const float inv = den > 0.f ? 1.f / den : 0.f;
        for (int c = 4 * lane; c < Ev; c += 128) {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int j = 0; j < kMaxPeerRanks; ++j) {
                if (j >= a.world || l[j] == 0.f) continue;
                float4 v = v0[j];
                if (c >= 128) {
                    const float* part = reinterpret_cast<const float*>(a.region[j] + slot_off);
                    v = *reinterpret_cast<const float4*>(part + row * Ev + c);
                }
                acc.x += l[j] * v.x; acc.y += l[j] * v.y; acc.z += l[j] * v.z; acc.w += l[j] * v.w;
            }
            store_quad<T>(orow + c, acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
        }
        if (a.lse_out && lane == 0) a.lse_out[row] = den > 0.f ? mx + __logf(den) : neg_inf();
    }
    // the last block to finish advances the call number (every block read it at its start)
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        uint32_t* done = ctl + 1;
        if (atomicAdd(done, 1u) == gridDim.x - 1) {
            *done = 0;
            __threadfence();
            *reinterpret_cast<volatile uint32_t*>(ctl) = e;
        }
    }
}

}  // namespace dvb

using namespace dvb;

extern "C" {

size_t dvattn_peer_region_bytes(long long rows, int Ev) {
    if (rows < 0 || Ev <= 0 || Ev % 4) return 0;
    return kPeerCtl + 2 * peer_slot_bytes(rows, Ev);
}

size_t dvattn_peer_slot_offset(long long rows, int Ev, int slot) {
    if (rows < 0 || Ev <= 0 || Ev % 4 || slot < 0 || slot > 1) return 0;
    return kPeerCtl + (size_t)slot * peer_slot_bytes(rows, Ev);
}

int dvattn_peer_region_alloc(size_t bytes, void** region, void* ipc_handle) {
    if (!region || !ipc_handle || bytes < kPeerCtl) return DVATTN_ERR_INVALID_ARGUMENT;
    *region = nullptr;
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return DVATTN_ERR_CUDA;
    cudaIpcMemHandle_t h;
    if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
        cudaFree(p);
        return DVATTN_ERR_CUDA;
    }
    memcpy(ipc_handle, &h, sizeof(h));
    *region = p;
    return DVATTN_OK;
}

int dvattn_peer_region_open(const void* ipc_handle, void** region) {
    if (!region || !ipc_handle) return DVATTN_ERR_INVALID_ARGUMENT;
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return DVATTN_ERR_CUDA;
    *region = p;
    return DVATTN_OK;
}

int dvattn_peer_region_close(void* region) {
    return region && cudaIpcCloseMemHandle(region) == cudaSuccess ? DVATTN_OK : DVATTN_ERR_CUDA;
}

int dvattn_peer_region_free(void* region) {
    return region && cudaFree(region) == cudaSuccess ? DVATTN_OK : DVATTN_ERR_CUDA;
}

int dvattn_lse_merge_peers(int dtype, int world, int rank, int slot, long long rows, int Ev, void* const* regions,
                           void* out, float* lse_out, dvattn_stream_t stream) {
    if (world < 1 || world > kMaxPeerRanks || rank < 0 || rank >= world || slot < 0 || slot > 1 || rows < 0 ||
        Ev <= 0 || Ev % 4 || !regions || !out)
        return DVATTN_ERR_INVALID_ARGUMENT;
    PeerArgs a{};
    a.world = world;
    a.rank = rank;
    a.slot = slot;
    a.Ev = Ev;
    a.rows = rows;
    for (int j = 0; j < world; ++j) {
        if (!regions[j] || (reinterpret_cast<uintptr_t>(regions[j]) & 255)) return DVATTN_ERR_INVALID_ARGUMENT;
        a.region[j] = static_cast<char*>(regions[j]);
    }
    a.out = out;
    a.lse_out = lse_out;
    long long blocks = (rows + 7) / 8;
    if (blocks < 1) blocks = 1;  // a call with no rows still signals and waits
    if (blocks > 148) blocks = 148;  // one wave on a B200 (rows are grid-strided)
    const void* fn = dtype == DVATTN_FLOAT32   ? (const void*)&lse_merge_peers_kernel<float>
                     : dtype == DVATTN_FLOAT16 ? (const void*)&lse_merge_peers_kernel<__half>
                     : dtype == DVATTN_BFLOAT16 ? (const void*)&lse_merge_peers_kernel<__nv_bfloat16>
                                                : nullptr;
    if (!fn) return DVATTN_ERR_UNSUPPORTED;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)blocks);
    cfg.blockDim = dim3(256);
    cfg.stream = reinterpret_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void* args[] = {&a};
    if (cudaLaunchKernelExC(&cfg, fn, args) != cudaSuccess) return DVATTN_ERR_CUDA;
    return cudaGetLastError() == cudaSuccess ? DVATTN_OK : DVATTN_ERR_CUDA;
}

}  // extern "C"
