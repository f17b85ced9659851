// Varlen chunked prefill on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// A CTA serves one work item: 2 x 128 packed query rows of one sequence and one KV head.
// A row is (token j, head g of the KV group); with G = gqa rounded up to a power of two,
// a 128-row tile holds 128 / G consecutive tokens (row = j * G + g), and the item holds
// two such tiles, A and B.  It streams the sequence's visible keys of every turn in
// 128-key windows:
//   warps 8, 10 producers of K and of V: 3-D TMA page boxes into a 3-stage K and a
//               2-stage V ring; the block-table entries of each window are fetched three
//               windows early by cp.async into a small shared-memory ring
//   warp 9      MMA issuer (one thread): S_A = Q_A K^T, S_B = Q_B K^T into TMEM, then
//               O_A += P_A V, O_B += P_B V with P read from TMEM; completion is signalled
//               by tcgen05.commit on mbarriers.  Issue order S_A(i), PV_B(i-1), S_B(i),
//               PV_A(i) lets the tensor core work for one tile while the other's softmax
//               runs (ping-pong).
//   warps 0..3  softmax of tile A, warps 4..7 softmax of tile B: each thread owns one
//               query row = one TMEM lane; it reads its S row, applies the row's causal
//               bound, keeps the online max/sum (rescaling its O row in TMEM only when
//               the max grows by more than 2^8, so the exponentials stay bounded), and
//               writes P (bf16/f16) over its S row in TMEM for the PV MMA.  At the end it
//               normalises its O row and stores the output row.
// The query rotation of each turn is fused: each softmax thread copies its raw q row
// (cp.async) into the swizzled A-operand tile and rotates it in place.
//
// Reference path replaced: rope_varlen_gpu + varlen_paged_v21::
// dvattn_varlen_paged_attention_gpu (src/rope.cuh:67-114,
// src/kernels/varlen_paged_kernel_v21.cuh:17-428), which runs one CTA per query token and
// re-reads the whole KV prefix for every token on CUDA cores.
#include "decode.cuh"
#include "tma_host.cuh"

#include <cstdio>
#include <cstdlib>

namespace dvb {
namespace pf {

constexpr int M = 128;                 // query rows per tile (two tiles per item)
constexpr int KT = 128;                // keys per window
constexpr int E = 128;                 // head dim (E == Ev)
constexpr int PANEL = 128 * 128;       // one 64-column panel of a 128-row tile (bytes)
constexpr int TILE = 2 * PANEL;        // 128 rows x 128 columns, 16-bit
constexpr int KSTAGES = 3;             // K ring (freed after S = Q K^T)
constexpr int VSTAGES = 2;             // V ring (freed after O += P V)
constexpr size_t OFF_Q = 0;                         // Q_A, Q_B
constexpr size_t OFF_K = OFF_Q + 2 * TILE;
constexpr size_t OFF_V = OFF_K + KSTAGES * TILE;
constexpr size_t OFF_BAR = OFF_V + VSTAGES * TILE;  // 24 mbarrier slots
constexpr size_t OFF_MISC = OFF_BAR + 24 * 8;       // tmem base, abort flag
constexpr size_t OFF_BT = OFF_MISC + 64;  // per producer warp: block-table entries of upcoming windows [8][16]
constexpr size_t SMEM = OFF_BT + 2 * 8 * 16 * 4;
constexpr int BT_AHEAD = 3;               // windows whose block-table entries are in flight
static_assert(SMEM <= 232448, "prefill shared memory exceeds the 227 KB a CTA may use");
constexpr int NT = 11 * 32;
// producer warps 8 (K) and 10 (V), MMA warp 9
constexpr int WARP_PRODUCER = 8, WARP_MMA = 9, WARP_PRODUCER_V = 10;

struct Item {
    int w, t0, nt, hkv;
};

struct Params {
    int F, T, W, Hq, Hkv, gqa, R, BS, maxb, cap;
    int gshift;  // log2 of G, the rows per token in a tile (gqa rounded up to a power of 2)
    int tpi;     // tokens per item = 2 * 128 / G
    long long NB;
    float scale_log2;
    void* out;
    const void* q;
    const float* cos;
    const float* sin;
    const int* loc;
    const int* L;
    const int* bt;
    const int* cu_q;
    float* lse_out;
    float* out_f32;
    Item* items;
    int* header;  // [0] item count, [3] error word (byte offset kErrorWordOffset, as in decode)
    int max_items;
    int stall_tile;  // test hook (DVATTN_TEST_STALL_TILE): CTA 0 never loads this K window; -1: off
};

// ---- tcgen05 helpers -------------------------------------------------------------
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;  // descriptor version for sm_100
    d |= (uint64_t)2 << 61;  // 128-byte swizzle
    return d;
}
// kind::f16 instruction descriptor: f32 accumulate, A/B both f16 or both bf16, A K-major.
__device__ __forceinline__ uint32_t idesc(bool bf16, int m, int n, bool b_mn_major) {
    const uint32_t fmt = bf16 ? 1u : 0u;
    return (1u << 4) | (fmt << 7) | (fmt << 10) | ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t id, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(id), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
        "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])),
        "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
        "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])),
        "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// Registers written by tcgen05.ld hold their values only after tcgen05.wait::ld: this
// empty volatile statement re-defines them after the wait so no use moves above it.
template <int N> __device__ __forceinline__ void reg_fence(float* v) {
#pragma unroll
    for (int i = 0; i < N; ++i) asm volatile("" : "+f"(v[i]));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
// A operand from TMEM (P), B from shared memory (V).
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t id, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b), "r"(id), "r"(accumulate)
        : "memory");
}
// Packed f32x2 arithmetic (one instruction for two lanes of a 64-bit register pair) and a
// three-input max, both native on sm_100.
__device__ __forceinline__ uint64_t f2u(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void u2f(uint64_t r, float& a, float& b) { asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r)); }
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ int turn_vis_pf(int L, int loc, int off, int cap) {
    int v = min(L, loc + 1);
    v = min(v, cap - off);
    return v > 0 ? v : 0;
}

// ---- work list ---------------------------------------------------------------------
// Token t belongs to the first sequence w with t < cu_q[w+1], else to sequence 0
// (varlen_paged_kernel_v21.cuh:40-47).  With a non-decreasing cu_q that gives W + 1
// contiguous segments: segment w = [w ? cu[w] : 0, cu[w+1]) of sequence w, and segment W
// = [cu[W], T) of sequence 0.  Each segment is cut into tpi-token pieces x Hkv items; the
// items are laid out segment by segment in decreasing order of the segment's key count
// (its last token's visible keys over all turns), the last tile of a segment first, so
// the longest work starts first.
__global__ void __launch_bounds__(1024) prefill_prep_kernel(Params p) {
    extern __shared__ long long shl[];  // cost[W+1] | a[W+1] | b[W+1] | start[W+1] | rank[W+1]
    const int tid = threadIdx.x, NS = p.W + 1;
    long long* cost = shl;
    int* sa = reinterpret_cast<int*>(shl + NS);
    int* sb = sa + NS;
    int* start = sb + NS;
    int* rank = start + NS;
    if (tid == 0) {
        int prev = 0;
        for (int w = 0; w < p.W; ++w) {
            const int c = min(max(p.cu_q[w + 1], prev), p.T);
            sa[w] = w ? prev : 0;
            sb[w] = c;
            prev = c;
        }
        sa[p.W] = prev;
        sb[p.W] = p.T;
    }
    __syncthreads();
    for (int s = tid; s < NS; s += 1024) {
        long long c = -1;
        if (sb[s] > sa[s]) {
            const int last = sb[s] - 1;
            c = 0;
            int off = 0;
            for (int f = 0; f < p.F; ++f) {
                c += turn_vis_pf(p.L[f], p.loc[(size_t)f * p.T + last], off, p.cap);
                off += p.L[f];
            }
        }
        cost[s] = c;
    }
    __syncthreads();
    for (int s = tid; s < NS; s += 1024) {
        int r = 0;
        for (int x = 0; x < NS; ++x) r += (cost[x] > cost[s]) || (cost[x] == cost[s] && x < s);
        rank[r] = s;  // rank is a permutation
    }
    __syncthreads();
    if (tid == 0) {
        int acc = 0;
        for (int r = 0; r < NS; ++r) {
            const int s = rank[r];
            start[s] = acc;
            acc += (sb[s] - sa[s] + p.tpi - 1) / p.tpi * p.Hkv;
        }
        p.header[0] = acc < p.max_items ? acc : p.max_items;
        p.header[3] = 0;
    }
    __syncthreads();
    for (int s = tid; s < NS; s += 1024) {
        const int a = sa[s], b = sb[s], ntile = (b - a + p.tpi - 1) / p.tpi;
        int k = start[s];
        for (int q = ntile - 1; q >= 0; --q)
            for (int h = 0; h < p.Hkv; ++h, ++k)
                if (k < p.max_items) p.items[k] = Item{s < p.W ? s : 0, a + q * p.tpi, min(p.tpi, b - a - q * p.tpi), h};
    }
}

// Waits of the producer and MMA warps: a poll every ~100 ns instead of a tight try_wait
// loop, so the two softmax warps on the same SM sub-partitions get the issue slots
// (bounded like mbar_wait).
__device__ __forceinline__ bool mbar_wait_lazy(uint32_t bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    for (;;) {
        __nanosleep(100);
        if (mbar_try_wait(bar, parity)) return true;
        if (global_ns() - t0 > kWaitNs) return false;
    }
}

// ---- the prefill kernel ---------------------------------------------------------
// Keys the item's tokens can see in turn f (the union of their visible ranges), by a
// whole warp: lanes split the tokens, then a max-reduction.
__device__ __forceinline__ int item_span(const Params& p, const Item& it, int f, int off, int lane) {
    const int L = __ldg(p.L + f);
    int v = 0;
    for (int j = lane; j < it.nt; j += 32) v = max(v, turn_vis_pf(L, __ldg(p.loc + (size_t)f * p.T + it.t0 + j), off, p.cap));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// The item's sequence of 128-key windows: turn by turn, the windows covering the union
// of the visible ranges.  Every role walks the same sequence (warp-wide calls).
struct TileSeq {
    int f, off, vmax, win;
    int base, nwin, k;
    bool valid;
    __device__ __forceinline__ void seek(const Params& p, const Item& it, int lane) {
        for (; f < p.F; ++f) {
            vmax = item_span(p, it, f, off, lane);
            if (vmax > 0) {
                base = off & ~(KT - 1);
                nwin = (off + vmax - base + KT - 1) / KT;
                k = 0;
                win = base;
                valid = true;
                return;
            }
            off += __ldg(p.L + f);
        }
        valid = false;
    }
    __device__ __forceinline__ void init(const Params& p, const Item& it, int lane) {
        f = 0;
        off = 0;
        seek(p, it, lane);
    }
    __device__ __forceinline__ void next(const Params& p, const Item& it, int lane) {
        if (++k < nwin) {
            win += KT;
            return;
        }
        off += __ldg(p.L + f);
        ++f;
        seek(p, it, lane);
    }
    __device__ __forceinline__ bool first() const { return k == 0; }
};

template <class T>
__global__ void __launch_bounds__(NT, 1) prefill_kernel(Params p, const __grid_constant__ CUtensorMap tmk,
                                                        const __grid_constant__ CUtensorMap tmv) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const uint32_t s0 = smem_u32(smem);
    if (s0 & 1023) {
        if (tid == 0) atomicOr(p.header + 3, 4);
        return;
    }
    if ((int)blockIdx.x >= p.header[0]) return;
    const Item it = p.items[blockIdx.x];
    const bool bf16 = Elem<T>::dtype == DVATTN_BFLOAT16;

    // mbarriers: k_full[3], k_empty[3], v_full[2], v_empty[2], s_full[2], p_full[2],
    // q_ready[2], o_done
    const uint32_t bar = s0 + (uint32_t)OFF_BAR;
    const uint32_t k_full = bar, k_empty = bar + 24, v_full = bar + 48, v_empty = bar + 64;
    const uint32_t s_full = bar + 80, p_full = bar + 96, q_ready = bar + 112, o_done = bar + 128;
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + OFF_MISC);
    volatile int* sAbort = reinterpret_cast<volatile int*>(smem + OFF_MISC + 8);

    if (tid == 0) {
        for (int s = 0; s < KSTAGES; ++s) {
            mbar_init(k_full + 8 * s, 1);
            mbar_init(k_empty + 8 * s, 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(v_full + 8 * s, 1);
            mbar_init(v_empty + 8 * s, 1);
            mbar_init(s_full + 8 * s, 1);
            mbar_init(p_full + 8 * s, 128);
            mbar_init(q_ready + 8 * s, 128);
        }
        mbar_init(o_done, 1);
        *sAbort = 0;
        fence_mbar_init();
    }
    if (wid == WARP_MMA) {  // TMEM columns: S_A [0,128), S_B [128,256), O_A [256,384), O_B [384,512)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(s0 + (uint32_t)OFF_MISC)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (wid == WARP_PRODUCER || wid == WARP_PRODUCER_V) {
        // =============================== producer ===============================
        if (lane == 0) {
            prefetch_tmap(&tmk);
            prefetch_tmap(&tmv);
        }
        const int* btw = p.bt + (size_t)it.w * p.maxb;
        const int pages = KT / p.BS;  // one page per lane (at most 16)
        // A 128-key window is a 3-D box {64 columns, 1 head, BS rows} per page and 64-column
        // panel; pages outside the window's needed range, outside the block table or the
        // pool load as zeros (out-of-bounds coordinate).  The block-table entries of window
        // w are fetched BT_AHEAD windows early by cp.async into a shared-memory ring (one
        // commit group per window), so their latency stays off the producer's path.
        const uint32_t bt_ring = (uint32_t)(OFF_BT + (wid == WARP_PRODUCER ? 0 : 512));
        auto needed = [&](const TileSeq& q, int& pos) {
            pos = q.win + lane * p.BS;
            return lane < pages && pos + p.BS > q.off && pos < q.off + q.vmax && (pos / p.BS) < p.maxb;
        };
        auto prefetch = [&](const TileSeq& q, int w) {
            int pos;
            if (q.valid && needed(q, pos)) {
                const uint32_t dst = s0 + bt_ring + (uint32_t)(((w & 7) * 16 + lane) * 4);
                asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(dst), "l"(btw + pos / p.BS) : "memory");
            }
            cp_async_commit();
        };
        auto coord = [&](const TileSeq& q, int w) {  // after window w's group completed
            int pos;
            if (!needed(q, pos)) return -2 * p.BS;
            const int page = reinterpret_cast<const int*>(smem + bt_ring)[(w & 7) * 16 + lane];
            return page >= 0 && page < p.NB ? page * p.BS : -2 * p.BS;
        };
        auto load = [&](const CUtensorMap* map, uint32_t dst, uint32_t fullbar, int z) {
            if (lane == 0) mbar_expect_tx(fullbar, (uint32_t)TILE);
            __syncwarp();
            if (lane < pages) {
                const uint32_t d = dst + (uint32_t)(lane * p.BS * 128);
                tma_load_3d(d, map, 0, it.hkv, z, fullbar);
                tma_load_3d(d + PANEL, map, 64, it.hkv, z, fullbar);
            }
        };
        // Warp 8 streams K, warp 10 V, each window into its ring once the window KSTAGES
        // (VSTAGES) before it has been consumed: issuing the 2 x 8 page boxes of a window
        // keeps one warp busy for about as long as the MMAs of half a window take.
        const bool is_k = wid == WARP_PRODUCER;
        const int nst = is_k ? KSTAGES : VSTAGES;
        const uint32_t fullb = is_k ? k_full : v_full, emptyb = is_k ? k_empty : v_empty;
        const uint32_t ring = s0 + (uint32_t)(is_k ? OFF_K : OFF_V);
        const CUtensorMap* map = is_k ? &tmk : &tmv;
        TileSeq kq, la;
        kq.init(p, it, lane);
        la.init(p, it, lane);
        for (int w = 0; w < BT_AHEAD; ++w) {
            prefetch(la, w);
            if (la.valid) la.next(p, it, lane);
        }
        int ik = 0;
        bool ok = true;
        while (kq.valid) {
            const int ks = ik % nst;
            if (*sAbort || (ik >= nst && !mbar_wait_lazy(emptyb + 8 * ks, (ik / nst - 1) & 1))) {
                ok = false;
                break;
            }
            cp_async_wait<BT_AHEAD - 1>();
            const int z = coord(kq, ik);
            prefetch(la, ik + BT_AHEAD);
            if (la.valid) la.next(p, it, lane);
            if (!(is_k && ik == p.stall_tile && blockIdx.x == 0))  // test hook: this K window never lands
                load(map, ring + (uint32_t)(ks * TILE), fullb + 8 * ks, z);
            kq.next(p, it, lane);
            ++ik;
        }
        cp_async_wait<0>();
        if (!ok) {
            if (lane == 0) {
                *sAbort = 1;
                atomicOr(p.header + 3, 1);
            }
            // the windows already requested land before the CTA can exit (bounded waits)
            for (int j = ik > nst ? ik - nst : 0; j < ik; ++j)
                if (!(is_k && j == p.stall_tile && blockIdx.x == 0)) mbar_wait(fullb + 8 * (j % nst), (j / nst) & 1);
        }
    } else if (wid == WARP_MMA) {
        // ================================ MMA ================================
        const uint32_t id_s = idesc(bf16, M, KT, false);
        const uint32_t id_o = idesc(bf16, M, E, true);
        // S_grp = Q_grp K^T over the 128 head dims (8 k-steps of 16)
        // Shared-memory descriptors: the 14-bit start-address field (address >> 4; shared
        // addresses stay below 256 KB, so no carry) advances by offset >> 4, so every MMA's
        // operands are one add from three base descriptors computed once.
        const uint64_t dq0 = sdesc(s0 + (uint32_t)OFF_Q, 16, 1024);
        const uint64_t dk0 = sdesc(s0 + (uint32_t)OFF_K, 16, 1024);
        const uint64_t dv0 = sdesc(s0 + (uint32_t)OFF_V, PANEL, 1024);
        auto issue_s = [&](int grp, int ks) {
            const uint64_t a0 = dq0 + (uint64_t)((grp * TILE) >> 4), b0 = dk0 + (uint64_t)((ks * TILE) >> 4);
            if (lane == 0) {
#pragma unroll
                for (int kk = 0; kk < E / 16; ++kk) {
                    const uint64_t ko = (uint64_t)(((kk >> 2) * PANEL + (kk & 3) * 32) >> 4);
                    umma(tmem + 128 * grp, a0 + ko, b0 + ko, id_s, kk > 0 ? 1u : 0u);
                }
                umma_commit(s_full + 8 * grp);
            }
            __syncwarp();
        };
        // O_grp += P_grp V over the 128 keys; P is packed 2 per column over S_grp's columns
        auto issue_pv = [&](int grp, int vs, bool acc) {
            const uint64_t b0 = dv0 + (uint64_t)((vs * TILE) >> 4);
            const uint32_t d = tmem + 256 + 128 * grp, a = tmem + 128 * grp;
            if (lane == 0) {
#pragma unroll
                for (int kk = 0; kk < KT / 16; ++kk)
                    umma_ts(d, a + 8 * kk, b0 + (uint64_t)((kk * 16 * 128) >> 4), id_o, (acc || kk > 0) ? 1u : 0u);
            }
            __syncwarp();
        };
        auto commit = [&](uint32_t b) {
            if (lane == 0) umma_commit(b);
            __syncwarp();
        };
        TileSeq ts;
        ts.init(p, it, lane);
        int i = 0, turn = 0;
        bool ok = true;
        for (; ts.valid; ts.next(p, it, lane), ++i) {
            const int ks = i % KSTAGES, vs = i & 1;
            const bool first = ts.first();
            if (!mbar_wait_lazy(k_full + 8 * ks, (i / KSTAGES) & 1)) { ok = false; break; }
            if (first && !mbar_wait_lazy(q_ready, turn & 1)) { ok = false; break; }
            tc_fence_after();
            issue_s(0, ks);
            // the softmax hand-offs (p_full) are polled without a pause: they are on every
            // tile's critical path (softmax -> PV -> next S)
            if (i > 0) {
                if (!mbar_wait(p_full + 8, (i - 1) & 1)) { ok = false; break; }
                tc_fence_after();
                issue_pv(1, vs ^ 1, i - 1 > 0);
                commit(v_empty + 8 * (vs ^ 1));
            }
            if (first && !mbar_wait_lazy(q_ready + 8, turn & 1)) { ok = false; break; }
            tc_fence_after();
            issue_s(1, ks);
            commit(k_empty + 8 * ks);
            if (!mbar_wait_lazy(v_full + 8 * vs, (i >> 1) & 1)) { ok = false; break; }
            if (!mbar_wait(p_full, i & 1)) { ok = false; break; }
            tc_fence_after();
            issue_pv(0, vs, i > 0);
            if (first) ++turn;
        }
        if (ok && i > 0) {
            if (mbar_wait_lazy(p_full + 8, (i - 1) & 1)) {
                tc_fence_after();
                issue_pv(1, (i - 1) & 1, i - 1 > 0);
            } else {
                ok = false;
            }
        }
        if (!ok && lane == 0) {
            *sAbort = 1;
            atomicOr(p.header + 3, 2);
        }
        // o_done: every MMA of the item has completed (the epilogue and the TMEM release
        // wait on it)
        if (lane == 0) umma_commit(o_done);
        __syncwarp();
        mbar_wait(o_done, 0);
    } else {
        // ============================== softmax ==============================
        const int grp = wid >> 2;                 // tile A (0) or B (1)
        const int r = (wid & 3) * 32 + lane;     // query row == TMEM lane
        const uint32_t lane_base = (uint32_t)((wid & 3) * 32) << 16;
        const uint32_t tS = tmem + lane_base + 128 * grp;
        const uint32_t tO = tmem + lane_base + 256 + 128 * grp;
        const int tok = (grp << (7 - p.gshift)) + (r >> p.gshift);  // token index within the item
        const int g = r & ((1 << p.gshift) - 1);
        const bool row_ok = tok < it.nt && g < p.gqa;
        const int t = it.t0 + (row_ok ? tok : 0);
        const int hq = it.hkv * p.gqa + (row_ok ? g : 0);
        const float sl2 = p.scale_log2;
        const uint32_t qtile = (uint32_t)(OFF_Q + grp * TILE);
        float m = neg_inf(), l = 0.f;  // running max (log2 units, stepped) and sum
        int i = 0;
        bool ok = true;
        const int hp = p.R >> 1;
        TileSeq ts;
        ts.init(p, it, lane);
        int lim = 0, vend = 0;
        for (; ts.valid; ts.next(p, it, lane), ++i) {
            const int f = ts.f, off = ts.off, win = ts.win, st = i & 1;
            if (ts.first()) {
                // ---- rotate this row's q for turn f into the A tile (in place) ----
                const T* qrow = static_cast<const T*>(p.q) + ((size_t)t * p.Hq + hq) * E;
#pragma unroll
                for (int ch = 0; ch < E / 8; ++ch)
                    cp_async16_zfill(s0 + qtile + (uint32_t)((ch >> 3) * PANEL + r * 128 + (((ch & 7) ^ (r & 7)) << 4)),
                                     qrow + ch * 8, row_ok ? 16 : 0);
                cp_async_commit();
                cp_async_wait<0>();
                if (row_ok) {
                    const float* cr = p.cos + ((size_t)f * p.T + t) * hp;
                    const float* sr = p.sin + ((size_t)f * p.T + t) * hp;
                    for (int c = 0; c < hp / 8; ++c) {
                        const int c2 = c + hp / 8;
                        uint4* xa = reinterpret_cast<uint4*>(smem + qtile + (c >> 3) * PANEL + r * 128 + (((c & 7) ^ (r & 7)) << 4));
                        uint4* ya = reinterpret_cast<uint4*>(smem + qtile + (c2 >> 3) * PANEL + r * 128 + (((c2 & 7) ^ (r & 7)) << 4));
                        uint4 xv = *xa, yv = *ya;
                        const T* x = reinterpret_cast<const T*>(&xv);
                        const T* y = reinterpret_cast<const T*>(&yv);
                        uint32_t lo[4], hi[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const float c0 = __ldg(cr + c * 8 + 2 * u), c1 = __ldg(cr + c * 8 + 2 * u + 1);
                            const float z0 = __ldg(sr + c * 8 + 2 * u), z1 = __ldg(sr + c * 8 + 2 * u + 1);
                            const float x0 = Elem<T>::to_f(x[2 * u]), x1 = Elem<T>::to_f(x[2 * u + 1]);
                            const float y0 = Elem<T>::to_f(y[2 * u]), y1 = Elem<T>::to_f(y[2 * u + 1]);
                            lo[u] = Elem<T>::pack2(x0 * c0 - y0 * z0, x1 * c1 - y1 * z1);
                            hi[u] = Elem<T>::pack2(y0 * c0 + x0 * z0, y1 * c1 + x1 * z1);
                        }
                        *xa = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                        *ya = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                    }
                }
                fence_proxy_async_smem();
                mbar_arrive(q_ready + 8 * grp);
                // visible window of this row in turn f: logical positions [off, lim]
                lim = row_ok ? off + turn_vis_pf(__ldg(p.L + f), __ldg(p.loc + (size_t)f * p.T + t), off, p.cap) - 1
                             : off - 1;
                vend = off + ts.vmax;
            }
            {
                {
                    if (!mbar_wait(s_full + 8 * grp, i & 1)) { ok = false; break; }
                    tc_fence_after();
                    float sv[KT];
#pragma unroll
                    for (int c = 0; c < KT / 32; ++c) tmem_ld32(tS + 32 * c, *reinterpret_cast<float(*)[32]>(sv + 32 * c));
                    tmem_wait_ld();
                    reg_fence<KT>(sv);
                    const int lo = off - win, hi = lim - win;  // visible columns [lo, hi]
                    if (!__all_sync(0xffffffffu, lo <= 0 && hi >= KT - 1)) {
#pragma unroll
                        for (int c = 0; c < KT; ++c)
                            if (c < lo || c > hi) sv[c] = neg_inf();
                    }
                    float mx[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) mx[u] = sv[u];
#pragma unroll
                    for (int c = 8; c < KT; c += 16)
#pragma unroll
                        for (int u = 0; u < 8; ++u) mx[u] = fmax3(mx[u], sv[c + u], sv[c + 8 + u < KT ? c + 8 + u : c + u]);
                    const float mxs = fmax3(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7])) * sl2;
                    // the reference point moves only when the max grows by more than 8
                    // (a factor 256 in the exponentials); the result is exact either way
                    const float mnew = mxs > m + 8.f ? mxs : m;
                    const float alpha = mnew == m ? 1.f : ex2(m - mnew);
                    const float mu = mnew == neg_inf() ? 0.f : mnew;
                    const uint64_t sc2 = f2u(sl2, sl2), nmu2 = f2u(-mu, -mu);
                    uint64_t ps2[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
                    for (int c = 0; c < KT / 32; ++c) {
                        uint32_t pk[16];
#pragma unroll
                        for (int u = 0; u < 16; ++u) {
                            float x0, x1;
                            u2f(ffma2(f2u(sv[32 * c + 2 * u], sv[32 * c + 2 * u + 1]), sc2, nmu2), x0, x1);
                            const float e0 = ex2(x0), e1 = ex2(x1);
                            const uint64_t e2 = f2u(e0, e1);
                            ps2[u & 3] = fadd2(ps2[u & 3], e2);
                            pk[u] = Elem<T>::pack2(e0, e1);
                        }
                        tmem_st16(tS + 16 * c, pk);
                    }
                    float psum;
                    {
                        float a0, a1, b0, b1;
                        u2f(fadd2(fadd2(ps2[0], ps2[1]), fadd2(ps2[2], ps2[3])), a0, a1);
                        (void)b0;
                        (void)b1;
                        psum = a0 + a1;
                    }
                    l = l * alpha + psum;
                    m = mnew;
                    if (i > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
                        // O holds the PV of every earlier window (their MMAs completed
                        // before S of this window was signalled)
#pragma unroll 1
                        for (int c = 0; c < E / 32; ++c) {
                            float ov[32];
                            tmem_ld32(tO + 32 * c, ov);
                            tmem_wait_ld();
                            reg_fence<32>(ov);
#pragma unroll
                            for (int u = 0; u < 32; ++u) ov[u] *= alpha;
                            tmem_st32(tO + 32 * c, ov);
                        }
                    }
                    if (grp == 0 && (win < off || win + KT > vend)) {
                        // V rows of this window outside [off, vend) may hold another turn's
                        // or uninitialised pool data: zero them (P is 0 there, 0 * NaN is NaN)
                        if (!mbar_wait(v_full + 8 * st, (i >> 1) & 1)) { ok = false; break; }
                        const int pos = win + r;
                        if (pos < off || pos >= vend) {
                            uint8_t* vrow = smem + OFF_V + st * TILE + r * 128;
#pragma unroll
                            for (int c = 0; c < 8; ++c) {
                                *reinterpret_cast<uint4*>(vrow + c * 16) = make_uint4(0u, 0u, 0u, 0u);
                                *reinterpret_cast<uint4*>(vrow + PANEL + c * 16) = make_uint4(0u, 0u, 0u, 0u);
                            }
                        }
                        fence_proxy_async_smem();
                    }
                    tmem_wait_st();
                    tc_fence_before();
                    mbar_arrive(p_full + 8 * grp);
                }
            }
        }
        if (!ok && lane == 0) {
            *sAbort = 1;
            atomicOr(p.header + 3, 8);
        }
        // ---- epilogue: O / l -> output ----
        const bool done = mbar_wait(o_done, 0);
        tc_fence_after();
        if (ok && done && i > 0) {
            const float inv = l > 0.f ? 1.f / l : 0.f;
            T* op = static_cast<T*>(p.out) + ((size_t)t * p.Hq + hq) * E;
            float* o32 = p.out_f32 ? p.out_f32 + ((size_t)t * p.Hq + hq) * E : nullptr;
#pragma unroll 1
            for (int c = 0; c < E / 32; ++c) {
                float ov[32];
                tmem_ld32(tO + 32 * c, ov);
                tmem_wait_ld();
                reg_fence<32>(ov);
                if (row_ok) {
#pragma unroll
                    for (int u = 0; u < 32; ++u) ov[u] *= inv;
#pragma unroll
                    for (int u = 0; u < 32; u += 8) {
                        uint4 pk;
                        pk.x = Elem<T>::pack2(ov[u], ov[u + 1]);
                        pk.y = Elem<T>::pack2(ov[u + 2], ov[u + 3]);
                        pk.z = Elem<T>::pack2(ov[u + 4], ov[u + 5]);
                        pk.w = Elem<T>::pack2(ov[u + 6], ov[u + 7]);
                        *reinterpret_cast<uint4*>(op + 32 * c + u) = pk;
                        if (o32) {
                            *reinterpret_cast<float4*>(o32 + 32 * c + u) = make_float4(ov[u], ov[u + 1], ov[u + 2], ov[u + 3]);
                            *reinterpret_cast<float4*>(o32 + 32 * c + u + 4) =
                                make_float4(ov[u + 4], ov[u + 5], ov[u + 6], ov[u + 7]);
                        }
                    }
                }
            }
            if (row_ok && p.lse_out) p.lse_out[(size_t)t * p.Hq + hq] = l > 0.f ? (m + __log2f(l)) * kLn2 : neg_inf();
        }
        if (row_ok && !(ok && done)) {
            // this item gave up on a bounded wait: its rows are marked invalid (NaN)
            const float nan = __int_as_float(0x7fc00000);
            T* op = static_cast<T*>(p.out) + ((size_t)t * p.Hq + hq) * E;
            const uint32_t hn = Elem<T>::pack2(nan, nan);
            for (int c = 0; c < E; c += 8) *reinterpret_cast<uint4*>(op + c) = make_uint4(hn, hn, hn, hn);
            if (p.out_f32)
                for (int c = 0; c < E; c += 4)
                    *reinterpret_cast<float4*>(p.out_f32 + ((size_t)t * p.Hq + hq) * E + c) = make_float4(nan, nan, nan, nan);
            if (p.lse_out) p.lse_out[(size_t)t * p.Hq + hq] = nan;
        }
        if (row_ok && ok && done && i == 0) {  // no visible key at all: zeros
            T* op = static_cast<T*>(p.out) + ((size_t)t * p.Hq + hq) * E;
            for (int c = 0; c < E; c += 8) *reinterpret_cast<uint4*>(op + c) = make_uint4(0u, 0u, 0u, 0u);
            if (p.out_f32)
                for (int c = 0; c < E; c += 4)
                    *reinterpret_cast<float4*>(p.out_f32 + ((size_t)t * p.Hq + hq) * E + c) = make_float4(0.f, 0.f, 0.f, 0.f);
            if (p.lse_out) p.lse_out[(size_t)t * p.Hq + hq] = neg_inf();
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (wid == WARP_MMA)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
}

}  // namespace pf

// ---------------------------------------------------------------------------------
static int prefill_gshift(const dvattn_varlen_args* v) {
    const int gqa = v->Hq / v->Hkv;
    int s = 0;
    while ((1 << s) < gqa) ++s;
    return s;
}
static int prefill_tokens_per_item(const dvattn_varlen_args* v) { return 2 * (pf::M >> prefill_gshift(v)); }

// DVATTN_PREFILL=0 keeps every varlen call on the split-KV decode schedule; =1 uses the
// tensor-core prefill for every shape it supports, however small; unset: large calls only.
static int prefill_mode() {
    const char* e = getenv("DVATTN_PREFILL");
    return e && e[0] == '0' ? 0 : e && e[0] == '1' ? 1 : 2;
}

bool prefill_eligible(const dvattn_varlen_args* v) {
    const int mode = prefill_mode();
    if (mode == 0) return false;
    if (!v || (v->dtype != DVATTN_FLOAT16 && v->dtype != DVATTN_BFLOAT16)) return false;
    if (v->E != 128 || v->Ev != 128 || v->Hkv <= 0 || v->Hq < v->Hkv || v->Hq % v->Hkv || v->Hq / v->Hkv > 16) return false;
    if (v->R % 16 || v->R > v->E) return false;
    const int BS = v->block_size;
    if (!(BS == 8 || BS == 16 || BS == 32 || BS == 64 || BS == 128)) return false;
    if (v->num_blocks <= 0 || v->num_blocks * (long long)BS > 0x7fffffffLL) return false;
    // enough items to fill the GPU; short prefills go through the split-KV decode schedule
    return mode == 1 || (long long)v->T * v->Hkv >= 148LL * prefill_tokens_per_item(v);
}

// DVATTN_TEST_STALL_TILE=<i>: tests only (see the decode launcher); read once per process.
static int prefill_stall_hook() {
    static const int t = [] {
        const char* e = getenv("DVATTN_TEST_STALL_TILE");
        return e && *e ? atoi(e) : -1;
    }();
    return t;
}

static int prefill_max_items(const dvattn_varlen_args* v) {
    return (v->T / prefill_tokens_per_item(v) + v->W + 1) * v->Hkv;
}

size_t prefill_workspace_size(const dvattn_varlen_args* v) {
    return 256 + sizeof(pf::Item) * (size_t)prefill_max_items(v);
}

int prefill_launch(const dvattn_varlen_args* v, void* workspace, size_t wbytes, cudaStream_t stream, int phase) {
    const size_t need = prefill_workspace_size(v);
    if (!workspace || wbytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255)) return DVATTN_ERR_WORKSPACE;
    pf::Params p{};
    p.F = v->F; p.T = v->T; p.W = v->W; p.Hq = v->Hq; p.Hkv = v->Hkv; p.gqa = v->Hq / v->Hkv; p.R = v->R;
    p.gshift = prefill_gshift(v); p.tpi = prefill_tokens_per_item(v);
    p.BS = v->block_size; p.maxb = v->max_blocks_per_seq;
    const long long cap = (long long)v->max_blocks_per_seq * v->block_size;
    p.cap = cap > 0x7fffffffLL ? 0x7fffffff : (int)cap;
    p.NB = v->num_blocks;
    p.scale_log2 = v->scale * kLog2e;
    p.out = v->out; p.q = v->queries; p.cos = v->cosines; p.sin = v->sines; p.loc = v->locations;
    p.L = v->fragment_lengths; p.bt = v->block_tables; p.cu_q = v->cu_seqlens_q;
    p.lse_out = v->lse_out; p.out_f32 = v->out_f32;
    p.header = static_cast<int*>(workspace);
    p.items = reinterpret_cast<pf::Item*>(static_cast<char*>(workspace) + 256);
    p.max_items = prefill_max_items(v);
    p.stall_tile = prefill_stall_hook();

    const size_t prep_smem = (sizeof(long long) + 4 * sizeof(int)) * ((size_t)p.W + 1);
    if (prep_smem > 48 * 1024) return DVATTN_ERR_UNSUPPORTED;
    if (phase == DVATTN_PHASE_ALL || phase == DVATTN_PHASE_SCHEDULE) pf::prefill_prep_kernel<<<1, 1024, prep_smem, stream>>>(p);
    if (phase != DVATTN_PHASE_ALL && phase != DVATTN_PHASE_ATTEND) return cudaGetLastError() == cudaSuccess ? DVATTN_OK : DVATTN_ERR_CUDA;

    alignas(64) CUtensorMap mk, mv;
    const long long tokens = p.NB * p.BS;
    if (!encode_cache_map(&mk, v->k_cache, v->dtype, 128, p.Hkv, tokens, p.BS) ||
        !encode_cache_map(&mv, v->v_cache, v->dtype, 128, p.Hkv, tokens, p.BS))
        return DVATTN_ERR_CUDA;
    const void* fn = v->dtype == DVATTN_BFLOAT16 ? (const void*)&pf::prefill_kernel<__nv_bfloat16>
                                                 : (const void*)&pf::prefill_kernel<__half>;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pf::SMEM) != cudaSuccess)
        return DVATTN_ERR_CUDA;
    void* args[] = {&p, &mk, &mv};
    const cudaError_t e = cudaLaunchKernel(fn, dim3(p.max_items), dim3(pf::NT), args, pf::SMEM, stream);
    if (e != cudaSuccess) {
        if (getenv("DVATTN_DEBUG")) fprintf(stderr, "dvattn prefill launch: %s\n", cudaGetErrorString(e));
        return DVATTN_ERR_CUDA;
    }
    return cudaGetLastError() == cudaSuccess ? DVATTN_OK : DVATTN_ERR_CUDA;
}

}  // namespace dvb
