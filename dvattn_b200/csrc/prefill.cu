// Varlen chunked prefill on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// A CTA serves one work item: 8 consecutive packed query tokens of one sequence and one
// KV head, i.e. M = 128 query rows (token j = row / 16, head g = row % 16).  It streams
// that sequence's visible keys of every turn in 128-key windows:
//   warp 0      producer: block-table lookups + 3-D TMA page boxes into a 2-stage ring
//   warp 1      MMA issuer (one thread): S = Q K^T into TMEM (double-buffered), then
//               O += P V into TMEM, completion signalled by tcgen05.commit on mbarriers
//   warps 2..5  softmax: each thread owns one query row = one TMEM lane; it reads its S
//               row, applies the row's causal bound, keeps the online max/sum, rescales
//               its O row in TMEM when the max moves, writes P (bf16/f16) to shared
//               memory for the PV MMA, and finally normalises and stores the output.
// The query rotation of each turn is fused: each softmax thread copies its raw q row
// (cp.async) into the swizzled A-operand tile and rotates it in place.
//
// Reference path replaced: rope_varlen_gpu + varlen_paged_v21::
// dvattn_varlen_paged_attention_gpu (src/rope.cuh:67-114,
// src/kernels/varlen_paged_kernel_v21.cuh:17-428), which runs one CTA per query token and
// re-reads the whole KV prefix for every token on CUDA cores.
#include "decode.cuh"
#include "tma_host.cuh"

#include <cstdlib>

namespace dvb {
namespace pf {

constexpr int QT = 8;                  // query tokens per work item
constexpr int M = 128;                 // query rows (QT x 16 heads)
constexpr int KT = 128;                // keys per window
constexpr int E = 128;                 // head dim (E == Ev)
constexpr int PANEL = 128 * 128;       // one 64-column panel of a 128-row tile (bytes)
constexpr int TILE = 2 * PANEL;        // 128 rows x 128 columns, 16-bit
constexpr int STAGES = 2;
constexpr size_t OFF_Q = 0;
constexpr size_t OFF_P = OFF_Q + TILE;
constexpr size_t OFF_K = OFF_P + TILE;
constexpr size_t OFF_V = OFF_K + STAGES * TILE;
constexpr size_t OFF_BAR = OFF_V + STAGES * TILE;  // 16 mbarriers
constexpr size_t OFF_MISC = OFF_BAR + 16 * 8;      // tmem base, abort flag
constexpr size_t SMEM = OFF_MISC + 64;
constexpr int NT = 6 * 32;

struct Item {
    int w, t0, nt, hkv;
};

struct Params {
    int F, T, W, Hq, Hkv, gqa, R, BS, maxb, cap;
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
    int* header;  // [0] item count, [1] error word
    int max_items;
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
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(id), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
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

__device__ __forceinline__ int turn_vis_pf(int L, int loc, int off, int cap) {
    int v = min(L, loc + 1);
    v = min(v, cap - off);
    return v > 0 ? v : 0;
}

// ---- work list ---------------------------------------------------------------------
// Token t belongs to the first sequence w with t < cu_q[w+1], else to sequence 0
// (varlen_paged_kernel_v21.cuh:40-47).  With a non-decreasing cu_q that gives W + 1
// contiguous segments: segment w = [w ? cu[w] : 0, cu[w+1]) of sequence w, and segment W
// = [cu[W], T) of sequence 0.  Each segment is cut into 8-token tiles x Hkv items; the
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
            acc += (sb[s] - sa[s] + QT - 1) / QT * p.Hkv;
        }
        p.header[0] = acc < p.max_items ? acc : p.max_items;
        p.header[1] = 0;
    }
    __syncthreads();
    for (int s = tid; s < NS; s += 1024) {
        const int a = sa[s], b = sb[s], ntile = (b - a + QT - 1) / QT;
        int k = start[s];
        for (int q = ntile - 1; q >= 0; --q)
            for (int h = 0; h < p.Hkv; ++h, ++k)
                if (k < p.max_items) p.items[k] = Item{s < p.W ? s : 0, a + q * QT, min(QT, b - a - q * QT), h};
    }
}

// ---- the prefill kernel ---------------------------------------------------------
template <class T>
__global__ void __launch_bounds__(NT, 1) prefill_kernel(Params p, const __grid_constant__ CUtensorMap tmk,
                                                        const __grid_constant__ CUtensorMap tmv) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const uint32_t s0 = smem_u32(smem);
    if (s0 & 1023) {
        if (tid == 0) atomicOr(p.header + 1, 4);
        return;
    }
    if ((int)blockIdx.x >= p.header[0]) return;
    const Item it = p.items[blockIdx.x];
    const bool bf16 = Elem<T>::dtype == DVATTN_BFLOAT16;

    const uint32_t bar = s0 + (uint32_t)OFF_BAR;
    const uint32_t kv_full = bar, kv_empty = bar + 16, s_full = bar + 32, s_free = bar + 48;
    const uint32_t p_full = bar + 64, o_done = bar + 72, q_ready = bar + 80, fin = bar + 88;
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + OFF_MISC);
    volatile int* sAbort = reinterpret_cast<volatile int*>(smem + OFF_MISC + 8);

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(kv_full + 8 * s, 1);
            mbar_init(kv_empty + 8 * s, 1);
            mbar_init(s_full + 8 * s, 1);
            mbar_init(s_free + 8 * s, 4);
        }
        mbar_init(p_full, 128);
        mbar_init(o_done, 1);
        mbar_init(q_ready, 128);
        mbar_init(fin, 1);
        *sAbort = 0;
        fence_mbar_init();
    }
    if (wid == 1) {  // TMEM: S0 [0,128), S1 [128,256), O [256,384)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(s0 + (uint32_t)OFF_MISC)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // per-turn window plan, identical in every role: the union of the tokens' visible
    // ranges, in 128-aligned windows of logical positions
    auto turn_span = [&](int f, int off) {
        int vmax = 0;
        for (int j = 0; j < it.nt; ++j)
            vmax = max(vmax, turn_vis_pf(p.L[f], p.loc[(size_t)f * p.T + it.t0 + j], off, p.cap));
        return vmax;
    };

    if (wid == 0) {
        // =============================== producer ===============================
        if (lane == 0) {
            prefetch_tmap(&tmk);
            prefetch_tmap(&tmv);
        }
        const int* btw = p.bt + (size_t)it.w * p.maxb;
        const int pages = KT / p.BS;
        const uint32_t bytes = 2u * TILE;
        int i = 0, off = 0;
        bool ok = true;
        for (int f = 0; f < p.F && ok; ++f) {
            const int L = p.L[f];
            const int vmax = turn_span(f, off);
            if (vmax > 0) {
                for (int win = off & ~(KT - 1); win < off + vmax && ok; win += KT, ++i) {
                    const int st = i & 1;
                    if (*sAbort || (i >= STAGES && !mbar_wait(kv_empty + 8 * st, ((i >> 1) - 1) & 1))) {
                        ok = false;
                        break;
                    }
                    if (lane == 0) mbar_expect_tx(kv_full + 8 * st, bytes);
                    __syncwarp();
                    for (int j = lane; j < pages; j += 32) {
                        const int pos = win + j * p.BS;  // first logical position of page j
                        const bool need = pos + p.BS > off && pos < off + vmax && (pos / p.BS) < p.maxb;
                        int page = need ? __ldg(btw + pos / p.BS) : -1;
                        const bool valid = need && (p.NB <= 0 || (page >= 0 && page < p.NB));
                        const int z = valid ? page * p.BS : -2 * p.BS;  // out of bounds -> zeros
                        const uint32_t dk = s0 + (uint32_t)(OFF_K + st * TILE + j * p.BS * 128);
                        const uint32_t dv = s0 + (uint32_t)(OFF_V + st * TILE + j * p.BS * 128);
#pragma unroll
                        for (int pn = 0; pn < 2; ++pn) {
                            tma_load_3d(dk + pn * PANEL, &tmk, pn * 64, it.hkv, z, kv_full + 8 * st);
                            tma_load_3d(dv + pn * PANEL, &tmv, pn * 64, it.hkv, z, kv_full + 8 * st);
                        }
                    }
                }
            }
            off += L;
        }
        if (!ok && lane == 0) {
            *sAbort = 1;
            atomicOr(p.header + 1, 1);
        }
    } else if (wid == 1) {
        // ================================ MMA ================================
        const uint32_t id_s = idesc(bf16, M, KT, false);
        const uint32_t id_o = idesc(bf16, M, E, true);
        int i = 0, off = 0, turn = 0;
        bool ok = true, any = false;
        int pend = -1;  // tile whose PV is still to be issued
        auto issue_pv = [&](int tile) {
            if (!mbar_wait(p_full, tile & 1)) return false;
            tc_fence_after();
            if (lane == 0) {
                const int st = tile & 1;
#pragma unroll
                for (int kk = 0; kk < KT / 16; ++kk) {
                    const uint64_t a = sdesc(s0 + (uint32_t)(OFF_P + (kk >> 2) * PANEL + (kk & 3) * 32), 16, 1024);
                    const uint64_t b = sdesc(s0 + (uint32_t)(OFF_V + st * TILE + kk * 16 * 128), PANEL, 1024);
                    umma(tmem + 256, a, b, id_o, (tile > 0 || kk > 0) ? 1u : 0u);
                }
                umma_commit(o_done);
                umma_commit(kv_empty + 8 * st);
            }
            __syncwarp();
            return true;
        };
        for (int f = 0; f < p.F && ok; ++f) {
            const int vmax = turn_span(f, off);
            if (vmax > 0) {
                if (!mbar_wait(q_ready, turn & 1)) { ok = false; break; }
                ++turn;
                for (int win = off & ~(KT - 1); win < off + vmax; win += KT, ++i) {
                    const int st = i & 1;
                    if (!mbar_wait(kv_full + 8 * st, (i >> 1) & 1)) { ok = false; break; }
                    if (i >= 2 && !mbar_wait(s_free + 8 * st, ((i >> 1) - 1) & 1)) { ok = false; break; }
                    tc_fence_after();
                    if (lane == 0) {
#pragma unroll
                        for (int kk = 0; kk < E / 16; ++kk) {
                            const uint64_t a = sdesc(s0 + (uint32_t)(OFF_Q + (kk >> 2) * PANEL + (kk & 3) * 32), 16, 1024);
                            const uint64_t b =
                                sdesc(s0 + (uint32_t)(OFF_K + st * TILE + (kk >> 2) * PANEL + (kk & 3) * 32), 16, 1024);
                            umma(tmem + 128 * st, a, b, id_s, kk > 0 ? 1u : 0u);
                        }
                        umma_commit(s_full + 8 * st);
                    }
                    __syncwarp();
                    any = true;
                    if (pend >= 0 && !issue_pv(pend)) { ok = false; break; }
                    pend = i;
                }
            }
            off += p.L[f];
        }
        if (ok && pend >= 0 && !issue_pv(pend)) ok = false;
        if (!ok && lane == 0) {
            *sAbort = 1;
            atomicOr(p.header + 1, 2);
        }
        (void)any;
        // all MMAs issued by this thread have completed before TMEM is released
        if (lane == 0) umma_commit(fin);
        __syncwarp();
        mbar_wait(fin, 0);
    } else {
        // ============================== softmax ==============================
        const int r = (wid & 3) * 32 + lane;     // query row == TMEM lane
        const uint32_t lane_base = (uint32_t)((wid & 3) * 32) << 16;
        const int j = r >> 4, g = r & 15;        // token, head within the KV group
        const bool row_ok = j < it.nt && g < p.gqa;
        const int t = it.t0 + j;
        const int hq = it.hkv * p.gqa + g;
        const float sl2 = p.scale_log2;
        float m = neg_inf(), l = 0.f;
        int i = 0, off = 0;
        bool ok = true;
        const int hp = p.R >> 1;
        for (int f = 0; f < p.F && ok; ++f) {
            const int L = p.L[f];
            const int vmax = turn_span(f, off);
            if (vmax > 0) {
                // ---- rotate this row's q for turn f into the A tile (in place) ----
                {
                    const T* qrow = static_cast<const T*>(p.q) + ((size_t)(row_ok ? t : 0) * p.Hq + (row_ok ? hq : 0)) * E;
                    for (int ch = 0; ch < E / 8; ++ch)
                        cp_async16_zfill(s0 + (uint32_t)(OFF_Q + (ch >> 3) * PANEL + r * 128 + (((ch & 7) ^ (r & 7)) << 4)),
                                         qrow + ch * 8, row_ok ? 16 : 0);
                    cp_async_commit();
                    cp_async_wait<0>();
                    if (row_ok) {
                        const float* cr = p.cos + ((size_t)f * p.T + t) * hp;
                        const float* sr = p.sin + ((size_t)f * p.T + t) * hp;
                        for (int c = 0; c < hp / 8; ++c) {
                            uint4* xa = reinterpret_cast<uint4*>(smem + OFF_Q + (c >> 3) * PANEL + r * 128 +
                                                                 (((c & 7) ^ (r & 7)) << 4));
                            const int c2 = c + hp / 8;
                            uint4* ya = reinterpret_cast<uint4*>(smem + OFF_Q + (c2 >> 3) * PANEL + r * 128 +
                                                                 (((c2 & 7) ^ (r & 7)) << 4));
                            uint4 xv = *xa, yv = *ya;
                            const T* x = reinterpret_cast<const T*>(&xv);
                            const T* y = reinterpret_cast<const T*>(&yv);
                            uint32_t lo[4], hi[4];
#pragma unroll
                            for (int u = 0; u < 4; ++u) {
                                const float c0 = cr[c * 8 + 2 * u], c1 = cr[c * 8 + 2 * u + 1];
                                const float z0 = sr[c * 8 + 2 * u], z1 = sr[c * 8 + 2 * u + 1];
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
                    mbar_arrive(q_ready);
                }
                // this row's last visible logical position in turn f (-1: none)
                const int lim = row_ok ? off + turn_vis_pf(L, p.loc[(size_t)f * p.T + t], off, p.cap) - 1 : -1;
                const int vend = off + vmax;  // keys of this turn past the union's end are zeroed in V
                for (int win = off & ~(KT - 1); win < off + vmax; win += KT, ++i) {
                    const int st = i & 1;
                    if (!mbar_wait(s_full + 8 * st, (i >> 1) & 1)) { ok = false; break; }
                    tc_fence_after();
                    float sv[KT];
#pragma unroll
                    for (int c = 0; c < KT / 32; ++c) tmem_ld32(tmem + lane_base + 128 * st + 32 * c, *reinterpret_cast<float(*)[32]>(sv + 32 * c));
                    tmem_wait_ld();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(s_free + 8 * st);
                    // mask: logical position win + c visible iff off <= pos <= lim
                    float mx = neg_inf();
#pragma unroll
                    for (int c = 0; c < KT; ++c) {
                        const int pos = win + c;
                        const float x = (pos >= off && pos <= lim) ? sv[c] * sl2 : neg_inf();
                        sv[c] = x;
                        mx = fmaxf(mx, x);
                    }
                    const float mn = fmaxf(m, mx);
                    const float mu = mn == neg_inf() ? 0.f : mn;
                    const float alpha = fast_exp2(m - mu);
                    float ps = 0.f;
#pragma unroll
                    for (int c = 0; c < KT; ++c) {
                        sv[c] = fast_exp2(sv[c] - mu);
                        ps += sv[c];
                    }
                    l = l * alpha + ps;
                    m = mn;
                    // PV of the previous window must be done before O and P are touched
                    if (i > 0) {
                        if (!mbar_wait(o_done, (i - 1) & 1)) { ok = false; break; }
                        tc_fence_after();
                        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
                            for (int c = 0; c < E / 32; ++c) {
                                float ov[32];
                                tmem_ld32(tmem + lane_base + 256 + 32 * c, ov);
                                tmem_wait_ld();
#pragma unroll
                                for (int u = 0; u < 32; ++u) ov[u] *= alpha;
                                tmem_st32(tmem + lane_base + 256 + 32 * c, ov);
                            }
                            tmem_wait_st();
                        }
                    }
                    // P row -> A tile of the PV MMA (keys along K, 128-byte swizzle)
#pragma unroll
                    for (int ch = 0; ch < KT / 8; ++ch) {
                        uint4 pk;
                        pk.x = Elem<T>::pack2(sv[8 * ch + 0], sv[8 * ch + 1]);
                        pk.y = Elem<T>::pack2(sv[8 * ch + 2], sv[8 * ch + 3]);
                        pk.z = Elem<T>::pack2(sv[8 * ch + 4], sv[8 * ch + 5]);
                        pk.w = Elem<T>::pack2(sv[8 * ch + 6], sv[8 * ch + 7]);
                        *reinterpret_cast<uint4*>(smem + OFF_P + (ch >> 3) * PANEL + r * 128 + (((ch & 7) ^ (r & 7)) << 4)) = pk;
                    }
                    // V rows of this window outside [off, vend) may hold another turn's or
                    // uninitialised pool data: zero them (P is 0 there, but 0 * NaN is NaN)
                    {
                        const int pos = win + r;  // this thread's key row of the window
                        if (pos < off || pos >= vend) {
                            uint8_t* vrow = smem + OFF_V + st * TILE + r * 128;
                            for (int c = 0; c < 8; ++c) {
                                *reinterpret_cast<uint4*>(vrow + c * 16) = make_uint4(0u, 0u, 0u, 0u);
                                *reinterpret_cast<uint4*>(vrow + PANEL + c * 16) = make_uint4(0u, 0u, 0u, 0u);
                            }
                        }
                    }
                    fence_proxy_async_smem();
                    tc_fence_before();
                    mbar_arrive(p_full);
                }
            }
            off += L;
        }
        if (!ok) {
            if (lane == 0) {
                *sAbort = 1;
                atomicOr(p.header + 1, 8);
            }
        } else if (i > 0) {
            // ---- epilogue: O / l -> output ----
            if (mbar_wait(o_done, (i - 1) & 1)) {
                tc_fence_after();
                const float inv = l > 0.f ? 1.f / l : 0.f;
                T* op = static_cast<T*>(p.out) + ((size_t)t * p.Hq + hq) * E;
#pragma unroll 1
                for (int c = 0; c < E / 32; ++c) {
                    float ov[32];
                    tmem_ld32(tmem + lane_base + 256 + 32 * c, ov);
                    tmem_wait_ld();
                    if (row_ok) {
#pragma unroll
                        for (int u = 0; u < 32; u += 8) {
                            uint4 pk;
                            pk.x = Elem<T>::pack2(ov[u] * inv, ov[u + 1] * inv);
                            pk.y = Elem<T>::pack2(ov[u + 2] * inv, ov[u + 3] * inv);
                            pk.z = Elem<T>::pack2(ov[u + 4] * inv, ov[u + 5] * inv);
                            pk.w = Elem<T>::pack2(ov[u + 6] * inv, ov[u + 7] * inv);
                            *reinterpret_cast<uint4*>(op + 32 * c + u) = pk;
                            if (p.out_f32) {
                                float* o32 = p.out_f32 + ((size_t)t * p.Hq + hq) * E + 32 * c + u;
                                *reinterpret_cast<float4*>(o32) = make_float4(ov[u] * inv, ov[u + 1] * inv, ov[u + 2] * inv, ov[u + 3] * inv);
                                *reinterpret_cast<float4*>(o32 + 4) =
                                    make_float4(ov[u + 4] * inv, ov[u + 5] * inv, ov[u + 6] * inv, ov[u + 7] * inv);
                            }
                        }
                    }
                }
                if (row_ok && p.lse_out) p.lse_out[(size_t)t * p.Hq + hq] = l > 0.f ? (m + __log2f(l)) * kLn2 : neg_inf();
            }
        }
        if (row_ok && i == 0) {  // no visible key at all: zeros
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
    if (wid == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
}

}  // namespace pf

// ---------------------------------------------------------------------------------
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
    if (v->E != 128 || v->Ev != 128 || v->Hkv <= 0 || v->Hq % v->Hkv || v->Hq / v->Hkv > 16) return false;
    if (v->R % 16 || v->R > v->E) return false;
    const int BS = v->block_size;
    if (!(BS == 8 || BS == 16 || BS == 32 || BS == 64 || BS == 128)) return false;
    if (v->num_blocks <= 0 || v->num_blocks * (long long)BS > 0x7fffffffLL) return false;
    // enough 8-token tiles to fill the GPU; short prefills go through the decode schedule
    return mode == 1 || (long long)(v->T / pf::QT) * v->Hkv >= 2 * 148;
}

static int prefill_max_items(const dvattn_varlen_args* v) { return (v->T / pf::QT + v->W + 1) * v->Hkv; }

size_t prefill_workspace_size(const dvattn_varlen_args* v) {
    return 256 + sizeof(pf::Item) * (size_t)prefill_max_items(v);
}

int prefill_launch(const dvattn_varlen_args* v, void* workspace, size_t wbytes, cudaStream_t stream) {
    const size_t need = prefill_workspace_size(v);
    if (!workspace || wbytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255)) return DVATTN_ERR_WORKSPACE;
    pf::Params p{};
    p.F = v->F; p.T = v->T; p.W = v->W; p.Hq = v->Hq; p.Hkv = v->Hkv; p.gqa = v->Hq / v->Hkv; p.R = v->R;
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

    const size_t prep_smem = (sizeof(long long) + 4 * sizeof(int)) * ((size_t)p.W + 1);
    if (prep_smem > 48 * 1024) return DVATTN_ERR_UNSUPPORTED;
    pf::prefill_prep_kernel<<<1, 1024, prep_smem, stream>>>(p);

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
    if (cudaLaunchKernel(fn, dim3(p.max_items), dim3(pf::NT), args, pf::SMEM, stream) != cudaSuccess)
        return DVATTN_ERR_CUDA;
    return cudaGetLastError() == cudaSuccess ? DVATTN_OK : DVATTN_ERR_CUDA;
}

}  // namespace dvb
