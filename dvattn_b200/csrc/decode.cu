// Paged GQA decode for sm_100a: fused per-turn query RoPE, page-indirect K/V streaming
// with cp.async (16-byte, zero-filled past the visible keys), QK^T and PV on tensor
// cores with the (up to) 16 query heads of one KV head packed as the M=16 of
// mma.sync.m16n8k16, online base-2 softmax, and a balanced split-KV schedule whose
// pieces are merged by log-sum-exp.
//
// Reference path replaced: rope_gpu (src/rope.cuh:2-65) + paged_v21::
// dvattn_paged_attention_gpu_kernel21 / dvattn_paged_attention_reduce_kernel /
// dvattn_paged_attention_gpu (src/kernels/paged_kernel_v21.cuh:17-431).
#include "decode.cuh"
#include "schedule.cuh"
#include "tma_host.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>
#include <vector>

namespace dvb {


// ----------------------------------------------------------------------------------
// query rotation of one (row ws, KV head, turn f) into shared memory.
// rotated[e] = q[e]*c[e] - q[e+R/2]*s[e]          for e < R/2
//            = q[e]*c[e-R/2] + q[e-R/2]*s[e-R/2]  for R/2 <= e < R
//            = q[e]                                for e >= R
// with c, s the first R/2 entries of the (f, ws) cos/sin row (src/rope.cuh:24-45), math
// in f32, rounded once to T (python/dvattn/attention.py:82-88).
// ----------------------------------------------------------------------------------
template <class T>
__device__ __forceinline__ float rotated_elem(const T* qrow, const float* cr, const float* sr, int e, int R) {
    const float x = Elem<T>::to_f(qrow[e]);
    const int h = R >> 1;
    if (e < h) return x * cr[e] - Elem<T>::to_f(qrow[e + h]) * sr[e];
    if (e < R) return x * cr[e - h] + Elem<T>::to_f(qrow[e - h]) * sr[e - h];
    return x;
}


// Rotated q of query row `ws`, turn `f`, for KV heads [h0, h0 + nh) into the swizzled
// buffer sQ = [head][64-col panel][16 rows][128 B] (rows g >= gqa are zero).  Threads
// tid < nth share the work; every global load of a thread is issued before any use, so
// a rotation costs one memory latency.  Fast path when R/2 is a multiple of 8: a thread
// owns a chunk of 8 rotary pairs (chunks c and c + R/16), or one pass-through chunk.
template <class T, int E, int MAXT>
__device__ __forceinline__ void rotate_q_rows(const PagedParams& p, int ws, int f, int h0, int nh, uint8_t* sQ, int tid,
                                              int nth, float* sCS, int bar_id) {
    constexpr int CH = E / 8;
    const int w = ws / p.S, s = ws - w * p.S;
    const float* cr = p.cos + ((size_t)f * p.WS + ws) * p.cs_stride;
    const float* sr = p.sin + ((size_t)f * p.WS + ws) * p.cs_stride;
    const int R = p.R, hp = R >> 1;
    auto dst = [&](int row, int ch) {
        return reinterpret_cast<uint4*>(sQ + ((row >> 4) * (E / 64) + (ch >> 3)) * 2048 + (row & 15) * 128 +
                                        (((ch & 7) ^ (row & 7)) << 4));
    };
    auto qrow_of = [&](int row) {
        const int hq = (h0 + (row >> 4)) * p.gqa + (row & 15);
        return static_cast<const T*>(p.q) + (size_t)f * p.q_turn_stride + (((size_t)w * p.Hq + hq) * p.S + s) * E;
    };
    if ((hp & 7) == 0 && ((reinterpret_cast<uintptr_t>(cr) | reinterpret_cast<uintptr_t>(sr)) & 15) == 0) {
        const int npair = hp >> 3, npass = (E - R) >> 3;
        const int per_row = npair + npass;
        const int ntask = nh * 16 * per_row;
        // one round of loads: the cos/sin rows into sCS, the q chunks into registers
        for (int k = tid; k < 2 * (hp >> 2); k += nth) {
            const int half = k / (hp >> 2), jj = k - half * (hp >> 2);
            reinterpret_cast<float4*>(sCS + half * hp)[jj] = reinterpret_cast<const float4*>(half ? sr : cr)[jj];
        }
        uint4 a[MAXT], b[MAXT];
#pragma unroll
        for (int k = 0; k < MAXT; ++k) {
            const int t = tid + k * nth;
            a[k] = b[k] = make_uint4(0u, 0u, 0u, 0u);
            if (t < ntask) {
                const int row = t / per_row, j = t - row * per_row;
                if ((row & 15) < p.gqa) {
                    const T* q = qrow_of(row);
                    if (j < npair) {
                        a[k] = *reinterpret_cast<const uint4*>(q + j * 8);
                        b[k] = *reinterpret_cast<const uint4*>(q + j * 8 + hp);
                    } else {
                        a[k] = *reinterpret_cast<const uint4*>(q + R + (j - npair) * 8);
                    }
                }
            }
        }
        named_bar_sync(bar_id, nth);
#pragma unroll
        for (int k = 0; k < MAXT; ++k) {
            const int t = tid + k * nth;
            if (t >= ntask) break;
            const int row = t / per_row, j = t - row * per_row;
            if (j < npair) {
                const T* x = reinterpret_cast<const T*>(&a[k]);
                const T* y = reinterpret_cast<const T*>(&b[k]);
                const float4 c0 = reinterpret_cast<const float4*>(sCS + j * 8)[0];
                const float4 c1 = reinterpret_cast<const float4*>(sCS + j * 8)[1];
                const float4 s0 = reinterpret_cast<const float4*>(sCS + hp + j * 8)[0];
                const float4 s1 = reinterpret_cast<const float4*>(sCS + hp + j * 8)[1];
                const float cc[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
                const float ss[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
                uint32_t lo[4], hi[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const float x0 = Elem<T>::to_f(x[2 * u]), x1 = Elem<T>::to_f(x[2 * u + 1]);
                    const float y0 = Elem<T>::to_f(y[2 * u]), y1 = Elem<T>::to_f(y[2 * u + 1]);
                    lo[u] = Elem<T>::pack2(x0 * cc[2 * u] - y0 * ss[2 * u], x1 * cc[2 * u + 1] - y1 * ss[2 * u + 1]);
                    hi[u] = Elem<T>::pack2(y0 * cc[2 * u] + x0 * ss[2 * u], y1 * cc[2 * u + 1] + x1 * ss[2 * u + 1]);
                }
                *dst(row, j) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                *dst(row, j + (hp >> 3)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
            } else {
                *dst(row, (R >> 3) + (j - npair)) = a[k];
            }
        }
    } else {
        for (int t = tid; t < nh * 16 * CH; t += nth) {
            const int row = t / CH, ch = t - row * CH;
            uint32_t pk[4] = {0u, 0u, 0u, 0u};
            if ((row & 15) < p.gqa) {
                const T* q = qrow_of(row);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int e = ch * 8 + 2 * u;
                    pk[u] = Elem<T>::pack2(rotated_elem(q, cr, sr, e, R), rotated_elem(q, cr, sr, e + 1, R));
                }
            }
            *dst(row, ch) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
    }
}

// In-place variant for the row kernel: cp.async copies every raw q chunk straight into
// the swizzled slot its rotated value will occupy (rows g >= gqa are zero-filled), then
// each thread rotates the pairs it owns -- both slots of a pair belong to one thread, so
// the update is in place with no register staging.  The caller follows with a barrier.
template <class T, int E>
__device__ __forceinline__ void rotate_q_inplace(const PagedParams& p, int ws, int f, int nh, uint8_t* sQ, int tid,
                                                 int nth, float* sCS, int bar_id) {
    constexpr int CH = E / 8;
    const int w = ws / p.S, s = ws - w * p.S;
    const float* cr = p.cos + ((size_t)f * p.WS + ws) * p.cs_stride;
    const float* sr = p.sin + ((size_t)f * p.WS + ws) * p.cs_stride;
    const int R = p.R, hp = R >> 1;
    if (!((hp & 7) == 0 && ((reinterpret_cast<uintptr_t>(cr) | reinterpret_cast<uintptr_t>(sr)) & 15) == 0)) {
        rotate_q_rows<T, E, 1>(p, ws, f, 0, nh, sQ, tid, nth, sCS, bar_id);  // general path (scalar)
        return;
    }
    auto slot = [&](int row, int ch) -> uint8_t* {
        return sQ + ((row >> 4) * (E / 64) + (ch >> 3)) * 2048 + (row & 15) * 128 + (((ch & 7) ^ (row & 7)) << 4);
    };
    for (int t = tid; t < nh * 16 * CH; t += nth) {
        const int row = t / CH, ch = t - row * CH;
        const int g = row & 15;
        const T* q = static_cast<const T*>(p.q) + (size_t)f * p.q_turn_stride +
                     (((size_t)w * p.Hq + (row >> 4) * p.gqa + (g < p.gqa ? g : 0)) * p.S + s) * E + ch * 8;
        cp_async16_zfill(smem_u32(slot(row, ch)), q, g < p.gqa ? 16 : 0);
    }
    for (int k = tid; k < 2 * (hp >> 2); k += nth) {
        const int half = k / (hp >> 2), jj = k - half * (hp >> 2);
        cp_async16_zfill(smem_u32(sCS + half * hp + jj * 4), (half ? sr : cr) + jj * 4, 16);
    }
    cp_async_commit();
    cp_async_wait<0>();
    named_bar_sync(bar_id, nth);
    const int npair = hp >> 3;
    for (int t = tid; t < nh * 16 * npair; t += nth) {
        const int row = t / npair, j = t - row * npair;
        uint4* xa = reinterpret_cast<uint4*>(slot(row, j));
        uint4* ya = reinterpret_cast<uint4*>(slot(row, j + npair));
        uint4 xv = *xa, yv = *ya;
        const T* x = reinterpret_cast<const T*>(&xv);
        const T* y = reinterpret_cast<const T*>(&yv);
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const float c0 = sCS[j * 8 + 2 * u], c1 = sCS[j * 8 + 2 * u + 1];
            const float s0 = sCS[hp + j * 8 + 2 * u], s1 = sCS[hp + j * 8 + 2 * u + 1];
            const float x0 = Elem<T>::to_f(x[2 * u]), x1 = Elem<T>::to_f(x[2 * u + 1]);
            const float y0 = Elem<T>::to_f(y[2 * u]), y1 = Elem<T>::to_f(y[2 * u + 1]);
            lo[u] = Elem<T>::pack2(x0 * c0 - y0 * s0, x1 * c1 - y1 * s1);
            hi[u] = Elem<T>::pack2(y0 * c0 + x0 * s0, y1 * c1 + x1 * s1);
        }
        *xa = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        *ya = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    }
}

// L2 prefetch of what rotate_q_rows will read for (ws, f): the q rows of all heads and
// the cos/sin rows (bulk prefetch wants 16-byte aligned, 16-byte multiple ranges).
template <class T, int E>
__device__ __forceinline__ void prefetch_rotation_inputs(const PagedParams& p, int ws, int f, int lane) {
    const int w = ws / p.S, s = ws - w * p.S;
    if (p.S == 1) {
        // the row's q block (Hq * E elements, contiguous): one L2 prefetch per 128-B line
        const char* q = reinterpret_cast<const char*>(static_cast<const T*>(p.q) + (size_t)f * p.q_turn_stride +
                                                      (size_t)w * p.Hq * E);
        const int lines = (int)((p.Hq * E * sizeof(T) + 127) / 128);
        for (int i = lane; i < lines; i += 32) asm volatile("prefetch.global.L2 [%0];" ::"l"(q + (size_t)i * 128));
    } else {
        for (int hq = lane; hq < p.Hq; hq += 32) {
            const T* q = static_cast<const T*>(p.q) + (size_t)f * p.q_turn_stride + (((size_t)w * p.Hq + hq) * p.S + s) * E;
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(q), "r"((uint32_t)(E * sizeof(T))) : "memory");
        }
    }
    const int hp = p.R >> 1;
    if (lane == 1 && hp > 0 && (hp & 3) == 0) {
        const float* cr = p.cos + ((size_t)f * p.WS + ws) * p.cs_stride;
        const float* sr = p.sin + ((size_t)f * p.WS + ws) * p.cs_stride;
        if (((reinterpret_cast<uintptr_t>(cr) | reinterpret_cast<uintptr_t>(sr)) & 15) == 0) {
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(cr), "r"((uint32_t)(hp * 4)) : "memory");
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(sr), "r"((uint32_t)(hp * 4)) : "memory");
        }
    }
}

// ==================================================================================
// tensor-core kernel (f16 / bf16)
// ==================================================================================
template <class T, int E, int WARPS, int STAGES>
struct TcCfg {
    static constexpr int NT = WARPS * 32;
    static constexpr int TILE = WARPS * 16;        // keys per pipeline stage
    static constexpr int ROWB = E * 2;             // bytes of one K/V/Q row
    static constexpr int CPR = ROWB / 16;          // 16-byte chunks per row
    static constexpr int STAGE_BYTES = TILE * ROWB;
    static constexpr int KS = E / 16;              // k16 steps of QK^T
    static constexpr bool QREG = (E <= 128);       // keep Q fragments in registers
    static constexpr size_t SMEM = 2ull * STAGES * STAGE_BYTES + 16 * ROWB + 16 * E * 4 + WARPS * 16 * 2 * 4 + 16 * 4;
};

template <class T, int E, int WARPS, int STAGES>
__global__ void __launch_bounds__(WARPS * 32) decode_tc_kernel(PagedParams p) {
    using C = TcCfg<T, E, WARPS, STAGES>;
    constexpr int NT = C::NT, TILE = C::TILE, ROWB = C::ROWB, CPR = C::CPR;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* sK = smem;
    uint8_t* sV = sK + STAGES * C::STAGE_BYTES;
    uint8_t* sQ = sV + STAGES * C::STAGE_BYTES;
    float* sO = reinterpret_cast<float*>(sQ + 16 * ROWB);
    float* sML = sO + 16 * E;           // [WARPS][16][2]
    float* sLse = sML + WARPS * 16 * 2; // [16]

    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    // the merge kernel may launch now: its CTAs wait (griddepcontrol.wait) for this grid
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // programmatic dependent of the schedule kernel: wait for its header and prefix sums
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const DecodeSched sch = *p.sched;
    const int c = blockIdx.x;
    if (c >= sch.n_eff) return;
    const long long u0 = p.cstart[c], u1 = p.cstart[c + 1];
    if (u0 >= u1) return;
    const int ws0 = find_row<NT>(p, u0);

    const T* __restrict__ kc = static_cast<const T*>(p.k);
    const T* __restrict__ vc = static_cast<const T*>(p.v);
    const uint32_t sK0 = smem_u32(sK), sV0 = smem_u32(sV), sQ0 = smem_u32(sQ);

    // ---- producer: issue one tile of K and V rows into stage `st` ----
    auto issue = [&](const TileDesc& d, int st) {
        const int* btw = p.nfrag ? nullptr : p.bt + (size_t)row_block_table(p, d.ws) * p.maxb;
        FragDesc fd{};
        if (p.nfrag) fd = p.frag[d.f];
        const uint32_t kd = sK0 + st * C::STAGE_BYTES, vd = sV0 + st * C::STAGE_BYTES;
#pragma unroll
        for (int i = 0; i < TILE * CPR / NT; ++i) {
            const int idx = i * NT + tid;
            const int r = idx / CPR, ch = idx % CPR;
            const T* ks = kc;
            const T* vs = vc;
            int bytes = 0;
            if (r < d.n) {
                const int pos = d.pos0 + r;
                if (p.nfrag) {  // contiguous fragment of turn d.f
                    const int l = pos - d.off;
                    if (l < fd.rows) {
                        const size_t row =
                            ((size_t)(d.ws / p.S) * fd.wmul * p.Hkv + d.hkv) * (size_t)fd.rows + (size_t)l;
                        ks = static_cast<const T*>(fd.k) + row * E + ch * 8;
                        vs = static_cast<const T*>(fd.v) + row * E + ch * 8;
                        bytes = 16;
                    }
                } else {
                    const int page = __ldg(btw + pos / p.BS);
                    if (p.NB <= 0 || (page >= 0 && page < p.NB)) {
                        const size_t row = ((size_t)page * p.BS + pos % p.BS) * p.Hkv + d.hkv;
                        ks = kc + row * E + ch * 8;
                        vs = vc + row * E + ch * 8;
                        bytes = 16;
                    }
                }
            }
            cp_async16_zfill(kd + swz(r, ch, ROWB), ks, bytes);
            cp_async16_zfill(vd + swz(r, ch, ROWB), vs, bytes);
        }
    };

    for (int i = tid; i < 16 * E; i += NT) sO[i] = 0.f;

    TileIter<TILE> prod, cons;
    prod.init(p, ws0, p.P[ws0], u0, u1);
    cons = prod;
#pragma unroll
    for (int st = 0; st < STAGES - 1; ++st) {
        TileDesc d;
        if (prod.next(p, d)) issue(d, st);
        cp_async_commit();
    }

    // ---- consumer state (per warp: 16 rows = query heads) ----
    uint32_t qf[C::QREG ? C::KS : 1][4];
    float o[E / 8][4];
    float m0 = 0.f, m1 = 0.f, l0 = 0.f, l1 = 0.f;
    int st_c = 0, st_p = STAGES - 1;
    TileDesc d;
    while (cons.next(p, d)) {
        if (d.new_seg) {
            m0 = m1 = neg_inf();
            l0 = l1 = 0.f;
#pragma unroll
            for (int j = 0; j < E / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
        }
        if (d.new_turn) {
            __syncthreads();
            const int w = d.ws / p.S;
            const float* cr = p.cos + ((size_t)d.f * p.WS + d.ws) * p.cs_stride;
            const float* sr = p.sin + ((size_t)d.f * p.WS + d.ws) * p.cs_stride;
            const int s = d.ws - w * p.S;
            for (int idx = tid; idx < 16 * CPR; idx += NT) {
                const int g = idx / CPR, ch = idx % CPR;
                uint32_t pk[4] = {0u, 0u, 0u, 0u};
                if (g < p.gqa) {
                    const int hq = d.hkv * p.gqa + g;
                    const T* qrow = static_cast<const T*>(p.q) + (size_t)d.f * p.q_turn_stride +
                                    (((size_t)w * p.Hq + hq) * p.S + s) * E;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int e = ch * 8 + 2 * j;
                        pk[j] = Elem<T>::pack2(rotated_elem(qrow, cr, sr, e, p.R), rotated_elem(qrow, cr, sr, e + 1, p.R));
                    }
                }
                *reinterpret_cast<uint4*>(sQ + swz(g, ch, ROWB)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            }
            __syncthreads();
            if constexpr (C::QREG) {
#pragma unroll
                for (int kk = 0; kk < C::KS; ++kk)
                    ldsm_x4(sQ0 + swz((lane & 7) + ((lane >> 3) & 1) * 8, kk * 2 + (lane >> 4), ROWB), qf[kk][0],
                            qf[kk][1], qf[kk][2], qf[kk][3]);
            }
        }

        {
            TileDesc dp;
            if (prod.next(p, dp)) issue(dp, st_p);
            cp_async_commit();
        }
        cp_async_wait<STAGES - 1>();
        __syncthreads();

        const int rb = wid * 16;
        const int nv = d.n - rb;
        if (nv > 0) {
            const uint32_t kb = sK0 + st_c * C::STAGE_BYTES, vb = sV0 + st_c * C::STAGE_BYTES;
            float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
            for (int kk = 0; kk < C::KS; ++kk) {
                uint32_t a[4];
                if constexpr (C::QREG) {
                    a[0] = qf[kk][0]; a[1] = qf[kk][1]; a[2] = qf[kk][2]; a[3] = qf[kk][3];
                } else {
                    ldsm_x4(sQ0 + swz((lane & 7) + ((lane >> 3) & 1) * 8, kk * 2 + (lane >> 4), ROWB), a[0], a[1], a[2], a[3]);
                }
                uint32_t b0, b1, b2, b3;
                ldsm_x4(kb + swz(rb + (lane & 7) + ((lane >> 4) << 3), kk * 2 + ((lane >> 3) & 1), ROWB), b0, b1, b2, b3);
                Mma<T>::run(sc[0], a, b0, b1);
                Mma<T>::run(sc[1], a, b2, b3);
            }
            // mask + online softmax (rows r = lane/4 and r + 8)
            float mx0 = neg_inf(), mx1 = neg_inf();
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int col = nt * 8 + 2 * (lane & 3) + (j & 1);
                    const float x = col < nv ? sc[nt][j] * p.scale_log2 : neg_inf();
                    sc[nt][j] = x;
                    if (j < 2) mx0 = fmaxf(mx0, x); else mx1 = fmaxf(mx1, x);
                }
            }
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
            const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
            const float al0 = fast_exp2(m0 - n0), al1 = fast_exp2(m1 - n1);
            m0 = n0;
            m1 = n1;
            float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
                sc[nt][0] = fast_exp2(sc[nt][0] - n0);
                sc[nt][1] = fast_exp2(sc[nt][1] - n0);
                sc[nt][2] = fast_exp2(sc[nt][2] - n1);
                sc[nt][3] = fast_exp2(sc[nt][3] - n1);
                ps0 += sc[nt][0] + sc[nt][1];
                ps1 += sc[nt][2] + sc[nt][3];
            }
            l0 = l0 * al0 + ps0;
            l1 = l1 * al1 + ps1;
#pragma unroll
            for (int j = 0; j < E / 8; ++j) {
                o[j][0] *= al0; o[j][1] *= al0;
                o[j][2] *= al1; o[j][3] *= al1;
            }
            uint32_t pa[4];
            pa[0] = Elem<T>::pack2(sc[0][0], sc[0][1]);
            pa[1] = Elem<T>::pack2(sc[0][2], sc[0][3]);
            pa[2] = Elem<T>::pack2(sc[1][0], sc[1][1]);
            pa[3] = Elem<T>::pack2(sc[1][2], sc[1][3]);
#pragma unroll
            for (int np = 0; np < E / 16; ++np) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(vb + swz(rb + (lane & 7) + (((lane >> 3) & 1) << 3), 2 * np + (lane >> 4), ROWB), b0, b1, b2, b3);
                Mma<T>::run(o[2 * np], pa, b0, b1);
                Mma<T>::run(o[2 * np + 1], pa, b2, b3);
            }
        }

        if (d.seg_last) {
            // ---- combine the WARPS per-warp states of this segment piece ----
            float lt0 = l0 + __shfl_xor_sync(0xffffffffu, l0, 1);
            lt0 += __shfl_xor_sync(0xffffffffu, lt0, 2);
            float lt1 = l1 + __shfl_xor_sync(0xffffffffu, l1, 1);
            lt1 += __shfl_xor_sync(0xffffffffu, lt1, 2);
            const int r0 = lane >> 2;
            if ((lane & 3) == 0) {
                sML[(wid * 16 + r0) * 2 + 0] = m0;
                sML[(wid * 16 + r0) * 2 + 1] = lt0;
                sML[(wid * 16 + r0 + 8) * 2 + 0] = m1;
                sML[(wid * 16 + r0 + 8) * 2 + 1] = lt1;
            }
            __syncthreads();
            float M0 = neg_inf(), M1 = neg_inf();
#pragma unroll
            for (int w2 = 0; w2 < WARPS; ++w2) {
                M0 = fmaxf(M0, sML[(w2 * 16 + r0) * 2]);
                M1 = fmaxf(M1, sML[(w2 * 16 + r0 + 8) * 2]);
            }
            float S0 = 0.f, S1 = 0.f;
#pragma unroll
            for (int w2 = 0; w2 < WARPS; ++w2) {
                const float a0 = sML[(w2 * 16 + r0) * 2], a1 = sML[(w2 * 16 + r0 + 8) * 2];
                if (a0 != neg_inf()) S0 += sML[(w2 * 16 + r0) * 2 + 1] * fast_exp2(a0 - M0);
                if (a1 != neg_inf()) S1 += sML[(w2 * 16 + r0 + 8) * 2 + 1] * fast_exp2(a1 - M1);
            }
            const float f0 = (m0 != neg_inf() && S0 > 0.f) ? fast_exp2(m0 - M0) / S0 : 0.f;
            const float f1 = (m1 != neg_inf() && S1 > 0.f) ? fast_exp2(m1 - M1) / S1 : 0.f;
            if (wid == 0 && (lane & 3) == 0) {
                sLse[r0] = S0 > 0.f ? M0 + __log2f(S0) : neg_inf();
                sLse[r0 + 8] = S1 > 0.f ? M1 + __log2f(S1) : neg_inf();
            }
            // fixed-order sum over warps (deterministic)
#pragma unroll 1
            for (int w2 = 0; w2 < WARPS; ++w2) {
                if (wid == w2) {
#pragma unroll
                    for (int j = 0; j < E / 8; ++j) {
                        const int e = j * 8 + 2 * (lane & 3);
                        float2* a = reinterpret_cast<float2*>(sO + r0 * E + e);
                        float2* b = reinterpret_cast<float2*>(sO + (r0 + 8) * E + e);
                        float2 va = *a, vb2 = *b;
                        va.x += o[j][0] * f0; va.y += o[j][1] * f0;
                        vb2.x += o[j][2] * f1; vb2.y += o[j][3] * f1;
                        *a = va;
                        *b = vb2;
                    }
                }
                __syncthreads();
            }
            // ---- write: final output if this CTA saw the whole segment, else a partial ----
            const int w = d.ws / p.S, s = d.ws - w * p.S;
            if (d.seg_complete) {
                for (int idx = tid * 4; idx < 16 * E; idx += NT * 4) {
                    const int g = idx / E, e = idx % E;
                    float4 v = *reinterpret_cast<float4*>(sO + idx);
                    *reinterpret_cast<float4*>(sO + idx) = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (g < p.gqa) {
                        const size_t orow = ((size_t)w * p.Hq + d.hkv * p.gqa + g) * p.S + s;
                        T* op = static_cast<T*>(p.out) + orow * E + e;
                        uint2 pk;
                        pk.x = Elem<T>::pack2(v.x, v.y);
                        pk.y = Elem<T>::pack2(v.z, v.w);
                        *reinterpret_cast<uint2*>(op) = pk;
                        if (p.out_f32) *reinterpret_cast<float4*>(p.out_f32 + orow * E + e) = v;
                        if (p.lse_out && e == 0) p.lse_out[orow] = sLse[g] * kLn2;
                    }
                }
            } else {
                const int slot = 2 * c + (d.first_piece ? 0 : 1);
                for (int idx = tid * 4; idx < 16 * E; idx += NT * 4) {
                    float4 v = *reinterpret_cast<float4*>(sO + idx);
                    *reinterpret_cast<float4*>(sO + idx) = make_float4(0.f, 0.f, 0.f, 0.f);
                    *reinterpret_cast<float4*>(p.part_o + (size_t)slot * 16 * E + idx) = v;
                }
                if (tid < 16) p.part_lse[slot * 16 + tid] = sLse[tid];
            }
        }
        __syncthreads();
        st_c = (st_c + 1 == STAGES) ? 0 : st_c + 1;
        st_p = (st_p + 1 == STAGES) ? 0 : st_p + 1;
    }
    cp_async_wait<0>();
}

// ==================================================================================
// TMA kernel (f16 / bf16, page sizes that tile 64-key windows): warp-specialised.
// Warp 4 (producer) walks the schedule, looks the window's pages up in the block table
// and issues one 3-D TMA box per (page, 64-column panel, K|V) into a stage of the ring;
// the stage's full mbarrier counts the bytes.  Warps 0-3 (consumers) each take 16 keys
// of the 64-key window: ldmatrix + mma.sync for S = Q K^T and O += P V, online softmax,
// then release the stage on its empty mbarrier.  Keys of a window outside the tile's
// visible range are masked (-inf scores) and their V rows are zeroed in shared memory
// first, so stale or uninitialised pool memory never reaches the output.
// Stage layout: [panel][64 rows][128 B], 128-byte TMA swizzle (16-byte chunk c of row r
// at c ^ (r & 7)).
// ==================================================================================
template <class T, int E, int STAGES>
struct TmaCfg {
    static constexpr int CW = 4;                       // consumer warps
    static constexpr int NT = (CW + 1) * 32;
    static constexpr int TILE = CW * 16;              // keys per window / stage
    static constexpr int NPANEL = E / 64;             // 64-column (128-byte) panels
    static constexpr int PANEL_BYTES = TILE * 128;
    static constexpr int STAGE_BYTES = NPANEL * PANEL_BYTES;  // K (or V) bytes per stage
    static constexpr int KS = E / 16;
    static constexpr bool QREG = (E <= 128);
    static constexpr size_t OFF_V = (size_t)STAGES * STAGE_BYTES;
    static constexpr size_t OFF_Q = 2 * OFF_V;
    static constexpr size_t OFF_O = OFF_Q + 16 * 2 * E;
    static constexpr size_t OFF_ML = OFF_O + 16 * E * 4;
    static constexpr size_t OFF_LSE = OFF_ML + (CW * 16 * 2 > E ? CW * 16 * 2 : E) * 4;
    static constexpr size_t OFF_DESC = OFF_LSE + 16 * 4;
    static constexpr size_t OFF_BAR = OFF_DESC + STAGES * 32;
    static constexpr size_t OFF_FLAG = OFF_BAR + STAGES * 16;
    static constexpr size_t OFF_CS = OFF_ML;  // cos/sin staging of a rotation aliases the merge stats
    static constexpr size_t SMEM = OFF_FLAG + 16;
};

struct StageDesc {
    int ws, hkv, f, r0, n, flags;  // flags: 1 new_seg, 2 new_turn, 4 seg_last, 8 seg_complete, 16 first_piece
};

template <class T, int E, int STAGES>
__global__ void __launch_bounds__(160, (E <= 128) ? 2 : 1) decode_tma_kernel(PagedParams p, const __grid_constant__ CUtensorMap tmk,
                                                         const __grid_constant__ CUtensorMap tmv, int boxr) {
    using C = TmaCfg<T, E, STAGES>;
    constexpr int CW = C::CW, TILE = C::TILE, NPANEL = C::NPANEL;
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t s0 = smem_u32(smem);
    if (s0 & 1023) {
        if (threadIdx.x == 0) atomicOr(&p.sched->error, 4);
        return;
    }
    const uint32_t sK0 = s0, sV0 = s0 + (uint32_t)C::OFF_V, sQ0 = s0 + (uint32_t)C::OFF_Q;
    uint8_t* sQ = smem + C::OFF_Q;
    float* sO = reinterpret_cast<float*>(smem + C::OFF_O);
    float* sML = reinterpret_cast<float*>(smem + C::OFF_ML);
    float* sLse = reinterpret_cast<float*>(smem + C::OFF_LSE);
    StageDesc* sDesc = reinterpret_cast<StageDesc*>(smem + C::OFF_DESC);
    const uint32_t bar_full = s0 + (uint32_t)C::OFF_BAR;          // STAGES x 8 B
    const uint32_t bar_empty = bar_full + STAGES * 8;            // STAGES x 8 B
    volatile int* sAbort = reinterpret_cast<volatile int*>(smem + C::OFF_FLAG);

    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    // the merge kernel may launch now: its CTAs wait (griddepcontrol.wait) for this grid
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // programmatic dependent of the schedule kernel: wait for its header and prefix sums
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const DecodeSched sch = *p.sched;
    const int c = blockIdx.x;
    if (c >= sch.n_eff) return;
    const long long u0 = p.cstart[c], u1 = p.cstart[c + 1];
    if (u0 >= u1) return;
    const int ws0 = find_row<C::NT>(p, u0);

    if (tid == 0) {
        for (int st = 0; st < STAGES; ++st) {
            mbar_init(bar_full + st * 8, 1);
            mbar_init(bar_empty + st * 8, CW);
        }
        *sAbort = 0;
        fence_mbar_init();
    }
    for (int i = tid; i < 16 * E; i += C::NT) sO[i] = 0.f;
    __syncthreads();

    if (wid == CW) {
        // =========================== producer warp ===========================
        if (lane == 0) {
            prefetch_tmap(&tmk);
            prefetch_tmap(&tmv);
        }
        TileIter<TILE> it;
        it.init(p, ws0, p.P[ws0], u0, u1);
        it.align = TILE;
        const uint32_t box_bytes = (uint32_t)boxr * 128u;
        int i = 0;
        bool ok = true;
        for (;; ++i) {
            TileDesc d;
            const bool have = it.next(p, d);
            const int st = i % STAGES;
            if (i >= STAGES && !*sAbort) {
                if (!mbar_wait(bar_empty + st * 8, ((i / STAGES) & 1) ^ 1)) {
                    ok = false;
                    break;
                }
            }
            if (!have) {
                if (lane == 0) {
                    sDesc[st].n = -1;
                    mbar_arrive(bar_full + st * 8);
                }
                break;
            }
            const int win = d.pos0 & ~(TILE - 1);
            int pfirst, npg;
            if (p.BS <= TILE) {
                pfirst = d.pos0 / p.BS;
                npg = (d.pos0 + d.n - 1) / p.BS - pfirst + 1;
            } else {
                pfirst = win / p.BS;
                npg = 1;
            }
            const int* btw = p.bt + (size_t)row_block_table(p, d.ws) * p.maxb;
            int page = lane < npg ? __ldg(btw + pfirst + lane) : 0;
            if (lane == 0) {
                StageDesc sd;
                sd.ws = d.ws;
                sd.hkv = d.hkv;
                sd.f = d.f;
                sd.r0 = d.pos0 - win;
                sd.n = d.n;
                sd.flags = (d.new_seg ? 1 : 0) | (d.new_turn ? 2 : 0) | (d.seg_last ? 4 : 0) |
                           (d.seg_complete ? 8 : 0) | (d.first_piece ? 16 : 0);
                sDesc[st] = sd;
                mbar_expect_tx(bar_full + st * 8, (uint32_t)npg * NPANEL * 2u * box_bytes);
            }
            __syncwarp();
            if (lane < npg) {
                int z, srow;
                const bool valid = p.NB <= 0 || (page >= 0 && page < p.NB);
                if (p.BS <= TILE) {
                    z = valid ? page * p.BS : -2 * boxr;
                    srow = (pfirst + lane) * p.BS - win;
                } else {
                    z = valid ? page * p.BS + (win - pfirst * p.BS) : -2 * boxr;
                    srow = 0;
                }
                const uint32_t kd = sK0 + st * C::STAGE_BYTES + srow * 128;
                const uint32_t vd = sV0 + st * C::STAGE_BYTES + srow * 128;
#pragma unroll
                for (int pn = 0; pn < NPANEL; ++pn) {
                    tma_load_3d(kd + pn * C::PANEL_BYTES, &tmk, pn * 64, d.hkv, z, bar_full + st * 8);
                    tma_load_3d(vd + pn * C::PANEL_BYTES, &tmv, pn * 64, d.hkv, z, bar_full + st * 8);
                }
            }
        }
        if (!ok) {
            if (lane == 0) {
                *sAbort = 1;
                atomicOr(&p.sched->error, 1);
            }
            // let the copies already issued land before the CTA can exit (bounded)
            for (int j = (i - STAGES + 1 > 0 ? i - STAGES + 1 : 0); j < i; ++j)
                mbar_wait(bar_full + (j % STAGES) * 8, (j / STAGES) & 1);
        }
        return;
    }

    // ============================ consumer warps ============================
    uint32_t qf[C::QREG ? C::KS : 1][4];
    float o[E / 8][4];
    float m0 = 0.f, m1 = 0.f, l0 = 0.f, l1 = 0.f;
    const float sl2 = p.scale_log2;
    const int rb = wid * 16;
    for (int i = 0;; ++i) {
        if (named_bar_or(1, CW * 32, *sAbort != 0)) break;
        const int st = i % STAGES;
        if (!mbar_wait(bar_full + st * 8, (i / STAGES) & 1)) {
            if (lane == 0) {
                *sAbort = 1;
                atomicOr(&p.sched->error, 2);
            }
            continue;
        }
        const StageDesc d = sDesc[st];
        if (d.n < 0) break;
        if (d.flags & 1) {
            m0 = m1 = neg_inf();
            l0 = l1 = 0.f;
#pragma unroll
            for (int j = 0; j < E / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
        }
        if (d.flags & 2) {
            named_bar_sync(2, CW * 32);
            rotate_q_rows<T, E, (16 * (E / 8) + CW * 32 - 1) / (CW * 32)>(p, d.ws, d.f, d.hkv, 1, sQ, tid, CW * 32,
                                                                         reinterpret_cast<float*>(smem + C::OFF_CS), 2);
            named_bar_sync(2, CW * 32);
            if constexpr (C::QREG) {
#pragma unroll
                for (int kk = 0; kk < C::KS; ++kk) {
                    const int ch = kk * 2 + (lane >> 4), row = (lane & 7) + ((lane >> 3) & 1) * 8;
                    ldsm_x4(sQ0 + (ch >> 3) * 2048 + row * 128 + (((ch & 7) ^ (row & 7)) << 4), qf[kk][0], qf[kk][1],
                            qf[kk][2], qf[kk][3]);
                }
            }
        }

        const int lo = max(0, d.r0 - rb), hi = min(16, d.r0 + d.n - rb);
        const uint32_t kb = sK0 + st * C::STAGE_BYTES, vb = sV0 + st * C::STAGE_BYTES;
        if (hi > lo) {
            const bool edge = (lo > 0) || (hi < 16);
            if (edge) {
                // zero the V rows of this warp's 16 keys that are outside the visible range
                for (int idx = lane; idx < 16 * NPANEL * 8; idx += 32) {
                    const int j = idx / (NPANEL * 8), rem = idx % (NPANEL * 8);
                    if (j < lo || j >= hi)
                        *reinterpret_cast<uint4*>(smem + C::OFF_V + (size_t)st * C::STAGE_BYTES + (rem >> 3) * C::PANEL_BYTES +
                                                  (rb + j) * 128 + (rem & 7) * 16) = make_uint4(0u, 0u, 0u, 0u);
                }
                fence_proxy_async_smem();
                __syncwarp();
            }
            float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
            for (int kk = 0; kk < C::KS; ++kk) {
                uint32_t a[4];
                if constexpr (C::QREG) {
                    a[0] = qf[kk][0]; a[1] = qf[kk][1]; a[2] = qf[kk][2]; a[3] = qf[kk][3];
                } else {
                    const int ch = kk * 2 + (lane >> 4), row = (lane & 7) + ((lane >> 3) & 1) * 8;
                    ldsm_x4(sQ0 + (ch >> 3) * 2048 + row * 128 + (((ch & 7) ^ (row & 7)) << 4), a[0], a[1], a[2], a[3]);
                }
                const int ch = kk * 2 + ((lane >> 3) & 1), row = rb + (lane & 7) + ((lane >> 4) << 3);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(kb + (ch >> 3) * C::PANEL_BYTES + row * 128 + (((ch & 7) ^ (row & 7)) << 4), b0, b1, b2, b3);
                Mma<T>::run(sc[0], a, b0, b1);
                Mma<T>::run(sc[1], a, b2, b3);
            }
            float mx0 = neg_inf(), mx1 = neg_inf();
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int col = nt * 8 + 2 * (lane & 3) + (j & 1);
                    float x = sc[nt][j] * sl2;
                    if (edge && (col < lo || col >= hi)) x = neg_inf();
                    sc[nt][j] = x;
                }
                mx0 = fmaxf(mx0, fmaxf(sc[nt][0], sc[nt][1]));
                mx1 = fmaxf(mx1, fmaxf(sc[nt][2], sc[nt][3]));
            }
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
            const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
            if (__any_sync(0xffffffffu, (n0 > m0) || (n1 > m1))) {
                const float al0 = fast_exp2(m0 - n0), al1 = fast_exp2(m1 - n1);
                l0 *= al0;
                l1 *= al1;
#pragma unroll
                for (int j = 0; j < E / 8; ++j) {
                    o[j][0] *= al0; o[j][1] *= al0;
                    o[j][2] *= al1; o[j][3] *= al1;
                }
                m0 = n0;
                m1 = n1;
            }
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
                sc[nt][0] = fast_exp2(sc[nt][0] - m0);
                sc[nt][1] = fast_exp2(sc[nt][1] - m0);
                sc[nt][2] = fast_exp2(sc[nt][2] - m1);
                sc[nt][3] = fast_exp2(sc[nt][3] - m1);
            }
            l0 += (sc[0][0] + sc[0][1]) + (sc[1][0] + sc[1][1]);
            l1 += (sc[0][2] + sc[0][3]) + (sc[1][2] + sc[1][3]);
            uint32_t pa[4];
            pa[0] = Elem<T>::pack2(sc[0][0], sc[0][1]);
            pa[1] = Elem<T>::pack2(sc[0][2], sc[0][3]);
            pa[2] = Elem<T>::pack2(sc[1][0], sc[1][1]);
            pa[3] = Elem<T>::pack2(sc[1][2], sc[1][3]);
#pragma unroll
            for (int np = 0; np < E / 16; ++np) {
                const int ch = 2 * np + (lane >> 4), row = rb + (lane & 7) + (((lane >> 3) & 1) << 3);
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(vb + (ch >> 3) * C::PANEL_BYTES + row * 128 + (((ch & 7) ^ (row & 7)) << 4), b0, b1, b2, b3);
                Mma<T>::run(o[2 * np], pa, b0, b1);
                Mma<T>::run(o[2 * np + 1], pa, b2, b3);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_empty + st * 8);

        if (d.flags & 4) {
            // ---- combine the CW per-warp states of this segment piece ----
            float lt0 = l0 + __shfl_xor_sync(0xffffffffu, l0, 1);
            lt0 += __shfl_xor_sync(0xffffffffu, lt0, 2);
            float lt1 = l1 + __shfl_xor_sync(0xffffffffu, l1, 1);
            lt1 += __shfl_xor_sync(0xffffffffu, lt1, 2);
            const int r0 = lane >> 2;
            if ((lane & 3) == 0) {
                sML[(wid * 16 + r0) * 2 + 0] = m0;
                sML[(wid * 16 + r0) * 2 + 1] = lt0;
                sML[(wid * 16 + r0 + 8) * 2 + 0] = m1;
                sML[(wid * 16 + r0 + 8) * 2 + 1] = lt1;
            }
            named_bar_sync(2, CW * 32);
            float M0 = neg_inf(), M1 = neg_inf();
#pragma unroll
            for (int w2 = 0; w2 < CW; ++w2) {
                M0 = fmaxf(M0, sML[(w2 * 16 + r0) * 2]);
                M1 = fmaxf(M1, sML[(w2 * 16 + r0 + 8) * 2]);
            }
            float S0 = 0.f, S1 = 0.f;
#pragma unroll
            for (int w2 = 0; w2 < CW; ++w2) {
                const float a0 = sML[(w2 * 16 + r0) * 2], a1 = sML[(w2 * 16 + r0 + 8) * 2];
                if (a0 != neg_inf()) S0 += sML[(w2 * 16 + r0) * 2 + 1] * fast_exp2(a0 - M0);
                if (a1 != neg_inf()) S1 += sML[(w2 * 16 + r0 + 8) * 2 + 1] * fast_exp2(a1 - M1);
            }
            const float f0 = (m0 != neg_inf() && S0 > 0.f) ? fast_exp2(m0 - M0) / S0 : 0.f;
            const float f1 = (m1 != neg_inf() && S1 > 0.f) ? fast_exp2(m1 - M1) / S1 : 0.f;
            if (wid == 0 && (lane & 3) == 0) {
                sLse[r0] = S0 > 0.f ? M0 + __log2f(S0) : neg_inf();
                sLse[r0 + 8] = S1 > 0.f ? M1 + __log2f(S1) : neg_inf();
            }
#pragma unroll 1
            for (int w2 = 0; w2 < CW; ++w2) {
                if (wid == w2) {
#pragma unroll
                    for (int j = 0; j < E / 8; ++j) {
                        const int e = j * 8 + 2 * (lane & 3);
                        float2* a = reinterpret_cast<float2*>(sO + r0 * E + e);
                        float2* b = reinterpret_cast<float2*>(sO + (r0 + 8) * E + e);
                        float2 va = *a, vb2 = *b;
                        va.x += o[j][0] * f0; va.y += o[j][1] * f0;
                        vb2.x += o[j][2] * f1; vb2.y += o[j][3] * f1;
                        *a = va;
                        *b = vb2;
                    }
                }
                named_bar_sync(2, CW * 32);
            }
            const int w = d.ws / p.S, s = d.ws - w * p.S;
            if (d.flags & 8) {
                for (int idx = tid * 4; idx < 16 * E; idx += CW * 32 * 4) {
                    const int g = idx / E, e = idx % E;
                    float4 v = *reinterpret_cast<float4*>(sO + idx);
                    *reinterpret_cast<float4*>(sO + idx) = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (g < p.gqa) {
                        const size_t orow = ((size_t)w * p.Hq + d.hkv * p.gqa + g) * p.S + s;
                        T* op = static_cast<T*>(p.out) + orow * E + e;
                        uint2 pk;
                        pk.x = Elem<T>::pack2(v.x, v.y);
                        pk.y = Elem<T>::pack2(v.z, v.w);
                        *reinterpret_cast<uint2*>(op) = pk;
                        if (p.out_f32) *reinterpret_cast<float4*>(p.out_f32 + orow * E + e) = v;
                        if (p.lse_out && e == 0) p.lse_out[orow] = sLse[g] * kLn2;
                    }
                }
            } else {
                const int slot = 2 * c + ((d.flags & 16) ? 0 : 1);
                for (int idx = tid * 4; idx < 16 * E; idx += CW * 32 * 4) {
                    float4 v = *reinterpret_cast<float4*>(sO + idx);
                    *reinterpret_cast<float4*>(sO + idx) = make_float4(0.f, 0.f, 0.f, 0.f);
                    *reinterpret_cast<float4*>(p.part_o + (size_t)slot * 16 * E + idx) = v;
                }
                if (tid < 16) p.part_lse[slot * 16 + tid] = sLse[tid];
            }
            // sO / sML / sLse are reused only after the next segment's first named barrier
        }
    }
}

// four consecutive output elements (8-byte store for 16-bit types, 16-byte for f32)



// ==================================================================================
// Row kernel (f16 / bf16, Hkv | CW): like the TMA kernel, but a CTA streams ALL KV heads
// of its keys.  A stage holds TOKB = 16*CW/Hkv keys x Hkv heads; consumer warp w serves
// head w % Hkv and keys [16*(w / Hkv), +16) of the stage.  The producer issues the boxes
// of every head of a page back to back, so the page's K (and V) rows -- Hkv*E elements
// contiguous per token -- are fetched from DRAM together instead of head by head at
// unrelated times.  Stage layout: slab (head h, panel p) = TOKB rows x 128 B, swizzled.
// ==================================================================================
template <class T, int E, int CW, int STAGES>
struct RowCfg {
    static constexpr int NT = (CW + 1) * 32;
    static constexpr int NPANEL = E / 64;
    static constexpr int KROWS = CW * 16;                         // key-head rows per stage
    static constexpr int STAGE_BYTES = KROWS * NPANEL * 128;      // K (or V) bytes per stage
    static constexpr int KS = E / 16;
    static constexpr bool QREG = (E <= 128);
    static constexpr int QBYTES = CW * 16 * 2 * E;                // rotated q of up to CW heads x 16 rows
    static constexpr int OBYTES = 2 * 16 * E * 4;                 // merge buffer (Hkv <= 2 only)
    static constexpr size_t OFF_V = (size_t)STAGES * STAGE_BYTES;
    static constexpr size_t OFF_Q = 2 * OFF_V;
    // With q fragments held in registers (E <= 128) the rotation buffer is only used at a
    // turn change and the merge buffer only at a row's end, so the two share memory.
    static constexpr size_t OFF_O = QREG ? OFF_Q : OFF_Q + QBYTES;
    static constexpr size_t OFF_ML = QREG ? OFF_Q + (QBYTES > OBYTES ? QBYTES : OBYTES) : OFF_O + OBYTES;
    static constexpr size_t OFF_LSE = OFF_ML + (CW * 16 * 2 > E ? CW * 16 * 2 : E) * 4;
    static constexpr size_t OFF_DESC = OFF_LSE + 2 * 16 * 4;
    static constexpr size_t OFF_BAR = OFF_DESC + STAGES * 32;
    static constexpr size_t OFF_FLAG = OFF_BAR + STAGES * 16;
    static constexpr size_t OFF_CS = OFF_ML;  // cos/sin staging of a rotation aliases the merge stats
    static constexpr size_t SMEM = OFF_FLAG + 16;
};

// Tensor maps of up to kParamFrags contiguous fragments, passed by value to the row kernel
// so that a dvattn_sdpa call needs no host-to-device copy (more fragments: the workspace).
constexpr int kParamFrags = 4;
struct alignas(64) FragMaps {
    CUtensorMap m[2 * kParamFrags];  // K then V of each fragment
    int wmul[kParamFrags];
};

template <class T, int E, int CW, int STAGES>
__global__ void __launch_bounds__((CW + 1) * 32, (CW <= 4 && E <= 128) ? 2 : 1)
    decode_row_kernel(PagedParams p, const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                      int boxr, const __grid_constant__ FragMaps fm) {
    using C = RowCfg<T, E, CW, STAGES>;
    constexpr int NPANEL = C::NPANEL;
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t s0 = smem_u32(smem);
    if (s0 & 1023) {  // the 128-byte TMA swizzle pattern needs 1024-byte aligned stages
        asm volatile("griddepcontrol.wait;" ::: "memory");
        if (threadIdx.x == 0) atomicOr(&p.sched->error, 4);
        return;
    }
    const uint32_t sK0 = s0, sV0 = s0 + (uint32_t)C::OFF_V, sQ0 = s0 + (uint32_t)C::OFF_Q;
    uint8_t* sQ = smem + C::OFF_Q;
    float* sO = reinterpret_cast<float*>(smem + C::OFF_O);
    float* sML = reinterpret_cast<float*>(smem + C::OFF_ML);
    float* sLse = reinterpret_cast<float*>(smem + C::OFF_LSE);
    StageDesc* sDesc = reinterpret_cast<StageDesc*>(smem + C::OFF_DESC);
    const uint32_t bar_full = s0 + (uint32_t)C::OFF_BAR;
    const uint32_t bar_empty = bar_full + STAGES * 8;
    volatile int* sAbort = reinterpret_cast<volatile int*>(smem + C::OFF_FLAG);

    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int Hkv = p.Hkv;
    const int TOKB = (CW / Hkv) * 16;           // keys per stage (window)
    // One TMA box = one page (or the window's part of it) for all heads and panels:
    // smem [page chunk][head][panel][boxr rows][128 B].
    const int boxr_shift = __ffs(boxr) - 1;
    const uint32_t box_bytes = (uint32_t)Hkv * NPANEL * boxr * 128u;
    // the merge kernel may launch now: its CTAs wait (griddepcontrol.wait) for this grid
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int c = blockIdx.x;
    long long u0, u1, P0, U = 0, pubP = 0;
    int ws0, n = 0;
    long long bseg = -1;  // first segment start inside (u0, u1) when p.rotate (else none)
    int wsb = 0;
    // fused schedule, producer warp: after the previous grid completed, publish P, cstart
    // and the header for the merge kernel
    auto publish = [&]() {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        if (32 * c + lane <= p.WS) p.P[32 * c + lane] = pubP;
        if (lane == 0 && c < n) {
            p.cstart[c] = u0;
            if (c == n - 1) p.cstart[n] = U;
        }
        if (lane == 0 && c == 0) {
            p.sched->U = U;
            p.sched->n_eff = n;
            // cleared once per call; a bounded wait sets a bit only after it has run out
            // (long after every CTA passed griddepcontrol.wait), so the clear comes first
            p.sched->error = 0;
        }
    };
    if (p.fused) {
        // In-kernel schedule (no prep kernel): every CTA scans the row unit counts into the
        // K/V stages (unused until the first TMA) and finds its own range.  Only inputs
        // are read here, so this and the streaming below overlap the previous grid; the
        // first global write of every warp comes after griddepcontrol.wait.
        long long* sP = reinterpret_cast<long long*>(smem);
        cta_prefix<C::NT>(p, sP, sP + p.WS + 1, U, n);
        u0 = cta_boundary(p, sP, U, n, c);
        u1 = cta_boundary(p, sP, U, n, c + 1);
        ws0 = u0 < u1 ? find_row_in(sP, p.WS, p.hsplit, u0) : 0;
        P0 = sP[ws0];
        if (p.rotate && u0 < u1 && ws0 < p.WS) {
            bseg = sP[ws0 + 1] * p.hsplit;
            if (bseg > u0 && bseg < u1) wsb = find_row_in(sP, p.WS, p.hsplit, bseg);
        }
        // this CTA publishes P[32c .. 32c+31] (producer warp lanes)
        if (wid == CW && 32 * c + lane <= p.WS) pubP = sP[32 * c + lane];
        __syncthreads();
        if (u0 >= u1) {
            if (wid == CW) publish();
            return;
        }
    } else {
        // programmatic dependent of the schedule kernel: wait for its header and prefix sums
        asm volatile("griddepcontrol.wait;" ::: "memory");
        const DecodeSched sch = *p.sched;
        if (c >= sch.n_eff) return;
        u0 = p.cstart[c];
        u1 = p.cstart[c + 1];
        if (u0 >= u1) return;
        ws0 = find_row<C::NT>(p, u0);
        P0 = p.P[ws0];
        if (p.rotate && ws0 < p.WS) {
            bseg = p.P[ws0 + 1] * p.hsplit;
            if (bseg > u0 && bseg < u1) wsb = find_row<C::NT>(p, bseg);
        }
    }

    if (tid == 0) {
        for (int st = 0; st < STAGES; ++st) {
            mbar_init(bar_full + st * 8, 1);
            mbar_init(bar_empty + st * 8, CW);
        }
        *sAbort = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (wid == CW) {
        // =========================== producer warp ===========================
        if (lane == 0 && !p.nfrag) {
            prefetch_tmap(&tmk);
            prefetch_tmap(&tmv);
        }
        RotTileIter<64> it;
        it.init(p, ws0, P0, u0, u1, wsb, bseg, TOKB);
        struct Pend {
            TileDesc d;
            int pfirst, npg, page;
            bool have;
        };
        // next tile: descriptor, its pages, and (lane j) the block-table entry of page j;
        // prepared one tile ahead so the table load is in flight during the stage wait.
        auto prep = [&](Pend& q) {
            q.have = it.next(p, q.d);
            if (!q.have) return;
            if (p.nfrag) {  // contiguous fragment: one box per window, no block table
                q.pfirst = 0;
                q.npg = 1;
                // batch multiplier, loaded a tile ahead
                q.page = p.fmaps ? __ldg(&p.frag[q.d.f].wmul) : fm.wmul[q.d.f];
                if (q.d.new_turn) prefetch_rotation_inputs<T, E>(p, q.d.ws, q.d.f, lane);
                return;
            }
            const int pos0 = q.d.pos0;
            if (p.BS <= TOKB) {
                const int last = pos0 + q.d.n - 1;
                q.pfirst = p.bs_shift >= 0 ? pos0 >> p.bs_shift : pos0 / p.BS;
                q.npg = (p.bs_shift >= 0 ? last >> p.bs_shift : last / p.BS) - q.pfirst + 1;
            } else {
                const int win = pos0 & ~(TOKB - 1);
                q.pfirst = p.bs_shift >= 0 ? win >> p.bs_shift : win / p.BS;
                q.npg = 1;
            }
            const int btrow = p.cu_q ? p.row_seq[q.d.ws] : (p.S == 1 ? q.d.ws : q.d.ws / p.S);
            q.page = lane < q.npg ? __ldg(p.bt + (size_t)btrow * p.maxb + q.pfirst + lane) : 0;
            if (q.d.new_turn) prefetch_rotation_inputs<T, E>(p, q.d.ws, q.d.f, lane);
        };
        Pend cur, nxt;
        prep(nxt);
        int i = 0;
        bool ok = true;
        for (;; ++i) {
            cur = nxt;
            if (cur.have) prep(nxt);
            const int st = i % STAGES;
            if (i >= STAGES && !*sAbort) {
                if (!mbar_wait(bar_empty + st * 8, ((i / STAGES) & 1) ^ 1)) {
                    ok = false;
                    break;
                }
            }
            if (!cur.have) {
                if (lane == 0) {
                    sDesc[st].n = -1;
                    mbar_arrive(bar_full + st * 8);
                }
                break;
            }
            if (i == p.stall_tile && c == 0) continue;  // test hook: this stage is never filled
            const TileDesc& d = cur.d;
            const int win = d.pos0 & ~(TOKB - 1);
            if (lane == 0) {
                StageDesc sd;
                sd.ws = d.ws;
                sd.hkv = 0;
                sd.f = d.f;
                sd.r0 = d.pos0 - win;
                sd.n = d.n;
                sd.flags = (d.new_seg ? 1 : 0) | (d.new_turn ? 2 : 0) | (d.seg_last ? 4 : 0) |
                           (d.seg_complete ? 8 : 0) | (d.first_piece ? 16 : 0);
                sDesc[st] = sd;
                mbar_expect_tx(bar_full + st * 8, (uint32_t)cur.npg * 2u * box_bytes);
            }
            __syncwarp();
            if (p.nfrag) {
                // rows [win - off, win - off + TOKB) of turn f's fragment (rows outside it
                // read as zeros), batch entry w (or 0 for a fragment all workers share)
                if (lane == 0) {
                    const int b = (p.S == 1 ? d.ws : d.ws / p.S) * cur.page;
                    const char* mk = p.fmaps ? p.fmaps + (size_t)d.f * 256
                                             : reinterpret_cast<const char*>(&fm.m[2 * d.f]);
                    const uint32_t off = (uint32_t)(st * C::STAGE_BYTES);
                    tma_load_5d(sK0 + off, mk, 0, win - d.off, 0, 0, b, bar_full + st * 8);
                    tma_load_5d(sV0 + off, mk + 128, 0, win - d.off, 0, 0, b, bar_full + st * 8);
                }
                continue;
            }
            if (lane < cur.npg) {
                const int page = cur.page;
                const bool valid = p.NB <= 0 || (page >= 0 && page < p.NB);
                int z, chunk;
                if (p.BS <= TOKB) {
                    z = valid ? page * p.BS : -2 * boxr;
                    chunk = ((cur.pfirst + lane) * p.BS - win) >> boxr_shift;
                } else {
                    z = valid ? page * p.BS + (win - cur.pfirst * p.BS) : -2 * boxr;
                    chunk = 0;
                }
                const uint32_t off = (uint32_t)(st * C::STAGE_BYTES) + (uint32_t)chunk * box_bytes;
                tma_load_4d(sK0 + off, &tmk, 0, z, 0, 0, bar_full + st * 8);
                tma_load_4d(sV0 + off, &tmv, 0, z, 0, 0, bar_full + st * 8);
            }
        }
        if (p.fused) publish();
        if (!ok) {
            if (lane == 0) {
                *sAbort = 1;
                atomicOr(&p.sched->error, 1);
            }
            for (int j = (i - STAGES + 1 > 0 ? i - STAGES + 1 : 0); j < i; ++j)
                mbar_wait(bar_full + (j % STAGES) * 8, (j / STAGES) & 1);
        }
        return;
    }

    // ============================ consumer warps ============================
    const int h = wid % Hkv, grp = wid / Hkv;
    const int rb = grp * 16;                    // this warp's first key row in the window
    const int wph = CW / Hkv;                   // warps per head
    uint32_t qf[C::QREG ? C::KS : 1][4];
    float o[E / 8][4];
    float m0 = 0.f, m1 = 0.f, l0 = 0.f, l1 = 0.f;
    const float sl2 = p.scale_log2;
    const uint32_t qh = sQ0 + h * NPANEL * 2048;
    // byte offset of 16-byte chunk `ch` of key row `row` of head h in a K/V stage
    auto kv_off = [&](int row, int ch) -> uint32_t {
        return (uint32_t)((((row >> boxr_shift) * Hkv + h) * NPANEL + (ch >> 3)) * boxr + (row & (boxr - 1))) * 128u +
               (uint32_t)(((ch & 7) ^ (row & 7)) << 4);
    };
    // The first tile always starts a turn: rotate its q now, while the first stage's TMA
    // loads are in flight, instead of after they land.
    {
        RotTileIter<64> it0;
        it0.init(p, ws0, P0, u0, u1, wsb, bseg, TOKB);
        TileDesc d0;
        if (it0.next(p, d0)) {
            rotate_q_inplace<T, E>(p, d0.ws, d0.f, Hkv, sQ, tid, CW * 32,
                                                                           reinterpret_cast<float*>(smem + C::OFF_CS), 2);
            named_bar_sync(2, CW * 32);
            if constexpr (C::QREG) {
#pragma unroll
                for (int kk = 0; kk < C::KS; ++kk) {
                    const int ch = kk * 2 + (lane >> 4), row = (lane & 7) + ((lane >> 3) & 1) * 8;
                    ldsm_x4(qh + (ch >> 3) * 2048 + row * 128 + (((ch & 7) ^ (row & 7)) << 4), qf[kk][0], qf[kk][1],
                            qf[kk][2], qf[kk][3]);
                }
            }
        }
    }
    for (int i = 0;; ++i) {
        if (named_bar_or(1, CW * 32, *sAbort != 0)) break;
        const int st = i % STAGES;
        if (!mbar_wait(bar_full + st * 8, (i / STAGES) & 1)) {
            if (lane == 0) {
                asm volatile("griddepcontrol.wait;" ::: "memory");
                *sAbort = 1;
                atomicOr(&p.sched->error, 2);
            }
            continue;
        }
        const StageDesc d = sDesc[st];
        if (d.n < 0) break;
        if (d.flags & 1) {
            m0 = m1 = neg_inf();
            l0 = l1 = 0.f;
#pragma unroll
            for (int j = 0; j < E / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
        }
        if ((d.flags & 2) && i > 0) {
            named_bar_sync(2, CW * 32);
            rotate_q_inplace<T, E>(p, d.ws, d.f, Hkv, sQ, tid, CW * 32,
                                                                           reinterpret_cast<float*>(smem + C::OFF_CS), 2);
            named_bar_sync(2, CW * 32);
            if constexpr (C::QREG) {
#pragma unroll
                for (int kk = 0; kk < C::KS; ++kk) {
                    const int ch = kk * 2 + (lane >> 4), row = (lane & 7) + ((lane >> 3) & 1) * 8;
                    ldsm_x4(qh + (ch >> 3) * 2048 + row * 128 + (((ch & 7) ^ (row & 7)) << 4), qf[kk][0], qf[kk][1],
                            qf[kk][2], qf[kk][3]);
                }
            }
        }

        const int lo = max(0, d.r0 - rb), hi = min(16, d.r0 + d.n - rb);
        const uint32_t kb = sK0 + st * C::STAGE_BYTES;
        const uint32_t vb = sV0 + st * C::STAGE_BYTES;
        if (hi > lo) {
            const bool edge = (lo > 0) || (hi < 16);
            if (edge) {
                uint8_t* vst = smem + C::OFF_V + (size_t)st * C::STAGE_BYTES;
                for (int idx = lane; idx < 16 * NPANEL * 8; idx += 32) {
                    const int j = idx / (NPANEL * 8), rem = idx % (NPANEL * 8);
                    if (j < lo || j >= hi)
                        *reinterpret_cast<uint4*>(vst + kv_off(rb + j, rem)) = make_uint4(0u, 0u, 0u, 0u);
                }
                fence_proxy_async_smem();
                __syncwarp();
            }
            float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
            for (int kk = 0; kk < C::KS; ++kk) {
                uint32_t a[4];
                if constexpr (C::QREG) {
                    a[0] = qf[kk][0]; a[1] = qf[kk][1]; a[2] = qf[kk][2]; a[3] = qf[kk][3];
                } else {
                    const int ch = kk * 2 + (lane >> 4), row = (lane & 7) + ((lane >> 3) & 1) * 8;
                    ldsm_x4(qh + (ch >> 3) * 2048 + row * 128 + (((ch & 7) ^ (row & 7)) << 4), a[0], a[1], a[2], a[3]);
                }
                const int ch = kk * 2 + ((lane >> 3) & 1), row = rb + (lane & 7) + ((lane >> 4) << 3);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(kb + kv_off(row, ch), b0, b1, b2, b3);
                Mma<T>::run(sc[0], a, b0, b1);
                Mma<T>::run(sc[1], a, b2, b3);
            }
            float mx0 = neg_inf(), mx1 = neg_inf();
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int col = nt * 8 + 2 * (lane & 3) + (j & 1);
                    float x = sc[nt][j] * sl2;
                    if (edge && (col < lo || col >= hi)) x = neg_inf();
                    sc[nt][j] = x;
                }
                mx0 = fmaxf(mx0, fmaxf(sc[nt][0], sc[nt][1]));
                mx1 = fmaxf(mx1, fmaxf(sc[nt][2], sc[nt][3]));
            }
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
            const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
            if (__any_sync(0xffffffffu, (n0 > m0) || (n1 > m1))) {
                const float al0 = fast_exp2(m0 - n0), al1 = fast_exp2(m1 - n1);
                l0 *= al0;
                l1 *= al1;
#pragma unroll
                for (int j = 0; j < E / 8; ++j) {
                    o[j][0] *= al0; o[j][1] *= al0;
                    o[j][2] *= al1; o[j][3] *= al1;
                }
                m0 = n0;
                m1 = n1;
            }
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
                sc[nt][0] = fast_exp2(sc[nt][0] - m0);
                sc[nt][1] = fast_exp2(sc[nt][1] - m0);
                sc[nt][2] = fast_exp2(sc[nt][2] - m1);
                sc[nt][3] = fast_exp2(sc[nt][3] - m1);
            }
            l0 += (sc[0][0] + sc[0][1]) + (sc[1][0] + sc[1][1]);
            l1 += (sc[0][2] + sc[0][3]) + (sc[1][2] + sc[1][3]);
            uint32_t pa[4];
            pa[0] = Elem<T>::pack2(sc[0][0], sc[0][1]);
            pa[1] = Elem<T>::pack2(sc[0][2], sc[0][3]);
            pa[2] = Elem<T>::pack2(sc[1][0], sc[1][1]);
            pa[3] = Elem<T>::pack2(sc[1][2], sc[1][3]);
#pragma unroll
            for (int np = 0; np < E / 16; ++np) {
                const int ch = 2 * np + (lane >> 4), row = rb + (lane & 7) + (((lane >> 3) & 1) << 3);
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(vb + kv_off(row, ch), b0, b1, b2, b3);
                Mma<T>::run(o[2 * np], pa, b0, b1);
                Mma<T>::run(o[2 * np + 1], pa, b2, b3);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_empty + st * 8);

        if (d.flags & 4) {
            // first global writes of this warp: after the previous grid has completed
            if (p.fused) asm volatile("griddepcontrol.wait;" ::: "memory");
            // ---- finish this row piece: per head, combine its wph warps ----
            float lt0 = l0 + __shfl_xor_sync(0xffffffffu, l0, 1);
            lt0 += __shfl_xor_sync(0xffffffffu, lt0, 2);
            float lt1 = l1 + __shfl_xor_sync(0xffffffffu, l1, 1);
            lt1 += __shfl_xor_sync(0xffffffffu, lt1, 2);
            const int r0 = lane >> 2;
            float M0 = m0, M1 = m1, S0 = lt0, S1 = lt1;
            float f0, f1;
            if (wph > 1) {
                if ((lane & 3) == 0) {
                    sML[(wid * 16 + r0) * 2 + 0] = m0;
                    sML[(wid * 16 + r0) * 2 + 1] = lt0;
                    sML[(wid * 16 + r0 + 8) * 2 + 0] = m1;
                    sML[(wid * 16 + r0 + 8) * 2 + 1] = lt1;
                }
                named_bar_sync(2, CW * 32);
                M0 = M1 = neg_inf();
                for (int g2 = 0; g2 < wph; ++g2) {
                    const int w2 = g2 * Hkv + h;
                    M0 = fmaxf(M0, sML[(w2 * 16 + r0) * 2]);
                    M1 = fmaxf(M1, sML[(w2 * 16 + r0 + 8) * 2]);
                }
                S0 = S1 = 0.f;
                for (int g2 = 0; g2 < wph; ++g2) {
                    const int w2 = g2 * Hkv + h;
                    const float a0 = sML[(w2 * 16 + r0) * 2], a1 = sML[(w2 * 16 + r0 + 8) * 2];
                    if (a0 != neg_inf()) S0 += sML[(w2 * 16 + r0) * 2 + 1] * fast_exp2(a0 - M0);
                    if (a1 != neg_inf()) S1 += sML[(w2 * 16 + r0 + 8) * 2 + 1] * fast_exp2(a1 - M1);
                }
            }
            f0 = (m0 != neg_inf() && S0 > 0.f) ? fast_exp2(m0 - M0) / S0 : 0.f;
            f1 = (m1 != neg_inf() && S1 > 0.f) ? fast_exp2(m1 - M1) / S1 : 0.f;
            const float lse0 = S0 > 0.f ? M0 + __log2f(S0) : neg_inf();
            const float lse1 = S1 > 0.f ? M1 + __log2f(S1) : neg_inf();
            const int w = d.ws / p.S, s = d.ws - w * p.S;
            const bool complete = (d.flags & 8) != 0;
            const int slot = 2 * c + ((d.flags & 16) ? 0 : 1);
            if (wph == 1) {
                // this warp alone holds head h: write straight from the fragments
                const int ga = r0, gb = r0 + 8;
                if (complete) {
                    const size_t oa = ((size_t)w * p.Hq + h * p.gqa + ga) * p.S + s;
                    const size_t ob = ((size_t)w * p.Hq + h * p.gqa + gb) * p.S + s;
                    T* pa_ = static_cast<T*>(p.out) + oa * E;
                    T* pb_ = static_cast<T*>(p.out) + ob * E;
#pragma unroll
                    for (int j = 0; j < E / 8; ++j) {
                        const int e = j * 8 + 2 * (lane & 3);
                        if (ga < p.gqa) {
                            *reinterpret_cast<uint32_t*>(pa_ + e) = Elem<T>::pack2(o[j][0] * f0, o[j][1] * f0);
                            if (p.out_f32) *reinterpret_cast<float2*>(p.out_f32 + oa * E + e) = make_float2(o[j][0] * f0, o[j][1] * f0);
                        }
                        if (gb < p.gqa) {
                            *reinterpret_cast<uint32_t*>(pb_ + e) = Elem<T>::pack2(o[j][2] * f1, o[j][3] * f1);
                            if (p.out_f32) *reinterpret_cast<float2*>(p.out_f32 + ob * E + e) = make_float2(o[j][2] * f1, o[j][3] * f1);
                        }
                    }
                    if (p.lse_out && (lane & 3) == 0) {
                        if (ga < p.gqa) p.lse_out[oa] = lse0 * kLn2;
                        if (gb < p.gqa) p.lse_out[ob] = lse1 * kLn2;
                    }
                } else {
                    float* po = p.part_o + ((size_t)(slot * Hkv + h) * 16) * E;
#pragma unroll
                    for (int j = 0; j < E / 8; ++j) {
                        const int e = j * 8 + 2 * (lane & 3);
                        *reinterpret_cast<float2*>(po + r0 * E + e) = make_float2(o[j][0] * f0, o[j][1] * f0);
                        *reinterpret_cast<float2*>(po + (r0 + 8) * E + e) = make_float2(o[j][2] * f1, o[j][3] * f1);
                    }
                    if ((lane & 3) == 0) {
                        p.part_lse[(slot * Hkv + h) * 16 + r0] = lse0;
                        p.part_lse[(slot * Hkv + h) * 16 + r0 + 8] = lse1;
                    }
                }
            } else {
                // wph warps per head (Hkv <= 2): fixed-order sum in sO[h], then write
                float* so = sO + h * 16 * E;
                if (grp == 0 && (lane & 3) == 0) {
                    sLse[h * 16 + r0] = lse0;
                    sLse[h * 16 + r0 + 8] = lse1;
                }
#pragma unroll 1
                for (int g2 = 0; g2 < wph; ++g2) {
                    if (grp == g2) {
#pragma unroll
                        for (int j = 0; j < E / 8; ++j) {
                            const int e = j * 8 + 2 * (lane & 3);
                            float2* a = reinterpret_cast<float2*>(so + r0 * E + e);
                            float2* b = reinterpret_cast<float2*>(so + (r0 + 8) * E + e);
                            float2 va = g2 ? *a : make_float2(0.f, 0.f), vb2 = g2 ? *b : make_float2(0.f, 0.f);
                            va.x += o[j][0] * f0; va.y += o[j][1] * f0;
                            vb2.x += o[j][2] * f1; vb2.y += o[j][3] * f1;
                            *a = va;
                            *b = vb2;
                        }
                    }
                    named_bar_sync(2, CW * 32);
                }
                for (int idx = tid * 4; idx < Hkv * 16 * E; idx += CW * 32 * 4) {
                    const int hg = idx / E, e = idx % E;
                    const int hk = hg >> 4, g = hg & 15;
                    const float4 v = *reinterpret_cast<float4*>(sO + idx);
                    if (complete) {
                        if (g < p.gqa) {
                            const size_t orow = ((size_t)w * p.Hq + hk * p.gqa + g) * p.S + s;
                            T* op = static_cast<T*>(p.out) + orow * E + e;
                            uint2 pk;
                            pk.x = Elem<T>::pack2(v.x, v.y);
                            pk.y = Elem<T>::pack2(v.z, v.w);
                            *reinterpret_cast<uint2*>(op) = pk;
                            if (p.out_f32) *reinterpret_cast<float4*>(p.out_f32 + orow * E + e) = v;
                            if (p.lse_out && e == 0) p.lse_out[orow] = sLse[hg] * kLn2;
                        }
                    } else {
                        *reinterpret_cast<float4*>(p.part_o + ((size_t)slot * Hkv * 16) * E + idx) = v;
                        if (e == 0) p.part_lse[slot * Hkv * 16 + hg] = sLse[hg];
                    }
                }
            }
        }
    }
}

// ==================================================================================
// f32 kernel (CUDA cores; tensor-core tf32 would miss the 1e-5 f32 tolerance)
// thread t owns query head h = t / 8 for scores and the output columns
// e = 4 * ((t % 8) + 8k) .. +3, so no cross-thread merge is needed.
// ==================================================================================
template <int E, int STAGES>
struct F32Cfg {
    static constexpr int NT = 128;
    static constexpr int TILE = 32;
    static constexpr int LD = E + 4;          // padded row (floats)
    static constexpr int STAGE_F = TILE * LD; // floats per stage
    static constexpr int CPR = E / 4;         // 16-byte chunks per row
    static constexpr size_t SMEM = (2ull * STAGES * STAGE_F + 16 * LD + 16 * TILE) * 4;
};

template <int E, int STAGES>
__global__ void __launch_bounds__(128) decode_f32_kernel(PagedParams p) {
    using C = F32Cfg<E, STAGES>;
    constexpr int NT = C::NT, TILE = C::TILE, LD = C::LD, CPR = C::CPR;
    constexpr int EC = E / 32;  // float4 column chunks per thread
    extern __shared__ __align__(1024) uint8_t smem[];
    float* sK = reinterpret_cast<float*>(smem);
    float* sV = sK + STAGES * C::STAGE_F;
    float* sQ = sV + STAGES * C::STAGE_F;
    float* sP = sQ + 16 * LD;

    const int tid = threadIdx.x;
    // the merge kernel may launch now: its CTAs wait (griddepcontrol.wait) for this grid
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // programmatic dependent of the schedule kernel: wait for its header and prefix sums
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const DecodeSched sch = *p.sched;
    const int c = blockIdx.x;
    if (c >= sch.n_eff) return;
    const long long u0 = p.cstart[c], u1 = p.cstart[c + 1];
    if (u0 >= u1) return;
    const int ws0 = find_row<NT>(p, u0);
    const float* __restrict__ kc = static_cast<const float*>(p.k);
    const float* __restrict__ vc = static_cast<const float*>(p.v);

    auto issue = [&](const TileDesc& d, int st) {
        const int* btw = p.nfrag ? nullptr : p.bt + (size_t)row_block_table(p, d.ws) * p.maxb;
        FragDesc fd{};
        if (p.nfrag) fd = p.frag[d.f];
        float* kd = sK + st * C::STAGE_F;
        float* vd = sV + st * C::STAGE_F;
#pragma unroll
        for (int i = 0; i < TILE * CPR / NT; ++i) {
            const int idx = i * NT + tid;
            const int r = idx / CPR, ch = idx % CPR;
            const float* ks = kc;
            const float* vs = vc;
            int bytes = 0;
            if (r < d.n) {
                const int pos = d.pos0 + r;
                if (p.nfrag) {  // contiguous fragment of turn d.f
                    const int l = pos - d.off;
                    if (l < fd.rows) {
                        const size_t row =
                            ((size_t)(d.ws / p.S) * fd.wmul * p.Hkv + d.hkv) * (size_t)fd.rows + (size_t)l;
                        ks = static_cast<const float*>(fd.k) + row * E + ch * 4;
                        vs = static_cast<const float*>(fd.v) + row * E + ch * 4;
                        bytes = 16;
                    }
                } else {
                    const int page = __ldg(btw + pos / p.BS);
                    if (p.NB <= 0 || (page >= 0 && page < p.NB)) {
                        const size_t row = ((size_t)page * p.BS + pos % p.BS) * p.Hkv + d.hkv;
                        ks = kc + row * E + ch * 4;
                        vs = vc + row * E + ch * 4;
                        bytes = 16;
                    }
                }
            }
            cp_async16_zfill(smem_u32(kd + r * LD + ch * 4), ks, bytes);
            cp_async16_zfill(smem_u32(vd + r * LD + ch * 4), vs, bytes);
        }
    };

    TileIter<TILE> prod, cons;
    prod.init(p, ws0, p.P[ws0], u0, u1);
    cons = prod;
#pragma unroll
    for (int st = 0; st < STAGES - 1; ++st) {
        TileDesc d;
        if (prod.next(p, d)) issue(d, st);
        cp_async_commit();
    }

    const int h = tid >> 3, sub = tid & 7;
    float o[EC][4];
    float m = 0.f, l = 0.f;
    int st_c = 0, st_p = STAGES - 1;
    TileDesc d;
    while (cons.next(p, d)) {
        if (d.new_seg) {
            m = neg_inf();
            l = 0.f;
#pragma unroll
            for (int j = 0; j < EC; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
        }
        if (d.new_turn) {
            __syncthreads();
            const int w = d.ws / p.S, s = d.ws - w * p.S;
            const float* cr = p.cos + ((size_t)d.f * p.WS + d.ws) * p.cs_stride;
            const float* sr = p.sin + ((size_t)d.f * p.WS + d.ws) * p.cs_stride;
            for (int idx = tid; idx < 16 * E; idx += NT) {
                const int g = idx / E, e = idx % E;
                float x = 0.f;
                if (g < p.gqa) {
                    const float* qrow = static_cast<const float*>(p.q) + (size_t)d.f * p.q_turn_stride +
                                        (((size_t)w * p.Hq + d.hkv * p.gqa + g) * p.S + s) * E;
                    x = rotated_elem(qrow, cr, sr, e, p.R);
                }
                sQ[g * LD + e] = x;
            }
        }
        {
            TileDesc dp;
            if (prod.next(p, dp)) issue(dp, st_p);
            cp_async_commit();
        }
        cp_async_wait<STAGES - 1>();
        __syncthreads();

        const float* kb = sK + st_c * C::STAGE_F;
        const float* vb = sV + st_c * C::STAGE_F;
        // scores of head h for keys sub, sub+8, sub+16, sub+24
        float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
        for (int e = 0; e < E; e += 4) {
            const float4 qv = *reinterpret_cast<const float4*>(sQ + h * LD + e);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float4 kv = *reinterpret_cast<const float4*>(kb + (sub + 8 * i) * LD + e);
                sc[i] = fmaf(qv.x, kv.x, sc[i]);
                sc[i] = fmaf(qv.y, kv.y, sc[i]);
                sc[i] = fmaf(qv.z, kv.z, sc[i]);
                sc[i] = fmaf(qv.w, kv.w, sc[i]);
            }
        }
        float mx = neg_inf();
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            sc[i] = (sub + 8 * i) < d.n ? sc[i] * p.scale_log2 : neg_inf();
            mx = fmaxf(mx, sc[i]);
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        const float mn = fmaxf(m, mx);
        const float al = fast_exp2(m - mn);
        m = mn;
        float ps = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float pv = fast_exp2(sc[i] - mn);
            ps += pv;
            sP[h * TILE + sub + 8 * i] = pv;
        }
        ps += __shfl_xor_sync(0xffffffffu, ps, 1);
        ps += __shfl_xor_sync(0xffffffffu, ps, 2);
        ps += __shfl_xor_sync(0xffffffffu, ps, 4);
        l = l * al + ps;
#pragma unroll
        for (int j = 0; j < EC; ++j) {
            o[j][0] *= al; o[j][1] *= al; o[j][2] *= al; o[j][3] *= al;
        }
        __syncwarp();
        // head h's probabilities were written by the 8 lanes of this same warp group
        for (int r = 0; r < d.n; ++r) {
            const float pv = sP[h * TILE + r];
#pragma unroll
            for (int j = 0; j < EC; ++j) {
                const float4 vv = *reinterpret_cast<const float4*>(vb + r * LD + 4 * (sub + 8 * j));
                o[j][0] = fmaf(pv, vv.x, o[j][0]);
                o[j][1] = fmaf(pv, vv.y, o[j][1]);
                o[j][2] = fmaf(pv, vv.z, o[j][2]);
                o[j][3] = fmaf(pv, vv.w, o[j][3]);
            }
        }

        if (d.seg_last) {
            const int w = d.ws / p.S, s = d.ws - w * p.S;
            const float inv = l > 0.f ? 1.f / l : 0.f;
            const float lse2 = l > 0.f ? m + __log2f(l) : neg_inf();
            if (d.seg_complete) {
                if (h < p.gqa) {
                    const size_t orow = ((size_t)w * p.Hq + d.hkv * p.gqa + h) * p.S + s;
                    float* op = static_cast<float*>(p.out) + orow * E;
#pragma unroll
                    for (int j = 0; j < EC; ++j) {
                        const float4 v = make_float4(o[j][0] * inv, o[j][1] * inv, o[j][2] * inv, o[j][3] * inv);
                        *reinterpret_cast<float4*>(op + 4 * (sub + 8 * j)) = v;
                        if (p.out_f32) *reinterpret_cast<float4*>(p.out_f32 + orow * E + 4 * (sub + 8 * j)) = v;
                    }
                    if (p.lse_out && sub == 0) p.lse_out[orow] = lse2 * kLn2;
                }
            } else {
                const int slot = 2 * c + (d.first_piece ? 0 : 1);
                float* po = p.part_o + ((size_t)slot * 16 + h) * E;
#pragma unroll
                for (int j = 0; j < EC; ++j)
                    *reinterpret_cast<float4*>(po + 4 * (sub + 8 * j)) =
                        make_float4(o[j][0] * inv, o[j][1] * inv, o[j][2] * inv, o[j][3] * inv);
                if (sub == 0) p.part_lse[slot * 16 + h] = lse2;
            }
        }
        __syncthreads();
        st_c = (st_c + 1 == STAGES) ? 0 : st_c + 1;
        st_p = (st_p + 1 == STAGES) ? 0 : st_p + 1;
    }
    cp_async_wait<0>();
}

// ==================================================================================
// merge of split segments (and zeros for rows that see no key)
// one CTA per segment, 128 threads: thread t -> row t/8, columns 4*((t%8) + 8k)
// ==================================================================================

// Thread layout of the merge: TPR threads per query row, each owning NC 4-column groups
// (c4, c4 + TPR, ...), 16 rows per block; pieces are loaded B at a time.  Up to E = 128 a
// thread owns one group; at E = 256 two, so the block stays at 512 threads and the B * NC
// values in flight fit in registers (a 1024-thread block would get 64 and spill).
template <int E>
struct MergeCfg {
    static constexpr int C4 = E / 4;
    static constexpr int TPR = C4 < 32 ? C4 : 32;
    static constexpr int NC = C4 / TPR;
    static constexpr int NTH = 16 * TPR;
    static constexpr int B = 16 / NC;
};

// Merge of one (row, KV head) segment; all threads of the block call it with the same
// segment.  Pieces are consumed in batches of B whose loads are all in flight before any
// is used (the merge is latency-bound, not bandwidth-bound).
template <class T, int E>
__device__ __forceinline__ void merge_segment(const PagedParams& p, int g_seg, const long long* cst, int n, int* s_part) {
    using MC = MergeCfg<E>;
    constexpr int TPR = MC::TPR, NC = MC::NC, NTH = MC::NTH, B = MC::B;
    const int ws = g_seg / p.Hkv, hkv = g_seg - ws * p.Hkv;
    const int tid = threadIdx.x, r = tid / TPR, c4 = tid - r * TPR;
    const long long P0 = p.P[ws], V = p.P[ws + 1] - P0;
    const int w = ws / p.S, s = ws - w * p.S;
    const size_t orow = ((size_t)w * p.Hq + hkv * p.gqa + r) * p.S + s;
    if (V == 0) {
        if (r < p.gqa) {
#pragma unroll
            for (int k = 0; k < NC; ++k) {
                const int q = c4 + TPR * k;
                store_quad<T>(static_cast<T*>(p.out) + orow * E + 4 * q, 0.f, 0.f, 0.f, 0.f);
                if (p.out_f32) reinterpret_cast<float4*>(p.out_f32 + orow * E)[q] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
            if (p.lse_out && c4 == 0) p.lse_out[orow] = neg_inf();
        }
        return;
    }
    const long long b = P0 * p.hsplit + (p.hsplit > 1 ? hkv * V : 0);
    const int ca = cta_of(cst, b, n), cb = cta_of(cst, b + V - 1, n);
    if (ca == cb) return;
    const int npc = cb - ca + 1;
    const int hh = p.slot_heads > 1 ? hkv : 0;
    const bool ca_not_first = cst[ca] < b;
    float4 acc[NC];
#pragma unroll
    for (int k = 0; k < NC; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    float M = neg_inf(), den = 0.f;
    for (int base = 0; base < npc; base += NTH) {
        const int cnt = min(NTH, npc - base);
        __syncthreads();
        if (tid < cnt) {
            const int cc = ca + base + tid;
            const int slot = (cc == ca && ca_not_first) ? 2 * ca + 1 : 2 * cc;
            // a CTA whose range is empty (boundaries snapped together) wrote no piece
            s_part[tid] = cst[cc] == cst[cc + 1] ? -1 : (slot * p.slot_heads + hh) * 16;
        }
        __syncthreads();
        if (r >= p.gqa) continue;
        for (int k0 = 0; k0 < cnt; k0 += B) {
            float l[B];
            float4 v[B][NC];
#pragma unroll
            for (int j = 0; j < B; ++j) {
                l[j] = neg_inf();
#pragma unroll
                for (int k = 0; k < NC; ++k) v[j][k] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (k0 + j < cnt && s_part[k0 + j] >= 0) {
                    const int pi = s_part[k0 + j] + r;
                    l[j] = p.part_lse[pi];
#pragma unroll
                    for (int k = 0; k < NC; ++k)
                        v[j][k] = reinterpret_cast<const float4*>(p.part_o + (size_t)pi * E)[c4 + TPR * k];
                }
            }
            float mb = M;
#pragma unroll
            for (int j = 0; j < B; ++j) mb = fmaxf(mb, l[j]);
            if (mb == neg_inf()) continue;
            const float sc = fast_exp2(M - mb);
            den *= sc;
#pragma unroll
            for (int k = 0; k < NC; ++k) {
                acc[k].x *= sc; acc[k].y *= sc; acc[k].z *= sc; acc[k].w *= sc;
            }
#pragma unroll
            for (int j = 0; j < B; ++j) {
                const float wj = fast_exp2(l[j] - mb);  // 0 for empty pieces
                den += wj;
#pragma unroll
                for (int k = 0; k < NC; ++k) {
                    acc[k].x += wj * v[j][k].x; acc[k].y += wj * v[j][k].y;
                    acc[k].z += wj * v[j][k].z; acc[k].w += wj * v[j][k].w;
                }
            }
            M = mb;
        }
    }
    if (r >= p.gqa) return;
    const float inv = den > 0.f ? 1.f / den : 0.f;
#pragma unroll
    for (int k = 0; k < NC; ++k) {
        const int q = c4 + TPR * k;
        const float4 o = make_float4(acc[k].x * inv, acc[k].y * inv, acc[k].z * inv, acc[k].w * inv);
        store_quad<T>(static_cast<T*>(p.out) + orow * E + 4 * q, o.x, o.y, o.z, o.w);
        if (p.out_f32) reinterpret_cast<float4*>(p.out_f32 + orow * E)[q] = o;
    }
    if (p.lse_out && c4 == 0) p.lse_out[orow] = den > 0.f ? (M + __log2f(den)) * kLn2 : neg_inf();
}

// Grid-stride over the (row, KV head) segments: few blocks, so that while they wait for
// the attention grid they hold few of the slots the next call's attention CTAs need.
template <class T, int E>
__global__ void __launch_bounds__(MergeCfg<E>::NTH) decode_merge_kernel(PagedParams p) {
    constexpr int NTH = MergeCfg<E>::NTH;
    // launched as a programmatic dependent of the attention kernel: wait for its results
    // let the next call's schedule kernel start its (read-only) work now
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int tid = threadIdx.x;
    // The CTA boundaries are searched twice below: stage them in shared memory with one
    // round of parallel loads instead of a chain of dependent global loads.
    constexpr int kMaxC = 1024;
    __shared__ long long s_cs[kMaxC + 1];
    const bool cs_shared = p.n_launch <= kMaxC;
    if (cs_shared)
        for (int i = tid; i <= p.n_launch; i += NTH) s_cs[i] = p.cstart[i];
    const DecodeSched sch = *p.sched;
    if (sch.error) {
        // a bounded wait of the attention kernel gave up: every output of the call is
        // marked invalid (NaN) rather than merged from pieces that may be missing
        const float nan = __int_as_float(0x7fc00000);
        for (int g_seg = blockIdx.x; g_seg < p.WS * p.Hkv; g_seg += gridDim.x) {
            const int ws = g_seg / p.Hkv, hkv = g_seg - ws * p.Hkv;
            constexpr int TPR = MergeCfg<E>::TPR;
            const int r = tid / TPR, c4 = tid - r * TPR;
            if (r >= p.gqa) continue;
            const int w = ws / p.S, s = ws - w * p.S;
            const size_t orow = ((size_t)w * p.Hq + hkv * p.gqa + r) * p.S + s;
            for (int q = c4; q < E / 4; q += TPR) {
                store_quad<T>(static_cast<T*>(p.out) + orow * E + 4 * q, nan, nan, nan, nan);
                if (p.out_f32) reinterpret_cast<float4*>(p.out_f32 + orow * E)[q] = make_float4(nan, nan, nan, nan);
            }
            if (p.lse_out && c4 == 0) p.lse_out[orow] = nan;
        }
        return;
    }
    __syncthreads();
    const long long* cst = cs_shared ? s_cs : p.cstart;
    __shared__ int s_part[NTH];
    for (int g_seg = blockIdx.x; g_seg < p.WS * p.Hkv; g_seg += gridDim.x)
        merge_segment<T, E>(p, g_seg, cst, sch.n_eff, s_part);
}

// ==================================================================================
// host side
// ==================================================================================
namespace {

struct KernelChoice {
    const void* fn;
    size_t smem;
    int nt;
    int min_units;
    bool tma = false;
    bool row = false;  // all KV heads per CTA (hsplit = 1)
    int cw = 4;
    size_t sched_smem = 0;  // shared bytes the row kernel lends to its in-kernel schedule
};

template <class T, int E, int CW, int STAGES>
KernelChoice row_choice() {
    using C = RowCfg<T, E, CW, STAGES>;
    KernelChoice k{reinterpret_cast<const void*>(&decode_row_kernel<T, E, CW, STAGES>), C::SMEM, C::NT, 64, true};
    k.row = true;
    k.cw = CW;
    k.sched_smem = 2 * C::OFF_V;
    return k;
}

// Row kernel: 16-bit types, Hkv in {1, 2, 4} (4 consumer warps) or 8 (8 warps), pages
// that tile the TOKB = 16*CW/Hkv-key windows.
bool pick_row(int dtype, int E, int Hkv, int BS, long long NB, KernelChoice& kc) {
    if (dtype != DVATTN_FLOAT16 && dtype != DVATTN_BFLOAT16) return false;
    if (!(Hkv == 1 || Hkv == 2 || Hkv == 4 || Hkv == 8)) return false;
    if (Hkv == 8 && E != 128 && E != 64) return false;
    const int cw = Hkv == 8 ? 8 : 4;
    const int tokb = 16 * cw / Hkv;
    const bool small = BS >= 8 && BS <= tokb && (tokb % BS) == 0;
    const bool big = BS > tokb && (BS % tokb) == 0;
    if (!(small || big) || NB <= 0 || NB * (long long)BS > 0x7fffffffLL) return false;
#define DVB_ROW(TT)                                                              \
    if (cw == 8) {                                                               \
        if (E == 64) { kc = row_choice<TT, 64, 8, 3>(); return true; }           \
        if (E == 128) { kc = row_choice<TT, 128, 8, 3>(); return true; }         \
    } else {                                                                     \
        if (E == 64) { kc = row_choice<TT, 64, 4, 3>(); return true; }           \
        if (E == 128) { kc = row_choice<TT, 128, 4, 3>(); return true; }         \
        if (E == 256) { kc = row_choice<TT, 256, 4, 2>(); return true; }         \
    }
    if (dtype == DVATTN_FLOAT16) { DVB_ROW(__half) } else { DVB_ROW(__nv_bfloat16) }
#undef DVB_ROW
    return false;
}

template <class T, int E>
KernelChoice tma_choice() {
    constexpr int STAGES = 3;
    using C = TmaCfg<T, E, STAGES>;
    return {reinterpret_cast<const void*>(&decode_tma_kernel<T, E, STAGES>), C::SMEM, C::NT, C::TILE, true};
}

// TMA path: 16-bit types, pages that tile the 64-key windows (BS | 64 with BS >= 8, or
// 64 | BS), and pool token indices that fit the 32-bit TMA coordinate.
bool tma_eligible(int dtype, int BS, long long NB) {
    if (dtype != DVATTN_FLOAT16 && dtype != DVATTN_BFLOAT16) return false;
    const bool small = BS >= 8 && BS <= 64 && (64 % BS) == 0;
    const bool big = BS > 64 && (BS % 64) == 0;
    return (small || big) && NB > 0 && NB * (long long)BS <= 0x7fffffffLL;
}

bool pick_tma(int dtype, int E, KernelChoice& kc) {
    if (dtype == DVATTN_FLOAT16) {
        if (E == 64) { kc = tma_choice<__half, 64>(); return true; }
        if (E == 128) { kc = tma_choice<__half, 128>(); return true; }
        if (E == 256) { kc = tma_choice<__half, 256>(); return true; }
    } else if (dtype == DVATTN_BFLOAT16) {
        if (E == 64) { kc = tma_choice<__nv_bfloat16, 64>(); return true; }
        if (E == 128) { kc = tma_choice<__nv_bfloat16, 128>(); return true; }
        if (E == 256) { kc = tma_choice<__nv_bfloat16, 256>(); return true; }
    }
    return false;
}


template <class T, int E>
KernelChoice tc_choice() {
    constexpr int WARPS = 4, STAGES = (E <= 128) ? 3 : 2;
    using C = TcCfg<T, E, WARPS, STAGES>;
    return {reinterpret_cast<const void*>(&decode_tc_kernel<T, E, WARPS, STAGES>), C::SMEM, C::NT, C::TILE};
}
template <int E>
KernelChoice f32_choice() {
    constexpr int STAGES = (E <= 128) ? 3 : 2;
    using C = F32Cfg<E, STAGES>;
    return {reinterpret_cast<const void*>(&decode_f32_kernel<E, STAGES>), C::SMEM, C::NT, C::TILE};
}

bool pick_kernel(int dtype, int E, KernelChoice& kc) {
    switch (dtype) {
        case DVATTN_FLOAT16:
            if (E == 64) { kc = tc_choice<__half, 64>(); return true; }
            if (E == 128) { kc = tc_choice<__half, 128>(); return true; }
            if (E == 256) { kc = tc_choice<__half, 256>(); return true; }
            return false;
        case DVATTN_BFLOAT16:
            if (E == 64) { kc = tc_choice<__nv_bfloat16, 64>(); return true; }
            if (E == 128) { kc = tc_choice<__nv_bfloat16, 128>(); return true; }
            if (E == 256) { kc = tc_choice<__nv_bfloat16, 256>(); return true; }
            return false;
        case DVATTN_FLOAT32:
            if (E == 64) { kc = f32_choice<64>(); return true; }
            if (E == 128) { kc = f32_choice<128>(); return true; }
            if (E == 256) { kc = f32_choice<256>(); return true; }
            return false;
        default:
            return false;
    }
}

}  // namespace

int decode_validate(const dvattn_paged_args* a) {
    if (!a) return DVATTN_ERR_INVALID_ARGUMENT;
    if (a->dtype < 0 || a->dtype > 2) return DVATTN_ERR_UNSUPPORTED;
    if (a->F < 0 || a->W < 0 || a->Hq < 0 || a->Hkv <= 0 || a->E <= 0 || a->Ev <= 0 || a->S < 0 || a->R < 0 ||
        a->block_size <= 0 || a->max_blocks_per_seq < 0)
        return DVATTN_ERR_INVALID_ARGUMENT;
    if (a->R > a->E || (a->R & 1)) return DVATTN_ERR_INVALID_ARGUMENT;
    if (a->Hq % a->Hkv) return DVATTN_ERR_INVALID_ARGUMENT;
    const int gqa = a->Hq / a->Hkv;
    if (gqa > 16 || (a->Hq > 0 && gqa < 1)) return DVATTN_ERR_UNSUPPORTED;
    if (a->E != a->Ev) return DVATTN_ERR_UNSUPPORTED;
    KernelChoice kc;
    if (!pick_kernel(a->dtype, a->E, kc)) return DVATTN_ERR_UNSUPPORTED;
    return DVATTN_OK;
}

// SM count x resident CTAs of a kernel on the current device, computed once per
// (device, kernel) and cached: the attribute / occupancy queries cost microseconds of
// host time per call otherwise.
static int device_sms_and_occ(const KernelChoice& kc, int& n_launch) {
    struct Entry {
        int dev;
        const void* fn;
        int n;
    };
    static Entry cache[256];
    static int ncache = 0;
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return DVATTN_ERR_CUDA;
    {
        std::lock_guard<std::mutex> lk(mu);
        for (int i = 0; i < ncache; ++i)
            if (cache[i].dev == dev && cache[i].fn == kc.fn) {
                n_launch = cache[i].n;
                return DVATTN_OK;
            }
    }
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return DVATTN_ERR_CUDA;
    if (cudaFuncSetAttribute(kc.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kc.smem) != cudaSuccess)
        return DVATTN_ERR_CUDA;
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kc.fn, kc.nt, kc.smem) != cudaSuccess) return DVATTN_ERR_CUDA;
    if (occ < 1) occ = 1;
    n_launch = sms * occ;
    std::lock_guard<std::mutex> lk(mu);
    if (ncache < 256) cache[ncache++] = {dev, kc.fn, n_launch};
    return DVATTN_OK;
}

struct DecodeLayout {
    size_t off_P, off_rs, off_cs, off_po, off_pl, off_fd, off_fm, total;
};
static DecodeLayout decode_layout(int WS, int E, int n_launch, bool varlen, int slot_heads, int nfrag = 0) {
    auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
    DecodeLayout L;
    L.off_P = 256;
    L.off_rs = L.off_P + up(sizeof(long long) * (size_t)(WS + 1));
    L.off_cs = L.off_rs + (varlen ? up(sizeof(int) * (size_t)WS) : 0);
    L.off_po = L.off_cs + up(sizeof(long long) * (size_t)(n_launch + 1));
    L.off_pl = L.off_po + up(sizeof(float) * (size_t)n_launch * 2 * slot_heads * 16 * E);
    L.off_fd = L.off_pl + up(sizeof(float) * (size_t)n_launch * 2 * slot_heads * 16);
    L.off_fm = L.off_fd + up(sizeof(FragDesc) * (size_t)nfrag);
    L.total = L.off_fm + (size_t)nfrag * 256;  // K and V tensor maps of each fragment (row kernel)
    return L;
}

static bool choose(int dtype, int E, int Hkv, int BS, long long NB, KernelChoice& kc) {
    if (pick_row(dtype, E, Hkv, BS, NB, kc)) return true;
    if (tma_eligible(dtype, BS, NB) && pick_tma(dtype, E, kc)) return true;
    return pick_kernel(dtype, E, kc);
}

// Contiguous fragments: the row kernel with one 5-D TMA box per window where it applies
// (16-bit types, Hkv in {1, 2, 4, 8}); the cp.async kernels otherwise.
// DVATTN_SDPA_ROW=0 keeps every call on the cp.async kernels.
// Every fragment needs at least one row for its tensor map (an empty one goes the cp.async way).
static bool choose_sdpa(int dtype, int E, int Hkv, bool all_rows, KernelChoice& kc) {
    const char* env = getenv("DVATTN_SDPA_ROW");
    if (all_rows && !(env && env[0] == '0')) {
        const int tokb = 16 * (Hkv == 8 ? 8 : 4) / (Hkv > 0 ? Hkv : 1);
        if (pick_row(dtype, E, Hkv, tokb, 1, kc)) return true;
    }
    return pick_kernel(dtype, E, kc);
}

size_t decode_workspace_size(const dvattn_paged_args* a) {
    if (decode_validate(a) != DVATTN_OK) return 0;
    KernelChoice kc;
    choose(a->dtype, a->E, a->Hkv, a->block_size, a->num_blocks, kc);
    int n_launch = 0;
    if (device_sms_and_occ(kc, n_launch) != DVATTN_OK) return 0;
    return decode_layout(a->W * a->S, a->E, n_launch, false, kc.row ? a->Hkv : 1).total;
}

// Programmatic dependent launch lets a call's first kernel start while the kernel before it
// in the stream still runs, and that kernel reads its inputs (block tables, locations,
// queries, pages) before its griddepcontrol.wait.  That is sound only while the kernel
// before it does not write those inputs.  This library's own kernels let their dependents
// launch early, so the launcher remembers, per (device, stream), the output ranges of its
// last call there and launches the next call's first kernel as an ordinary, fully ordered
// launch when one of its inputs overlaps them (a call whose queries are the previous call's
// output).  Early-triggering kernels of other libraries are not visible here:
// DVATTN_PDL=0 makes every call's first kernel an ordinary launch.
struct Span {
    uintptr_t lo, hi;
};
static Span span_of(const void* p, long long bytes) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    return (p && bytes > 0) ? Span{a, a + (uintptr_t)bytes} : Span{0, 0};
}
struct LastOutputs {
    int dev;
    cudaStream_t stream;
    Span out[3];
};
static std::mutex g_last_mu;
static LastOutputs g_last[64];
static int g_last_n = 0, g_last_next = 0;

static bool pdl_enabled() {
    static const bool on = [] {
        const char* e = getenv("DVATTN_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

// DVATTN_TEST_STALL_TILE=<i>: tests only.  CTA 0 of the row kernel skips the loads of its
// tile i, so the consumers' bounded wait runs out (after ~2 s) and the call's error word
// is set; read once per process.
static int stall_tile_hook() {
    static const int t = [] {
        const char* e = getenv("DVATTN_TEST_STALL_TILE");
        return e && *e ? atoi(e) : -1;
    }();
    return t;
}

static bool first_launch_may_overlap(int dev, cudaStream_t s, const Span* in, int nin) {
    if (!pdl_enabled()) return false;
    std::lock_guard<std::mutex> lk(g_last_mu);
    for (int i = 0; i < g_last_n; ++i) {
        if (g_last[i].dev != dev || g_last[i].stream != s) continue;
        for (const Span& o : g_last[i].out)
            for (int j = 0; j < nin; ++j)
                if (o.lo < o.hi && in[j].lo < in[j].hi && in[j].lo < o.hi && o.lo < in[j].hi) return false;
        return true;
    }
    return true;
}

static void remember_outputs(int dev, cudaStream_t s, const Span* out) {
    std::lock_guard<std::mutex> lk(g_last_mu);
    int slot = -1;
    for (int i = 0; i < g_last_n; ++i)
        if (g_last[i].dev == dev && g_last[i].stream == s) slot = i;
    if (slot < 0) {
        if (g_last_n < 64) {
            slot = g_last_n++;
        } else {
            slot = g_last_next;
            g_last_next = (g_last_next + 1) % 64;
        }
    }
    g_last[slot] = LastOutputs{dev, s, {out[0], out[1], out[2]}};
}

// Runs prep -> split kernel -> merge for a filled PagedParams (pointers, sizes, R,
// cs_stride, cu_q/nseq); fills the workspace-derived fields.
static int run_schedule(PagedParams p, int dtype, void* workspace, size_t wbytes, cudaStream_t stream, int phase) {
    KernelChoice kc;
    bool all_rows = true;
    for (int f = 0; f < p.nfrag; ++f) all_rows = all_rows && p.frag[f].rows > 0;
    if (p.nfrag ? !choose_sdpa(dtype, p.E, p.Hkv, all_rows, kc) : !choose(dtype, p.E, p.Hkv, p.BS, p.NB, kc))
        return DVATTN_ERR_UNSUPPORTED;
    int n_launch = 0;
    int st = device_sms_and_occ(kc, n_launch);
    if (st != DVATTN_OK) return st;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return DVATTN_ERR_CUDA;
    const int esz = dtype == DVATTN_FLOAT32 ? 4 : 2;
    const long long rowsz = (long long)p.WS * p.Hq * p.E;  // elements of queries / out per turn
    std::vector<Span> in_spans;
    in_spans.reserve(10 + 2 * (size_t)p.nfrag);
    in_spans.push_back(span_of(p.q, (p.nfrag ? p.F : 1) * rowsz * esz));
    in_spans.push_back(span_of(p.loc, 4LL * p.F * p.WS));
    in_spans.push_back(span_of(p.L, 4LL * p.F));
    in_spans.push_back(span_of(p.cos, 4LL * p.F * p.WS * p.cs_stride));
    in_spans.push_back(span_of(p.sin, 4LL * p.F * p.WS * p.cs_stride));
    in_spans.push_back(span_of(p.bt, 4LL * (p.cu_q ? p.nseq : p.W) * p.maxb));
    in_spans.push_back(span_of(p.cu_q, 4LL * (p.nseq + 1)));
    in_spans.push_back(span_of(p.k, p.NB * p.BS * p.Hkv * p.E * esz));
    in_spans.push_back(span_of(p.v, p.NB * p.BS * p.Hkv * p.E * esz));
    for (int f = 0; f < p.nfrag; ++f) {
        const long long fb = (long long)p.frag[f].rows * (p.frag[f].wmul ? p.W : 1) * p.Hkv * p.E * esz;
        in_spans.push_back(span_of(p.frag[f].k, fb));
        in_spans.push_back(span_of(p.frag[f].v, fb));
    }
    const Span out_spans[3] = {span_of(p.out, rowsz * esz), span_of(p.out_f32, rowsz * 4),
                               span_of(p.lse_out, 4LL * p.WS * p.Hq)};
    p.hsplit = kc.row ? 1 : p.Hkv;
    p.bs_shift = (p.BS & (p.BS - 1)) == 0 ? __builtin_ctz((unsigned)p.BS) : -1;
    p.slot_heads = kc.row ? p.Hkv : 1;
    const DecodeLayout L = decode_layout(p.WS, p.E, n_launch, p.cu_q != nullptr, p.slot_heads, p.nfrag);
    if (!workspace || wbytes < L.total || (reinterpret_cast<uintptr_t>(workspace) & 255)) return DVATTN_ERR_WORKSPACE;
    char* wsb = static_cast<char*>(workspace);
    p.sched = reinterpret_cast<DecodeSched*>(wsb);
    p.P = reinterpret_cast<long long*>(wsb + L.off_P);
    p.row_seq = p.cu_q ? reinterpret_cast<int*>(wsb + L.off_rs) : nullptr;
    p.part_o = reinterpret_cast<float*>(wsb + L.off_po);
    p.part_lse = reinterpret_cast<float*>(wsb + L.off_pl);
    p.cstart = reinterpret_cast<long long*>(wsb + L.off_cs);
    alignas(64) FragMaps fm;
    memset(&fm, 0, sizeof(fm));
    if (p.nfrag && kc.row && p.nfrag <= kParamFrags) {
        // few fragments: their tensor maps travel as a kernel parameter (no copy in the
        // stream, so consecutive calls' kernels still overlap)
        const int boxr = 16 * kc.cw / p.Hkv;
        for (int f = 0; f < p.nfrag; ++f) {
            const FragDesc& fd = p.frag[f];
            const int B = fd.wmul ? p.W : 1;
            if (!encode_fragment_map(&fm.m[2 * f], fd.k, dtype, p.E, p.Hkv, fd.rows, B, boxr) ||
                !encode_fragment_map(&fm.m[2 * f + 1], fd.v, dtype, p.E, p.Hkv, fd.rows, B, boxr))
                return DVATTN_ERR_CUDA;
            fm.wmul[f] = fd.wmul;
        }
        p.frag = nullptr;
        p.fmaps = nullptr;
    } else if (p.nfrag) {
        // the fragment descriptors (and, for the row kernel, each fragment's K and V tensor
        // maps) travel in the workspace: one copy from a host staging array
        if (phase == DVATTN_PHASE_ALL || phase == DVATTN_PHASE_SCHEDULE) {
            std::vector<unsigned char> stage(L.total - L.off_fd, 0);
            memcpy(stage.data(), p.frag, sizeof(FragDesc) * (size_t)p.nfrag);
            size_t n = sizeof(FragDesc) * (size_t)p.nfrag;
            if (kc.row) {
                const int boxr = 16 * kc.cw / p.Hkv;
                for (int f = 0; f < p.nfrag; ++f) {
                    const FragDesc& fd = p.frag[f];
                    alignas(64) CUtensorMap m[2];
                    const int B = fd.wmul ? p.W : 1;
                    if (!encode_fragment_map(&m[0], fd.k, dtype, p.E, p.Hkv, fd.rows, B, boxr) ||
                        !encode_fragment_map(&m[1], fd.v, dtype, p.E, p.Hkv, fd.rows, B, boxr))
                        return DVATTN_ERR_CUDA;
                    memcpy(stage.data() + (L.off_fm - L.off_fd) + (size_t)f * 256, m, sizeof(m));
                }
                n = stage.size();
            }
            if (cudaMemcpyAsync(wsb + L.off_fd, stage.data(), n, cudaMemcpyHostToDevice, stream) != cudaSuccess)
                return DVATTN_ERR_CUDA;
        }
        p.frag = reinterpret_cast<const FragDesc*>(wsb + L.off_fd);
        p.fmaps = wsb + L.off_fm;
    }
    {
        // a query rotation costs about as long as streaming ~96 KB of the cache
        const long long unit_bytes = (long long)(kc.row ? p.Hkv : 1) * 2 * p.E * esz;
        const long long ru = (96 * 1024) / unit_bytes;
        p.rot_units = (int)(ru < 8 ? 8 : ru);
    }
    p.n_launch = n_launch;
    p.min_units = kc.min_units;
    {
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return DVATTN_ERR_CUDA;
        p.n_sm = sms;
        p.unit_bytes = (long long)(kc.row ? p.Hkv : 1) * 2 * p.E * esz;
    }
    // Row kernel on paged decode: the split is computed inside the attention kernel (its
    // stages hold the prefix sums; CTA c publishes P[32c..32c+31] for the merge), so no
    // prep kernel runs and a call's streaming starts while the previous call's merge runs.
    p.fused = (kc.row && !p.cu_q && (size_t)(p.WS + 1 + 32) * 8 <= kc.sched_smem &&
               (long long)p.WS + 1 <= 32LL * n_launch) ? 1 : 0;
    p.stall_tile = stall_tile_hook();
    p.rotate = kc.row ? 1 : 0;

    // the first kernel this call launches may overlap the kernel before it only if that
    // kernel cannot have written this call's inputs (see first_launch_may_overlap)
    const bool overlap_ok = first_launch_may_overlap(dev, stream, in_spans.data(), (int)in_spans.size());
    if ((phase == DVATTN_PHASE_ALL || phase == DVATTN_PHASE_SCHEDULE) && !p.fused) {
        // programmatic dependent of whatever precedes it (the previous call's merge): it
        // computes the schedule before waiting, and writes it after
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(1);
        cfg.blockDim = dim3(1024);
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = overlap_ok ? 1 : 0;
        void* pargs[] = {&p};
        if (cudaLaunchKernelExC(&cfg, (const void*)&decode_prep_kernel, pargs) != cudaSuccess) return DVATTN_ERR_CUDA;
    }
    if (phase == DVATTN_PHASE_ALL || phase == DVATTN_PHASE_ATTEND) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(n_launch);
        cfg.blockDim = dim3(kc.nt);
        cfg.dynamicSmemBytes = kc.smem;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        // the fused row kernel reads its inputs before griddepcontrol.wait; the others wait
        // first (for the schedule kernel)
        cfg.numAttrs = (!p.fused || overlap_ok) ? 1 : 0;
        if (kc.tma) {
            alignas(64) CUtensorMap mk, mv;
            const int win = kc.row ? 16 * kc.cw / p.Hkv : 64;
            int boxr = p.BS < win ? p.BS : win;
            if (p.nfrag) {
                boxr = win;  // one fragment box per window; the maps are in fm or the workspace
                memset(&mk, 0, sizeof(mk));
                memset(&mv, 0, sizeof(mv));
            } else {
                const long long tokens = p.NB * p.BS;
                auto enc = kc.row ? encode_cache_map_all_heads : encode_cache_map;
                if (!enc(&mk, p.k, dtype, p.E, p.Hkv, tokens, boxr) || !enc(&mv, p.v, dtype, p.E, p.Hkv, tokens, boxr))
                    return DVATTN_ERR_CUDA;
            }
            if (kc.row) {
                void* args[] = {&p, &mk, &mv, &boxr, &fm};
                if (cudaLaunchKernelExC(&cfg, kc.fn, args) != cudaSuccess) return DVATTN_ERR_CUDA;
            } else {
                void* args[] = {&p, &mk, &mv, &boxr};
                if (cudaLaunchKernelExC(&cfg, kc.fn, args) != cudaSuccess) return DVATTN_ERR_CUDA;
            }
        } else {
            void* args[] = {&p};
            if (cudaLaunchKernelExC(&cfg, kc.fn, args) != cudaSuccess) return DVATTN_ERR_CUDA;
        }
    }
    if (phase == DVATTN_PHASE_ALL || phase == DVATTN_PHASE_MERGE) {
        const void* mk = nullptr;
        switch (dtype) {
            case DVATTN_FLOAT16:
                mk = p.E == 64 ? (const void*)&decode_merge_kernel<__half, 64>
                   : p.E == 128 ? (const void*)&decode_merge_kernel<__half, 128> : (const void*)&decode_merge_kernel<__half, 256>;
                break;
            case DVATTN_BFLOAT16:
                mk = p.E == 64 ? (const void*)&decode_merge_kernel<__nv_bfloat16, 64>
                   : p.E == 128 ? (const void*)&decode_merge_kernel<__nv_bfloat16, 128>
                                : (const void*)&decode_merge_kernel<__nv_bfloat16, 256>;
                break;
            default:
                mk = p.E == 64 ? (const void*)&decode_merge_kernel<float, 64>
                   : p.E == 128 ? (const void*)&decode_merge_kernel<float, 128> : (const void*)&decode_merge_kernel<float, 256>;
                break;
        }
        cudaLaunchConfig_t cfg = {};
#ifndef DVB_MERGE_CTAS
#define DVB_MERGE_CTAS 64
#endif
        // few blocks (grid-stride over the segments): they hold few of the slots the next
        // call's attention CTAs need while they wait for this call's attention grid
        const long long nseg = (long long)p.WS * p.Hkv;
        cfg.gridDim = dim3((unsigned)(nseg < DVB_MERGE_CTAS ? nseg : DVB_MERGE_CTAS));
        cfg.blockDim = dim3(p.E == 64 ? MergeCfg<64>::NTH : p.E == 128 ? MergeCfg<128>::NTH : MergeCfg<256>::NTH);
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        void* margs[] = {&p};
        if (cudaLaunchKernelExC(&cfg, mk, margs) != cudaSuccess) return DVATTN_ERR_CUDA;
    }
    if (phase != DVATTN_PHASE_SCHEDULE) remember_outputs(dev, stream, out_spans);
    return cudaGetLastError() == cudaSuccess ? DVATTN_OK : DVATTN_ERR_CUDA;
}

static bool misaligned16(const void* a) { return (reinterpret_cast<uintptr_t>(a) & 15) != 0; }

int decode_launch(const dvattn_paged_args* a, void* workspace, size_t wbytes, cudaStream_t stream, int phase) {
    if (phase < DVATTN_PHASE_ALL || phase > DVATTN_PHASE_MERGE) return DVATTN_ERR_INVALID_ARGUMENT;
    int st = decode_validate(a);
    if (st != DVATTN_OK) return st;
    const int WS = a->W * a->S;
    if (WS == 0 || a->Hq == 0) return DVATTN_OK;
    if (!a->out || !a->queries || !a->k_cache || !a->v_cache || !a->block_tables ||
        (a->F > 0 && (!a->locations || !a->fragment_lengths)))
        return DVATTN_ERR_INVALID_ARGUMENT;
    if (a->R > 0 && (!a->cosines || !a->sines)) return DVATTN_ERR_INVALID_ARGUMENT;
    if (misaligned16(a->queries) || misaligned16(a->k_cache) || misaligned16(a->v_cache) || misaligned16(a->out) ||
        (a->out_f32 && misaligned16(a->out_f32)))
        return DVATTN_ERR_INVALID_ARGUMENT;

    PagedParams p{};
    p.F = a->F; p.W = a->W; p.Hq = a->Hq; p.Hkv = a->Hkv; p.E = a->E; p.S = a->S; p.R = a->R;
    p.BS = a->block_size; p.maxb = a->max_blocks_per_seq; p.WS = WS; p.gqa = a->Hq / a->Hkv;
    const long long cap = (long long)a->max_blocks_per_seq * a->block_size;
    p.cap = cap > 0x7fffffffLL ? 0x7fffffff : (int)cap;
    p.NB = a->num_blocks;
    p.scale_log2 = a->scale * kLog2e;
    p.out = a->out; p.q = a->queries; p.cos = a->cosines; p.sin = a->sines; p.loc = a->locations;
    p.L = a->fragment_lengths; p.k = a->k_cache; p.v = a->v_cache; p.bt = a->block_tables;
    p.lse_out = a->lse_out; p.out_f32 = a->out_f32;
    p.cu_q = nullptr; p.nseq = 0; p.cs_stride = a->R;
    return run_schedule(p, a->dtype, workspace, wbytes, stream, phase);
}

// ---------------------------------------------------------------------------------
// varlen prefill through the same schedule: packed token t is query row ws = t of a
// decode with W = T, S = 1; its block-table row comes from cu_seqlens_q and its cos/sin
// rows are half width ([F,T,R/2]).
// ---------------------------------------------------------------------------------
static dvattn_paged_args varlen_as_paged(const dvattn_varlen_args* v) {
    dvattn_paged_args a{};
    a.dtype = v->dtype; a.F = v->F; a.W = v->T; a.Hq = v->Hq; a.Hkv = v->Hkv; a.E = v->E; a.Ev = v->Ev; a.S = 1;
    a.R = v->R; a.block_size = v->block_size; a.max_blocks_per_seq = v->max_blocks_per_seq;
    a.num_blocks = v->num_blocks; a.scale = v->scale;
    return a;
}

size_t varlen_workspace_size(const dvattn_varlen_args* v) {
    if (!v || v->W < 0 || v->T < 0) return 0;
    dvattn_paged_args a = varlen_as_paged(v);
    if (decode_validate(&a) != DVATTN_OK) return 0;
    if (prefill_eligible(v)) return prefill_workspace_size(v);
    KernelChoice kc;
    choose(a.dtype, a.E, a.Hkv, a.block_size, a.num_blocks, kc);
    int n_launch = 0;
    if (device_sms_and_occ(kc, n_launch) != DVATTN_OK) return 0;
    return decode_layout(v->T, v->E, n_launch, true, kc.row ? v->Hkv : 1).total;
}

int varlen_launch(const dvattn_varlen_args* v, void* workspace, size_t wbytes, cudaStream_t stream, int phase) {
    if (!v || v->W < 0 || v->T < 0) return DVATTN_ERR_INVALID_ARGUMENT;
    dvattn_paged_args a = varlen_as_paged(v);
    int st = decode_validate(&a);
    if (st != DVATTN_OK) return st;
    if (v->T == 0 || v->Hq == 0) return DVATTN_OK;
    if (!v->out || !v->queries || !v->k_cache || !v->v_cache || !v->block_tables || !v->cu_seqlens_q ||
        (v->F > 0 && (!v->locations || !v->fragment_lengths)))
        return DVATTN_ERR_INVALID_ARGUMENT;
    if (v->R > 0 && (!v->cosines || !v->sines)) return DVATTN_ERR_INVALID_ARGUMENT;
    if (misaligned16(v->queries) || misaligned16(v->k_cache) || misaligned16(v->v_cache) || misaligned16(v->out) ||
        (v->out_f32 && misaligned16(v->out_f32)))
        return DVATTN_ERR_INVALID_ARGUMENT;
    if (phase < DVATTN_PHASE_ALL || phase > DVATTN_PHASE_MERGE) return DVATTN_ERR_INVALID_ARGUMENT;
    if (prefill_eligible(v)) return prefill_launch(v, workspace, wbytes, stream, phase);
    PagedParams p{};
    p.F = v->F; p.W = v->T; p.Hq = v->Hq; p.Hkv = v->Hkv; p.E = v->E; p.S = 1; p.R = v->R;
    p.BS = v->block_size; p.maxb = v->max_blocks_per_seq; p.WS = v->T; p.gqa = v->Hq / v->Hkv;
    const long long cap = (long long)v->max_blocks_per_seq * v->block_size;
    p.cap = cap > 0x7fffffffLL ? 0x7fffffff : (int)cap;
    p.NB = v->num_blocks;
    p.scale_log2 = v->scale * kLog2e;
    p.out = v->out; p.q = v->queries; p.cos = v->cosines; p.sin = v->sines; p.loc = v->locations;
    p.L = v->fragment_lengths; p.k = v->k_cache; p.v = v->v_cache; p.bt = v->block_tables;
    p.lse_out = v->lse_out; p.out_f32 = v->out_f32;
    p.cu_q = v->cu_seqlens_q; p.nseq = v->W; p.cs_stride = v->R / 2;
    return run_schedule(p, v->dtype, workspace, wbytes, stream, phase);
}

// ---------------------------------------------------------------------------------
// Contiguous fragments (dvattn_sdpa): the paged machinery with per-turn fragment
// addressing, per-turn rotated queries and no rotation.
static int sdpa_validate(const dvattn_sdpa_args* a) {
    if (!a) return DVATTN_ERR_INVALID_ARGUMENT;
    if (a->dtype < 0 || a->dtype > 2) return DVATTN_ERR_UNSUPPORTED;
    if (a->F < 1 || a->F > 4096 || a->W < 0 || a->Hq < 0 || a->Hkv <= 0 || a->E <= 0 || a->Ev <= 0 || a->S < 0)
        return DVATTN_ERR_INVALID_ARGUMENT;
    if (a->Hq % a->Hkv) return DVATTN_ERR_INVALID_ARGUMENT;
    const int gqa = a->Hq / a->Hkv;
    if (gqa > 16 || (a->Hq > 0 && gqa < 1)) return DVATTN_ERR_UNSUPPORTED;
    if (a->E != a->Ev) return DVATTN_ERR_UNSUPPORTED;
    KernelChoice kc;
    if (!pick_kernel(a->dtype, a->E, kc)) return DVATTN_ERR_UNSUPPORTED;
    if (!a->key_fragments || !a->value_fragments || !a->fragment_rows || !a->fragment_batch)
        return DVATTN_ERR_INVALID_ARGUMENT;
    for (int f = 0; f < a->F; ++f) {
        if (a->fragment_rows[f] < 0) return DVATTN_ERR_INVALID_ARGUMENT;
        if (a->fragment_batch[f] != 1 && a->fragment_batch[f] != a->W) return DVATTN_ERR_INVALID_ARGUMENT;
        if (a->fragment_rows[f] > 0 && (!a->key_fragments[f] || !a->value_fragments[f] ||
                                        misaligned16(a->key_fragments[f]) || misaligned16(a->value_fragments[f])))
            return DVATTN_ERR_INVALID_ARGUMENT;
    }
    return DVATTN_OK;
}

size_t sdpa_workspace_size(const dvattn_sdpa_args* a) {
    if (sdpa_validate(a) != DVATTN_OK) return 0;
    KernelChoice kc;
    bool all_rows = true;
    for (int f = 0; f < a->F; ++f) all_rows = all_rows && a->fragment_rows[f] > 0;
    choose_sdpa(a->dtype, a->E, a->Hkv, all_rows, kc);
    int n_launch = 0;
    if (device_sms_and_occ(kc, n_launch) != DVATTN_OK) return 0;
    return decode_layout(a->W * a->S, a->E, n_launch, false, kc.row ? a->Hkv : 1, a->F).total;
}

int sdpa_launch(const dvattn_sdpa_args* a, void* workspace, size_t wbytes, cudaStream_t stream) {
    int st = sdpa_validate(a);
    if (st != DVATTN_OK) return st;
    const int WS = a->W * a->S;
    if (WS == 0 || a->Hq == 0) return DVATTN_OK;
    if (!a->out || !a->queries || !a->locations || !a->fragment_lengths) return DVATTN_ERR_INVALID_ARGUMENT;
    if (misaligned16(a->queries) || misaligned16(a->out) || (a->out_f32 && misaligned16(a->out_f32)))
        return DVATTN_ERR_INVALID_ARGUMENT;
    std::vector<FragDesc> fd((size_t)a->F);
    for (int f = 0; f < a->F; ++f)
        fd[f] = FragDesc{a->key_fragments[f], a->value_fragments[f], a->fragment_rows[f], a->fragment_batch[f] == 1 ? 0 : 1};
    PagedParams p{};
    p.F = a->F; p.W = a->W; p.Hq = a->Hq; p.Hkv = a->Hkv; p.E = a->E; p.S = a->S; p.R = 0;
    p.BS = 1; p.maxb = 0; p.WS = WS; p.gqa = a->Hq / a->Hkv;
    p.cap = 0x7fffffff;
    p.NB = 0;
    p.scale_log2 = a->scale * kLog2e;
    p.out = a->out; p.q = a->queries; p.cos = nullptr; p.sin = nullptr; p.loc = a->locations;
    p.L = a->fragment_lengths; p.k = nullptr; p.v = nullptr; p.bt = nullptr;
    p.lse_out = a->lse_out; p.out_f32 = a->out_f32;
    p.cu_q = nullptr; p.nseq = 0; p.cs_stride = 0;
    p.nfrag = a->F;
    p.q_turn_stride = (long long)a->W * a->Hq * a->S * a->E;
    p.frag = fd.data();  // staged into the workspace by run_schedule
    return run_schedule(p, a->dtype, workspace, wbytes, stream, DVATTN_PHASE_ALL);
}

}  // namespace dvb
