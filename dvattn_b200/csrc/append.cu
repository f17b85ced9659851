// Paged KV append with fused K rotation (the step before the attention path): the new
// keys of each worker are rotated and written with their values into the worker's pages.
//
// Reference behaviour replaced (PyTorch / HF cache in the reference, no CUDA op there):
//   AttentionModule.forward rotates the new keys with apply_rotary_pos_emb(key_states,
//   cos, sin) (python/dvattn/attention.py:302-304) and DVAttnCache.update appends the
//   last n_w tokens of worker w (left padding, attention.py:131-149) to the worker's
//   write cache; merge_caches re-rotates a source cache by the target's length and
//   appends it (attention.py:245-251).  Here the write cache is a range of logical
//   positions of the worker's block table, so both become one pass over the new tokens.
//
// The rotation is apply_rotary_pos_emb's: for e < R/2, o[e] = x[e]*c[e] - x[e+R/2]*s[e]
// and o[e+R/2] = x[e+R/2]*c[e+R/2] + x[e]*s[e+R/2] (full-width cos/sin rows, both
// halves read), dims e >= R copied; f32 math, one rounding to T.
//
// A warp per new token, a lane per 16-byte chunk of its K / V rows: a K chunk in the
// first rotary half also reads its partner chunk R/2 further, and vice versa.  HBM-bound.
#include "decode.cuh"

namespace dvb {

struct AppendParams {
    int W, Hkv, E, Ev, n, R, BS, maxb;
    int vec;  // 1: R/2 a multiple of the chunk width (or R = 0) and cos/sin 16-byte aligned
    long long NB;
    void* k_cache;
    void* v_cache;
    const void* keys;
    const void* values;
    const float* cos;
    const float* sin;
    const int* bt;
    const int* pos;
    const int* cnt;
};

template <class T>
__device__ __forceinline__ float rot_k(const T* x, const float* c, const float* s, int e, int R) {
    // separate roundings of the two products and the sum, as the reference's elementwise
    // (x * cos) + (rotate_half(x) * sin)
    const int h = R >> 1;
    const float v = Elem<T>::to_f(x[e]);
    if (e < h) return __fadd_rn(__fmul_rn(v, c[e]), __fmul_rn(-Elem<T>::to_f(x[e + h]), s[e]));
    if (e < R) return __fadd_rn(__fmul_rn(v, c[e]), __fmul_rn(Elem<T>::to_f(x[e - h]), s[e]));
    return v;
}

// One warp per (worker, token): the page lookup is done once per token and the lanes
// cover the token's 16-byte chunks of K (all heads) and V (all heads).
#ifndef APPEND_UNROLL
#define APPEND_UNROLL 2  // chunks a lane loads before it stores
#endif
#ifndef APPEND_MINB
#define APPEND_MINB 3  // resident 256-thread blocks per SM (85 registers: no spills at UNROLL 2)
#endif

template <class T>
__global__ void __launch_bounds__(256, APPEND_MINB) paged_append_kernel(AppendParams p) {
    constexpr int PER = 16 / sizeof(T);  // elements per 16-byte chunk
    const int ck = p.E / PER, cv = p.Ev / PER;
    const int per_tok = p.Hkv * (ck + cv);
    const int lane = threadIdx.x & 31;
    // 32-bit token / position arithmetic: the launch checks W*n and maxb*BS < 2^31
    const int ntok = p.W * p.n;
    const int nwarp = gridDim.x * (blockDim.x >> 5);
    for (int wt = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); wt < ntok; wt += nwarp) {
        const int w = wt / p.n, t = wt - w * p.n;
        const int cnt = p.cnt ? __ldg(p.cnt + w) : p.n;
        const int first = p.n - (cnt < p.n ? (cnt > 0 ? cnt : 0) : p.n);
        if (t < first) continue;  // left padding: only the last cnt tokens are new
        const long long lp64 = (long long)__ldg(p.pos + w) + (t - first);
        if (lp64 < 0 || lp64 >= (long long)p.maxb * p.BS) continue;
        const int lp = (int)lp64;
        const int pg = lp / p.BS;
        const int page = __ldg(p.bt + (size_t)w * p.maxb + pg);
        const bool page_ok = page >= 0 && page < p.NB;  // checked before any store
        const long long slot = (long long)page * p.BS + (lp - pg * p.BS);
        const size_t crow = (size_t)wt * p.R;
        if (p.vec) {
            // every chunk lies inside one rotary half (or past R): a lane issues all the
            // 16-byte loads of its APPEND_UNROLL chunks, in flight with the block-table
            // read, before any store
            const int h = p.R >> 1;
            constexpr int U = APPEND_UNROLL;
            for (int j0 = lane; j0 < per_tok; j0 += 32 * U) {
                uint4 xs[U], xp[U];
                float cs[U][PER], sn[U][PER];
                T* dst[U];
                int kind[U];  // 0: none, 1: copy, 2: rotate (low half), 3: rotate (high half)
#pragma unroll
                for (int q = 0; q < U; ++q) {
                    const int j = j0 + 32 * q;
                    kind[q] = 0;
                    if (j >= per_tok) continue;
                    const bool is_k = j < p.Hkv * ck;
                    const int jj = is_k ? j : j - p.Hkv * ck;
                    const int cpr = is_k ? ck : cv, Ed = is_k ? p.E : p.Ev;
                    const int hh = jj / cpr, c = jj - hh * cpr, e0 = c * PER;
                    const T* src = static_cast<const T*>(is_k ? p.keys : p.values) + (((size_t)w * p.Hkv + hh) * p.n + t) * Ed;
                    dst[q] = static_cast<T*>(is_k ? p.k_cache : p.v_cache) + ((size_t)slot * p.Hkv + hh) * Ed + e0;
                    xs[q] = __ldg(reinterpret_cast<const uint4*>(src + e0));
                    kind[q] = 1;
                    if (is_k && e0 < p.R) {
                        const bool lo = e0 < h;
                        kind[q] = lo ? 2 : 3;
                        xp[q] = __ldg(reinterpret_cast<const uint4*>(src + (lo ? e0 + h : e0 - h)));
#pragma unroll
                        for (int u = 0; u < PER; u += 4) {
                            *reinterpret_cast<float4*>(&cs[q][u]) = __ldg(reinterpret_cast<const float4*>(p.cos + crow + e0 + u));
                            *reinterpret_cast<float4*>(&sn[q][u]) = __ldg(reinterpret_cast<const float4*>(p.sin + crow + e0 + u));
                        }
                    }
                }
                if (!page_ok) break;
#pragma unroll
                for (int q = 0; q < U; ++q) {
                    if (kind[q] == 0) continue;
                    if (kind[q] == 1) {
                        *reinterpret_cast<uint4*>(dst[q]) = xs[q];
                        continue;
                    }
                    // the same roundings as rot_k
                    const T* xa = reinterpret_cast<const T*>(&xs[q]);
                    const T* xb = reinterpret_cast<const T*>(&xp[q]);
                    alignas(16) T o[PER];
#pragma unroll
                    for (int u = 0; u < PER; ++u) {
                        const float va = Elem<T>::to_f(xa[u]), vb = Elem<T>::to_f(xb[u]);
                        o[u] = Elem<T>::from_f(__fadd_rn(__fmul_rn(va, cs[q][u]), __fmul_rn(kind[q] == 2 ? -vb : vb, sn[q][u])));
                    }
                    *reinterpret_cast<uint4*>(dst[q]) = *reinterpret_cast<const uint4*>(o);
                }
            }
            continue;
        }
        if (!page_ok) continue;
        for (int j = lane; j < per_tok; j += 32) {
            const bool is_k = j < p.Hkv * ck;
            const int jj = is_k ? j : j - p.Hkv * ck;
            const int cpr = is_k ? ck : cv, Ed = is_k ? p.E : p.Ev;
            const int h = jj / cpr, c = jj - h * cpr;
            const size_t src_row = (((size_t)w * p.Hkv + h) * p.n + t) * Ed;
            const size_t dst_row = ((size_t)slot * p.Hkv + h) * Ed;
            if (!is_k) {
                const uint4 v = *reinterpret_cast<const uint4*>(static_cast<const T*>(p.values) + src_row + c * PER);
                *reinterpret_cast<uint4*>(static_cast<T*>(p.v_cache) + dst_row + c * PER) = v;
                continue;
            }
            const T* x = static_cast<const T*>(p.keys) + src_row;
            T* dst = static_cast<T*>(p.k_cache) + dst_row + c * PER;
            const int e0 = c * PER;
            if (e0 >= p.R) {  // pass-through chunk
                *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(x + e0);
                continue;
            }
            const float* cr = p.cos + crow;
            const float* sr = p.sin + crow;
            alignas(16) T o[PER];
#pragma unroll
            for (int u = 0; u < PER; ++u)
                o[u] = Elem<T>::from_f(e0 + u < p.R ? rot_k(x, cr, sr, e0 + u, p.R) : Elem<T>::to_f(x[e0 + u]));
            *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(o);
        }
    }
}

int paged_append_launch(const dvattn_append_args* a, cudaStream_t stream) {
    if (!a) return DVATTN_ERR_INVALID_ARGUMENT;
    if (a->dtype < 0 || a->dtype > 2) return DVATTN_ERR_UNSUPPORTED;
    if (a->W < 0 || a->n < 0 || a->Hkv <= 0 || a->E <= 0 || a->Ev <= 0 || a->R < 0 || a->R > a->E || (a->R & 1) ||
        a->block_size <= 0 || a->max_blocks_per_seq < 0 || a->num_blocks < 0)
        return DVATTN_ERR_INVALID_ARGUMENT;
    const int esz = a->dtype == DVATTN_FLOAT32 ? 4 : 2;
    if ((a->E * esz) % 16 || (a->Ev * esz) % 16) return DVATTN_ERR_UNSUPPORTED;
    if ((long long)a->W * a->n == 0) return DVATTN_OK;
    if ((long long)a->W * a->n >= (1LL << 31) || (long long)a->max_blocks_per_seq * a->block_size >= (1LL << 31))
        return DVATTN_ERR_UNSUPPORTED;
    if (!a->k_cache || !a->v_cache || !a->keys || !a->values || !a->block_tables || !a->positions ||
        (a->R > 0 && (!a->cosines || !a->sines)))
        return DVATTN_ERR_INVALID_ARGUMENT;
    for (const void* q : {(const void*)a->k_cache, (const void*)a->v_cache, a->keys, a->values})
        if (reinterpret_cast<uintptr_t>(q) & 15) return DVATTN_ERR_INVALID_ARGUMENT;
    AppendParams p{};
    p.W = a->W; p.Hkv = a->Hkv; p.E = a->E; p.Ev = a->Ev; p.n = a->n; p.R = a->R;
    p.BS = a->block_size; p.maxb = a->max_blocks_per_seq; p.NB = a->num_blocks;
    p.k_cache = a->k_cache; p.v_cache = a->v_cache; p.keys = a->keys; p.values = a->values;
    p.cos = a->cosines; p.sin = a->sines; p.bt = a->block_tables; p.pos = a->positions; p.cnt = a->counts;
    {
        const int per = 16 / esz;
        p.vec = ((a->R >> 1) % per) == 0 && !(reinterpret_cast<uintptr_t>(a->cosines) & 15) &&
                !(reinterpret_cast<uintptr_t>(a->sines) & 15);
    }
    int sms = 148;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long want = ((long long)a->W * a->n + 7) / 8;  // 8 warps (tokens) per block
    const long long cap = (long long)sms * APPEND_MINB;  // one wave of resident blocks
    const int grid = (int)(want < cap ? want : cap);
    switch (a->dtype) {
        case DVATTN_FLOAT16: paged_append_kernel<__half><<<grid, 256, 0, stream>>>(p); break;
        case DVATTN_BFLOAT16: paged_append_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(p); break;
        default: paged_append_kernel<float><<<grid, 256, 0, stream>>>(p); break;
    }
    return cudaGetLastError() == cudaSuccess ? DVATTN_OK : DVATTN_ERR_CUDA;
}

}  // namespace dvb
