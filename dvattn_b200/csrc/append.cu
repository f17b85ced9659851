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
template <class T>
__global__ void __launch_bounds__(256) paged_append_kernel(AppendParams p) {
    constexpr int PER = 16 / sizeof(T);  // elements per 16-byte chunk
    const int ck = p.E / PER, cv = p.Ev / PER;
    const int per_tok = p.Hkv * (ck + cv);
    const int lane = threadIdx.x & 31;
    const long long ntok = (long long)p.W * p.n;
    const long long nwarp = (long long)gridDim.x * (blockDim.x >> 5);
    for (long long wt = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5); wt < ntok; wt += nwarp) {
        const int w = (int)(wt / p.n), t = (int)(wt - (long long)w * p.n);
        const int cnt = p.cnt ? __ldg(p.cnt + w) : p.n;
        const int first = p.n - (cnt < p.n ? (cnt > 0 ? cnt : 0) : p.n);
        if (t < first) continue;  // left padding: only the last cnt tokens are new
        const long long lp = (long long)__ldg(p.pos + w) + (t - first);
        if (lp < 0 || lp >= (long long)p.maxb * p.BS) continue;
        const int page = __ldg(p.bt + (size_t)w * p.maxb + lp / p.BS);
        if (page < 0 || page >= p.NB) continue;
        const long long slot = (long long)page * p.BS + lp % p.BS;
        const size_t crow = ((size_t)w * p.n + t) * p.R;
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
    int sms = 148;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long want = ((long long)a->W * a->n + 7) / 8;  // 8 warps (tokens) per block
    const int grid = (int)(want < (long long)sms * 8 ? want : (long long)sms * 8);
    switch (a->dtype) {
        case DVATTN_FLOAT16: paged_append_kernel<__half><<<grid, 256, 0, stream>>>(p); break;
        case DVATTN_BFLOAT16: paged_append_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(p); break;
        default: paged_append_kernel<float><<<grid, 256, 0, stream>>>(p); break;
    }
    return cudaGetLastError() == cudaSuccess ? DVATTN_OK : DVATTN_ERR_CUDA;
}

}  // namespace dvb
