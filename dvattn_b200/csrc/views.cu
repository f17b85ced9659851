// Device-side turn/view metadata (the bookkeeping before the attention path).
//
// Reference behaviour replaced: DVAttnCache.update at layer 0 (python/dvattn/attention.py:
// 161-191) walks every worker's list of cache segments on the host: for worker w and the
// segment at list index k, the new tokens' location in that segment is
//     loc = (sum of the lengths of the segments at index >= k in w's list) - n + i,
// i = 0..n-1 (arange(pos - n, pos) after pos += length, iterating the list backwards);
// then the model's rotary embedding turns the locations into cos/sin
// (attention.py:185: cos(loc * inv_freq), inv_freq_j = base^(-2j/R), both halves equal,
// times attention_scaling, returned in the model dtype and widened to f32), followed by a
// torch._dynamo.graph_break.  Here one kernel writes locations [F, W, n] and cos/sin
// [F, W, n, R] from the segment lengths and each worker's segment order.
#include "decode.cuh"

namespace dvb {


__device__ __forceinline__ int view_location(const dvattn_views_args& a, long long row) {
    const int i = (int)(row % a.n);
    const long long fw = row / a.n;
    const int w = (int)(fw % a.W), f = (int)(fw / a.W);
    const int k = __ldg(a.seg_order + (size_t)w * a.F + f);
    long long suffix = 0;  // lengths of the segments from index k to the end of w's list
    for (int g = 0; g < a.F; ++g)
        if (__ldg(a.seg_order + (size_t)w * a.F + g) >= k) suffix += __ldg(a.seg_lengths + g);
    return (int)(suffix - a.n + i);
}

__device__ __forceinline__ void view_cs(const dvattn_views_args& a, int j, float pos, float& c, float& s) {
    rotary_cos_sin(a.inv_freq, a.rope_base, a.R, j, pos, a.attention_scaling, a.round_dtype, c, s);
}

// General form: a thread per (segment, worker, token) row.
__global__ void __launch_bounds__(256) build_views_kernel(dvattn_views_args a) {
    const long long tot = (long long)a.F * a.W * a.n;
    const int hr = a.R >> 1;
    for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < tot;
         idx += (long long)gridDim.x * blockDim.x) {
        const int loc = view_location(a, idx);
        a.locations[idx] = loc;
        if (hr == 0) continue;
        float* cr = a.cosines + idx * a.R;
        float* sr = a.sines + idx * a.R;
        for (int j = 0; j < hr; ++j) {
            float c, s;
            view_cs(a, j, (float)loc, c, s);
            cr[j] = cr[j + hr] = c;
            sr[j] = sr[j + hr] = s;
        }
    }
}

// Coalesced form (R/2 a multiple of 4): a thread per 4 rotary pairs of a row, so a warp's
// 16-byte stores cover consecutive parts of consecutive rows.
__global__ void __launch_bounds__(256) build_views_vec_kernel(dvattn_views_args a) {
    const int hr = a.R >> 1, q4 = hr >> 2;  // 4-pair chunks per row
    const long long tot = (long long)a.F * a.W * a.n * q4;
    for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < tot; t += (long long)gridDim.x * blockDim.x) {
        const long long row = t / q4;
        const int j0 = (int)(t - row * q4) * 4;
        const int loc = view_location(a, row);
        if (j0 == 0) a.locations[row] = loc;
        float c[4], s[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) view_cs(a, j0 + u, (float)loc, c[u], s[u]);
        float* cr = a.cosines + row * a.R + j0;
        float* sr = a.sines + row * a.R + j0;
        const float4 cv = make_float4(c[0], c[1], c[2], c[3]), sv = make_float4(s[0], s[1], s[2], s[3]);
        *reinterpret_cast<float4*>(cr) = cv;
        *reinterpret_cast<float4*>(cr + hr) = cv;
        *reinterpret_cast<float4*>(sr) = sv;
        *reinterpret_cast<float4*>(sr + hr) = sv;
    }
}

int build_views_launch(const dvattn_views_args* a, cudaStream_t stream) {
    if (!a) return DVATTN_ERR_INVALID_ARGUMENT;
    if (a->F < 0 || a->W < 0 || a->n < 0 || a->R < 0 || (a->R & 1) || a->round_dtype < 0 || a->round_dtype > 2)
        return DVATTN_ERR_INVALID_ARGUMENT;
    const long long tot = (long long)a->F * a->W * a->n;
    if (tot == 0) return DVATTN_OK;
    if (!a->seg_lengths || !a->seg_order || !a->locations || (a->R > 0 && (!a->cosines || !a->sines)))
        return DVATTN_ERR_INVALID_ARGUMENT;
    if (a->R > 0 && !(a->rope_base > 0.f)) return DVATTN_ERR_INVALID_ARGUMENT;
    const bool vec = a->R > 0 && ((a->R >> 1) & 3) == 0 &&
                     !((reinterpret_cast<uintptr_t>(a->cosines) | reinterpret_cast<uintptr_t>(a->sines)) & 15);
    const long long work = vec ? tot * ((a->R >> 1) >> 2) : tot;
    const long long want = (work + 255) / 256;
    const int grid = (int)(want < 148LL * 16 ? want : 148LL * 16);
    if (vec)
        build_views_vec_kernel<<<grid, 256, 0, stream>>>(*a);
    else
        build_views_kernel<<<grid, 256, 0, stream>>>(*a);
    return cudaGetLastError() == cudaSuccess ? DVATTN_OK : DVATTN_ERR_CUDA;
}

}  // namespace dvb
