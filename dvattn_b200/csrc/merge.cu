// Log-sum-exp merge of partial attention results over disjoint key sets, used to
// combine per-GPU partials of a KV-sharded long-context decode.  Same arithmetic as the
// split-KV reduce of the reference (src/kernels/paged_kernel_v21.cuh:307-374): weights
// exp(lse_i - max lse), empty parts (lse = -inf) skipped, rows with no part -> zeros.
// One warp per row; lane j owns columns 4j + 128k .. +3.
#include "decode.cuh"

namespace dvb {

// Part i of the outputs starts at po + i * so, of the LSEs at pl + i * sl (floats).
template <class T>
__global__ void __launch_bounds__(256) lse_merge_kernel(int parts, long long rows, int Ev, const float* po,
                                                        const float* pl, long long so, long long sl, T* out,
                                                        float* lse_out) {
    const long long row = blockIdx.x * 8ll + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    float mx = neg_inf();
    for (int i = 0; i < parts; ++i) mx = fmaxf(mx, pl[(long long)i * sl + row]);
    float den = 0.f;
    for (int i = 0; i < parts; ++i) {
        const float l = pl[(long long)i * sl + row];
        if (l != neg_inf()) den += fast_exp2((l - mx) * kLog2e);
    }
    const float inv = den > 0.f ? 1.f / den : 0.f;
    for (int e = 4 * lane; e < Ev; e += 128) {
        float a[4] = {0.f, 0.f, 0.f, 0.f};
        for (int i = 0; i < parts; ++i) {
            const float l = pl[(long long)i * sl + row];
            if (l == neg_inf()) continue;
            const float wgt = fast_exp2((l - mx) * kLog2e) * inv;
            const float* src = po + (long long)i * so + row * Ev + e;
            for (int j = 0; j < 4 && e + j < Ev; ++j) a[j] += wgt * src[j];
        }
        for (int j = 0; j < 4 && e + j < Ev; ++j) out[row * Ev + e + j] = Elem<T>::from_f(a[j]);
    }
    if (lse_out && lane == 0) lse_out[row] = den > 0.f ? mx + __logf(den) : neg_inf();
}

static int lse_merge_strided(int dtype, int parts, long long rows, int Ev, const float* po, const float* pl,
                             long long so, long long sl, void* out, float* lse_out, cudaStream_t stream) {
    if (parts < 0 || rows < 0 || Ev <= 0) return DVATTN_ERR_INVALID_ARGUMENT;
    if (rows == 0) return DVATTN_OK;
    if (!out || (parts > 0 && (!po || !pl))) return DVATTN_ERR_INVALID_ARGUMENT;
    const unsigned g = (unsigned)((rows + 7) / 8);
    switch (dtype) {
        case DVATTN_FLOAT32:
            lse_merge_kernel<float><<<g, 256, 0, stream>>>(parts, rows, Ev, po, pl, so, sl, (float*)out, lse_out);
            break;
        case DVATTN_FLOAT16:
            lse_merge_kernel<__half><<<g, 256, 0, stream>>>(parts, rows, Ev, po, pl, so, sl, (__half*)out, lse_out);
            break;
        case DVATTN_BFLOAT16:
            lse_merge_kernel<__nv_bfloat16><<<g, 256, 0, stream>>>(parts, rows, Ev, po, pl, so, sl, (__nv_bfloat16*)out,
                                                                   lse_out);
            break;
        default: return DVATTN_ERR_UNSUPPORTED;
    }
    return cudaGetLastError() == cudaSuccess ? DVATTN_OK : DVATTN_ERR_CUDA;
}

int lse_merge_launch(int dtype, int parts, long long rows, int Ev, const float* po, const float* pl, void* out,
                     float* lse_out, cudaStream_t stream) {
    return lse_merge_strided(dtype, parts, rows, Ev, po, pl, rows * (long long)Ev, rows, out, lse_out, stream);
}

// Packed parts: part i = packed + i * rows * (Ev + 1) holds [rows][Ev] outputs, then [rows] LSEs.
int lse_merge_packed_launch(int dtype, int parts, long long rows, int Ev, const float* packed, void* out,
                            float* lse_out, cudaStream_t stream) {
    const long long stride = rows * ((long long)Ev + 1);
    return lse_merge_strided(dtype, parts, rows, Ev, packed, packed ? packed + rows * (long long)Ev : nullptr, stride,
                             stride, out, lse_out, stream);
}

}  // namespace dvb
