// Standalone query rotation ops (schemas dvattn_rope / dvattn_varlen_rope).  The
// attention ops never call these: they rotate q inside the attention kernel.
// Reference: rope_kernel / rope_varlen_kernel (src/rope.cuh:2-114).
//
// One thread per 2 adjacent output elements; each (row, turn) reads its q row and the
// first R/2 entries of its cos/sin row and writes the rotated row (f32 math, one
// rounding to T).
#include "decode.cuh"

namespace dvb {

template <class T> __device__ __forceinline__ float ld_f(const T* p) { return Elem<T>::to_f(*p); }

template <class T>
__device__ __forceinline__ float rot1(const T* q, const float* c, const float* s, int e, int R) {
    const int h = R >> 1;
    const float x = ld_f(q + e);
    if (e < h) return x * c[e] - ld_f(q + e + h) * s[e];
    if (e < R) return x * c[e - h] + ld_f(q + e - h) * s[e - h];
    return x;
}

// out row index o = ((f*W + w)*Hq + hq)*S + s  <-  q row ((w*Hq + hq)*S + s),
// cos row (f*W + w)*S + s with row stride R   (src/rope.cuh:2-52)
template <class T>
__global__ void rope_kernel(T* out, const T* q, const float* cs, const float* sn, int F, int W, int Hq, int S, int E,
                            int R) {
    const long long rows = (long long)F * W * Hq * S;
    const long long tot = rows * E;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < tot; i += (long long)gridDim.x * blockDim.x) {
        const long long row = i / E;
        const int e = (int)(i - row * E);
        const int s = (int)(row % S);
        long long r2 = row / S;
        const int hq = (int)(r2 % Hq);
        r2 /= Hq;
        const int w = (int)(r2 % W);
        const int f = (int)(r2 / W);
        const T* qr = q + (((long long)w * Hq + hq) * S + s) * E;
        const long long crow = ((long long)f * W + w) * S + s;
        out[i] = Elem<T>::from_f(rot1(qr, cs + crow * R, sn + crow * R, e, R));
    }
}

// out [F,T,H,E] <- q [T,H,E], cos/sin [F,T,R/2]   (src/rope.cuh:54-101)
template <class T>
__global__ void varlen_rope_kernel(T* out, const T* q, const float* cs, const float* sn, int F, int Tn, int H, int E,
                                   int R) {
    const long long tot = (long long)F * Tn * H * E;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < tot; i += (long long)gridDim.x * blockDim.x) {
        const long long row = i / E;
        const int e = (int)(i - row * E);
        const int h = (int)(row % H);
        const long long ft = row / H;
        const int t = (int)(ft % Tn);
        const T* qr = q + ((long long)t * H + h) * E;
        out[i] = Elem<T>::from_f(rot1(qr, cs + ft * (R / 2), sn + ft * (R / 2), e, R));
    }
}

static int grid_for(long long n) {
    long long b = (n + 255) / 256;
    if (b > 148 * 32) b = 148 * 32;
    return (int)(b > 0 ? b : 1);
}

int rope_launch(int dtype, int F, int W, int Hq, int S, int E, int R, void* out, const void* q, const float* cos,
                const float* sin, cudaStream_t stream) {
    if (F < 0 || W < 0 || Hq < 0 || S < 0 || E <= 0 || R < 0 || R > E || (R & 1)) return DVATTN_ERR_INVALID_ARGUMENT;
    const long long n = (long long)F * W * Hq * S * E;
    if (n == 0) return DVATTN_OK;
    if (!out || !q || (R > 0 && (!cos || !sin))) return DVATTN_ERR_INVALID_ARGUMENT;
    const int g = grid_for(n);
    switch (dtype) {
        case DVATTN_FLOAT32: rope_kernel<float><<<g, 256, 0, stream>>>((float*)out, (const float*)q, cos, sin, F, W, Hq, S, E, R); break;
        case DVATTN_FLOAT16: rope_kernel<__half><<<g, 256, 0, stream>>>((__half*)out, (const __half*)q, cos, sin, F, W, Hq, S, E, R); break;
        case DVATTN_BFLOAT16: rope_kernel<__nv_bfloat16><<<g, 256, 0, stream>>>((__nv_bfloat16*)out, (const __nv_bfloat16*)q, cos, sin, F, W, Hq, S, E, R); break;
        default: return DVATTN_ERR_UNSUPPORTED;
    }
    return cudaGetLastError() == cudaSuccess ? DVATTN_OK : DVATTN_ERR_CUDA;
}

int varlen_rope_launch(int dtype, int F, int T, int H, int E, int R, void* out, const void* q, const float* cos,
                       const float* sin, cudaStream_t stream) {
    if (F < 0 || T < 0 || H < 0 || E <= 0 || R < 0 || R > E || (R & 1)) return DVATTN_ERR_INVALID_ARGUMENT;
    const long long n = (long long)F * T * H * E;
    if (n == 0) return DVATTN_OK;
    if (!out || !q || (R > 0 && (!cos || !sin))) return DVATTN_ERR_INVALID_ARGUMENT;
    const int g = grid_for(n);
    switch (dtype) {
        case DVATTN_FLOAT32: varlen_rope_kernel<float><<<g, 256, 0, stream>>>((float*)out, (const float*)q, cos, sin, F, T, H, E, R); break;
        case DVATTN_FLOAT16: varlen_rope_kernel<__half><<<g, 256, 0, stream>>>((__half*)out, (const __half*)q, cos, sin, F, T, H, E, R); break;
        case DVATTN_BFLOAT16: varlen_rope_kernel<__nv_bfloat16><<<g, 256, 0, stream>>>((__nv_bfloat16*)out, (const __nv_bfloat16*)q, cos, sin, F, T, H, E, R); break;
        default: return DVATTN_ERR_UNSUPPORTED;
    }
    return cudaGetLastError() == cudaSuccess ? DVATTN_OK : DVATTN_ERR_CUDA;
}

}  // namespace dvb
