// Attention with the query rotation tables built on the device from the locations.
//
// The reference's caller (DVAttnCache.update, python/dvattn/attention.py:161-191) computes
// each (turn, worker) view's locations on the host and then the model's rotary embedding
// of them, and passes both to the attention op as `locations` and `cosines`/`sines`.  The
// rotation of a query in turn f is the rotary embedding at its own location there.  These
// entry points take the locations and the rotary parameters instead: one small kernel
// writes the cos/sin tables into the workspace (bit-identical to dvattn_build_views,
// through the same rotary_cos_sin), then the ordinary attention path runs on them.
#include "decode.cuh"

namespace dvb {
namespace {

constexpr size_t up256(size_t x) { return (x + 255) & ~size_t(255); }

// One thread per (row, rotary pair j) of the table; row = (f, query) in the order of the
// locations.  `full`: the decode layout [.., R] with both halves written; otherwise the
// varlen layout [.., R/2].
__global__ void __launch_bounds__(256) rope_table_kernel(const int* __restrict__ loc, long long rows, int R, bool full,
                                                         dvattn_rotary_args r, float* __restrict__ cos,
                                                         float* __restrict__ sin) {
    const int hp = R >> 1, stride = full ? R : hp;
    const long long tot = rows * hp;
    for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < tot;
         idx += (long long)gridDim.x * blockDim.x) {
        const long long row = idx / hp;
        const int j = (int)(idx - row * hp);
        float c, s;
        rotary_cos_sin(r.inv_freq, r.rope_base, R, j, (float)__ldg(loc + row), r.attention_scaling, r.round_dtype, c,
                       s);
        float* cr = cos + row * stride;
        float* sr = sin + row * stride;
        cr[j] = c;
        sr[j] = s;
        if (full) {
            cr[j + hp] = c;
            sr[j + hp] = s;
        }
    }
}

int rotary_check(const dvattn_rotary_args* r, int R) {
    if (!r) return DVATTN_ERR_INVALID_ARGUMENT;
    if (R < 0 || (R & 1) || r->round_dtype < 0 || r->round_dtype > 2) return DVATTN_ERR_INVALID_ARGUMENT;
    if (R > 0 && !r->inv_freq && !(r->rope_base > 0.f)) return DVATTN_ERR_INVALID_ARGUMENT;
    return DVATTN_OK;
}

size_t table_bytes(long long rows, int R, bool full) { return up256((size_t)rows * (size_t)(full ? R : R / 2) * 4); }

int launch_tables(const int* loc, long long rows, int R, bool full, const dvattn_rotary_args* r, float* cos, float* sin,
                  cudaStream_t stream) {
    const long long work = rows * (R >> 1);
    if (work == 0) return DVATTN_OK;
    const long long want = (work + 255) / 256;
    const int grid = (int)(want < 148LL * 8 ? want : 148LL * 8);
    rope_table_kernel<<<grid, 256, 0, stream>>>(loc, rows, R, full, *r, cos, sin);
    return cudaGetLastError() == cudaSuccess ? DVATTN_OK : DVATTN_ERR_CUDA;
}

}  // namespace

size_t paged_rope_workspace_size(const dvattn_paged_args* a, const dvattn_rotary_args* r) {
    if (!a || rotary_check(r, a->R) != DVATTN_OK) return 0;
    const size_t t0 = decode_workspace_size(a);
    if (t0 == 0 || a->R == 0) return t0;
    const long long rows = (long long)a->F * a->W * a->S;
    return up256(t0) + 2 * table_bytes(rows, a->R, true);
}

int paged_rope_launch(const dvattn_paged_args* a, const dvattn_rotary_args* r, void* workspace, size_t wbytes,
                      cudaStream_t stream) {
    if (!a) return DVATTN_ERR_INVALID_ARGUMENT;
    int st = rotary_check(r, a->R);
    if (st != DVATTN_OK) return st;
    st = decode_validate(a);
    if (st != DVATTN_OK) return st;
    dvattn_paged_args b = *a;
    const size_t t0 = decode_workspace_size(a);
    const long long rows = (long long)a->F * a->W * a->S;
    if (a->R > 0 && rows > 0 && a->Hq > 0) {
        if (!a->locations) return DVATTN_ERR_INVALID_ARGUMENT;
        const size_t tb = table_bytes(rows, a->R, true);
        if (!workspace || t0 == 0 || wbytes < up256(t0) + 2 * tb) return DVATTN_ERR_WORKSPACE;
        float* cos = reinterpret_cast<float*>(static_cast<char*>(workspace) + up256(t0));
        float* sin = reinterpret_cast<float*>(static_cast<char*>(workspace) + up256(t0) + tb);
        st = launch_tables(a->locations, rows, a->R, true, r, cos, sin, stream);
        if (st != DVATTN_OK) return st;
        b.cosines = cos;
        b.sines = sin;
        wbytes = t0;
    }
    return decode_launch(&b, workspace, wbytes, stream, DVATTN_PHASE_ALL);
}

size_t varlen_rope_workspace_size(const dvattn_varlen_args* a, const dvattn_rotary_args* r) {
    if (!a || rotary_check(r, a->R) != DVATTN_OK) return 0;
    const size_t t0 = varlen_workspace_size(a);
    if (t0 == 0 || a->R == 0) return t0;
    return up256(t0) + 2 * table_bytes((long long)a->F * a->T, a->R, false);
}

int varlen_rope_attn_launch(const dvattn_varlen_args* a, const dvattn_rotary_args* r, void* workspace, size_t wbytes,
                            cudaStream_t stream) {
    if (!a) return DVATTN_ERR_INVALID_ARGUMENT;
    int st = rotary_check(r, a->R);
    if (st != DVATTN_OK) return st;
    dvattn_varlen_args b = *a;
    const size_t t0 = varlen_workspace_size(a);
    const long long rows = (long long)a->F * a->T;
    if (a->R > 0 && rows > 0 && a->Hq > 0) {
        if (!a->locations) return DVATTN_ERR_INVALID_ARGUMENT;
        const size_t tb = table_bytes(rows, a->R, false);
        if (!workspace || t0 == 0 || wbytes < up256(t0) + 2 * tb) return DVATTN_ERR_WORKSPACE;
        float* cos = reinterpret_cast<float*>(static_cast<char*>(workspace) + up256(t0));
        float* sin = reinterpret_cast<float*>(static_cast<char*>(workspace) + up256(t0) + tb);
        st = launch_tables(a->locations, rows, a->R, false, r, cos, sin, stream);
        if (st != DVATTN_OK) return st;
        b.cosines = cos;
        b.sines = sin;
        wbytes = t0;
    }
    return varlen_launch(&b, workspace, wbytes, stream, DVATTN_PHASE_ALL);
}

}  // namespace dvb
