// extern "C" boundary of libdvattn_b200.so (declared in include/dvattn_b200.h).
#include "decode.cuh"

extern "C" {

int dvattn_abi_version(void) { return 1; }

const char* dvattn_status_string(int status) {
    switch (status) {
        case DVATTN_OK: return "ok";
        case DVATTN_ERR_INVALID_ARGUMENT: return "invalid argument (null pointer, bad size or misaligned tensor)";
        case DVATTN_ERR_UNSUPPORTED: return "unsupported configuration (dtype, head dim, Ev != E or GQA > 16)";
        case DVATTN_ERR_WORKSPACE: return "workspace missing, too small or not 256-byte aligned";
        case DVATTN_ERR_CUDA: return "CUDA error";
        default: return "unknown status";
    }
}

size_t dvattn_paged_sdpa_workspace_size(const dvattn_paged_args* args) { return dvb::decode_workspace_size(args); }

int dvattn_workspace_status(const void* workspace, dvattn_stream_t stream, int* error_word) {
    if (!error_word) return DVATTN_ERR_INVALID_ARGUMENT;
    *error_word = 0;
    void* ws = const_cast<void*>(workspace);
    if (!ws && dvb::noalloc_scratch(&ws) != DVATTN_OK) return DVATTN_ERR_CUDA;
    if (reinterpret_cast<uintptr_t>(ws) & 255) return DVATTN_ERR_WORKSPACE;
    int word = 0;
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (cudaMemcpyAsync(&word, static_cast<const char*>(ws) + dvb::kErrorWordOffset, sizeof(int),
                        cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return DVATTN_ERR_CUDA;
    *error_word = word;
    return DVATTN_OK;
}

int dvattn_paged_sdpa(const dvattn_paged_args* args, void* workspace, size_t workspace_bytes, dvattn_stream_t stream) {
    return dvb::decode_launch(args, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream),
                              DVATTN_PHASE_ALL);
}

int dvattn_paged_sdpa_phase(const dvattn_paged_args* args, void* workspace, size_t workspace_bytes, int phase,
                            dvattn_stream_t stream) {
    return dvb::decode_launch(args, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream), phase);
}

size_t dvattn_varlen_paged_sdpa_workspace_size(const dvattn_varlen_args* args) { return dvb::varlen_workspace_size(args); }

int dvattn_varlen_paged_sdpa(const dvattn_varlen_args* args, void* workspace, size_t workspace_bytes,
                             dvattn_stream_t stream) {
    return dvb::varlen_launch(args, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream), DVATTN_PHASE_ALL);
}

size_t dvattn_paged_sdpa_rope_workspace_size(const dvattn_paged_args* args, const dvattn_rotary_args* rotary) {
    return dvb::paged_rope_workspace_size(args, rotary);
}

int dvattn_paged_sdpa_rope(const dvattn_paged_args* args, const dvattn_rotary_args* rotary, void* workspace,
                           size_t workspace_bytes, dvattn_stream_t stream) {
    return dvb::paged_rope_launch(args, rotary, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

size_t dvattn_varlen_paged_sdpa_rope_workspace_size(const dvattn_varlen_args* args, const dvattn_rotary_args* rotary) {
    return dvb::varlen_rope_workspace_size(args, rotary);
}

int dvattn_varlen_paged_sdpa_rope(const dvattn_varlen_args* args, const dvattn_rotary_args* rotary, void* workspace,
                                  size_t workspace_bytes, dvattn_stream_t stream) {
    return dvb::varlen_rope_attn_launch(args, rotary, workspace, workspace_bytes,
                                        reinterpret_cast<cudaStream_t>(stream));
}

int dvattn_build_views(const dvattn_views_args* args, dvattn_stream_t stream) {
    return dvb::build_views_launch(args, reinterpret_cast<cudaStream_t>(stream));
}

int dvattn_paged_append(const dvattn_append_args* args, dvattn_stream_t stream) {
    return dvb::paged_append_launch(args, reinterpret_cast<cudaStream_t>(stream));
}

size_t dvattn_sdpa_workspace_size(const dvattn_sdpa_args* args) { return dvb::sdpa_workspace_size(args); }

int dvattn_sdpa(const dvattn_sdpa_args* args, void* workspace, size_t workspace_bytes, dvattn_stream_t stream) {
    return dvb::sdpa_launch(args, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

int dvattn_varlen_paged_sdpa_phase(const dvattn_varlen_args* args, void* workspace, size_t workspace_bytes, int phase,
                                   dvattn_stream_t stream) {
    return dvb::varlen_launch(args, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream), phase);
}

int dvattn_rope(int dtype, int F, int W, int Hq, int S, int E, int R, void* out, const void* queries,
                const float* cosines, const float* sines, dvattn_stream_t stream) {
    return dvb::rope_launch(dtype, F, W, Hq, S, E, R, out, queries, cosines, sines, reinterpret_cast<cudaStream_t>(stream));
}

int dvattn_varlen_rope(int dtype, int F, int T, int H, int E, int R, void* out, const void* queries,
                       const float* cosines, const float* sines, dvattn_stream_t stream) {
    return dvb::varlen_rope_launch(dtype, F, T, H, E, R, out, queries, cosines, sines,
                                   reinterpret_cast<cudaStream_t>(stream));
}

int dvattn_lse_merge(int dtype, int num_parts, long long rows, int Ev, const float* part_out, const float* part_lse,
                     void* out, float* lse_out, dvattn_stream_t stream) {
    return dvb::lse_merge_launch(dtype, num_parts, rows, Ev, part_out, part_lse, out, lse_out,
                                 reinterpret_cast<cudaStream_t>(stream));
}

int dvattn_lse_merge_packed(int dtype, int num_parts, long long rows, int Ev, const float* packed, void* out,
                            float* lse_out, dvattn_stream_t stream) {
    return dvb::lse_merge_packed_launch(dtype, num_parts, rows, Ev, packed, out, lse_out,
                                        reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
