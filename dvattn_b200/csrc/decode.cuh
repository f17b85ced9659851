// Host entry points of the paged-decode machinery (decode.cu) and the standalone
// rotation / merge kernels (rope.cu, merge.cu).  All return DVATTN_* status codes.
#pragma once

#include "common.cuh"

namespace dvb {

// The error word sits at this byte offset of every attention workspace (DecodeSched of
// the decode header, header[3] of the prefill); dvattn_workspace_status reads it.
constexpr size_t kErrorWordOffset = 12;

int decode_validate(const dvattn_paged_args* a);
size_t decode_workspace_size(const dvattn_paged_args* a);
int decode_launch(const dvattn_paged_args* a, void* workspace, size_t wbytes, cudaStream_t stream, int phase);

size_t varlen_workspace_size(const dvattn_varlen_args* a);
int varlen_launch(const dvattn_varlen_args* a, void* workspace, size_t wbytes, cudaStream_t stream, int phase);
// turn/view metadata (views.cu)
int build_views_launch(const dvattn_views_args* a, cudaStream_t stream);
// attention with the rotary tables computed on the device from the locations (rope_tables.cu)
size_t paged_rope_workspace_size(const dvattn_paged_args* a, const dvattn_rotary_args* r);
int paged_rope_launch(const dvattn_paged_args* a, const dvattn_rotary_args* r, void* workspace, size_t wbytes,
                      cudaStream_t stream);
size_t varlen_rope_workspace_size(const dvattn_varlen_args* a, const dvattn_rotary_args* r);
int varlen_rope_attn_launch(const dvattn_varlen_args* a, const dvattn_rotary_args* r, void* workspace, size_t wbytes,
                            cudaStream_t stream);
// paged KV append with fused K rotation (append.cu)
int paged_append_launch(const dvattn_append_args* a, cudaStream_t stream);
// contiguous fragments (the dvattn_sdpa op)
size_t sdpa_workspace_size(const dvattn_sdpa_args* a);
int sdpa_launch(const dvattn_sdpa_args* a, void* workspace, size_t wbytes, cudaStream_t stream);
// tcgen05 varlen prefill (prefill.cu): used by varlen_launch when prefill_eligible()
bool prefill_eligible(const dvattn_varlen_args* a);
size_t prefill_workspace_size(const dvattn_varlen_args* a);
int prefill_launch(const dvattn_varlen_args* a, void* workspace, size_t wbytes, cudaStream_t stream, int phase);

int rope_launch(int dtype, int F, int W, int Hq, int S, int E, int R, void* out, const void* q, const float* cos,
                const float* sin, cudaStream_t stream);
int varlen_rope_launch(int dtype, int F, int T, int H, int E, int R, void* out, const void* q, const float* cos,
                       const float* sin, cudaStream_t stream);
int lse_merge_launch(int dtype, int num_parts, long long rows, int Ev, const float* part_out, const float* part_lse,
                     void* out, float* lse_out, cudaStream_t stream);
// device address of the no-alloc scratch on the current device (noalloc.cu)
int noalloc_scratch(void** out);

int lse_merge_packed_launch(int dtype, int parts, long long rows, int Ev, const float* packed, void* out,
                            float* lse_out, cudaStream_t stream);

}  // namespace dvb
