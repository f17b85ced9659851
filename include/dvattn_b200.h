/*
 * dvattn_b200.h -- C ABI of the B200 (sm_100a) DVAttn attention forward.
 *
 * Plain pointers and sizes only: no torch or C++ types cross this boundary, so the
 * library can be bound from ctypes, cgo, JNI or a C++ engine.  Every entry point is
 * asynchronous on the given stream and returns a status code (DVATTN_OK == 0).
 *
 * Tensor layouts (all row-major, contiguous; T = the args' dtype):
 *   paged decode   queries [W,Hq,S,E] T, cosines/sines [F,W,S,R] f32 (only the first
 *                  R/2 entries of each row are read), locations [F,W,S] i32,
 *                  fragment_lengths [F] i32, k_cache [NB,BS,Hkv,E] T,
 *                  v_cache [NB,BS,Hkv,Ev] T, block_tables [W,max_blocks] i32,
 *                  out [W,Hq,S,Ev] T.
 *   varlen prefill queries [T,Hq,E] T, cosines/sines [F,T,R/2] f32, locations [F,T] i32,
 *                  cu_seqlens_q [W+1] i32, out [T,Hq,Ev] T.
 * Semantics: cache turn f occupies logical positions [sum_{f'<f} L_f', +L_f) of each
 * sequence's block table; key l of turn f is visible to a query iff l <= loc[f,.] and
 * l < L_f; the query is rotated per turn by that turn's cos/sin (NeoX rotate-half
 * pairing (e, e+R/2) for e < R/2, dims >= R pass through) and rounded to T first.
 * A query row that sees no key at all gets an output of zeros.
 */
#ifndef DVATTN_B200_H
#define DVATTN_B200_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same handle type as cudaStream_t (a CUstream_st*); NULL = legacy default stream. */
typedef struct CUstream_st* dvattn_stream_t;

/* Status codes. */
#define DVATTN_OK 0
#define DVATTN_ERR_INVALID_ARGUMENT 1 /* null pointer, negative or inconsistent size      */
#define DVATTN_ERR_UNSUPPORTED 2      /* dtype / head dim / GQA ratio outside the kernels */
#define DVATTN_ERR_WORKSPACE 3        /* workspace missing, too small or misaligned        */
#define DVATTN_ERR_CUDA 4             /* a CUDA runtime call or kernel launch failed       */

/* Element types (the dtype of queries, caches and output; cos/sin are always f32). */
#define DVATTN_FLOAT32 0
#define DVATTN_FLOAT16 1
#define DVATTN_BFLOAT16 2

/*
 * Arguments of one paged decode call.  Mirrors `Shape` (src/common.h:5-20) plus the
 * tensors of the `dvattn_paged_sdpa` schema (src/binding.cu:412-413, 151-203).
 */
typedef struct dvattn_paged_args {
    int dtype;                    /* DVATTN_FLOAT32 / FLOAT16 / BFLOAT16                 */
    int F, W, Hq, Hkv, E, Ev, S;  /* turns, sequences, heads, head dims, queries/seq     */
    int R;                        /* rotary dim = cosines.size(3); even, 0 <= R <= E     */
    int block_size;               /* tokens per page (k_cache.size(1))                  */
    int max_blocks_per_seq;       /* block_tables.size(1)                               */
    long long num_blocks;         /* k_cache.size(0); pages outside [0,NB) are not read  */
    float scale;                  /* softmax scale applied to q.k                        */
    void* out;
    const void* queries;
    const float* cosines;
    const float* sines;
    const int* locations;
    const int* fragment_lengths;
    const void* k_cache;
    const void* v_cache;
    const int* block_tables;
    float* lse_out;               /* optional [W,Hq,S] natural-log LSE of scale*q.k      */
    float* out_f32;               /* optional [W,Hq,S,Ev] f32 copy of the output        */
} dvattn_paged_args;

/*
 * Arguments of one varlen (packed, chunked-prefill) call.  Mirrors the
 * `dvattn_varlen_paged_sdpa` schema (src/binding.cu:418-420, 249-296).
 */
typedef struct dvattn_varlen_args {
    int dtype;
    int F, W, Hq, Hkv, E, Ev;     /* W = number of sequences = cu_seqlens_q.size(0)-1   */
    int T;                        /* total packed query tokens                          */
    int R;                        /* rotary dim = 2 * cosines.size(2)                   */
    int block_size;
    int max_blocks_per_seq;
    long long num_blocks;
    float scale;
    void* out;
    const void* queries;
    const float* cosines;
    const float* sines;
    const int* locations;
    const int* fragment_lengths;
    const void* k_cache;
    const void* v_cache;
    const int* block_tables;
    const int* cu_seqlens_q;      /* [W+1] packed query offsets                          */
    const int* cu_seqlens_k;      /* [W+1] accepted, unused (as in the reference)        */
    float* lse_out;               /* optional [T,Hq] natural-log LSE                     */
    float* out_f32;               /* optional [T,Hq,Ev] f32 copy of the output          */
} dvattn_varlen_args;

/*
 * Arguments of one contiguous-fragment call, the `dvattn_sdpa` schema
 * (src/binding.cu:79-149, 410-411): already rotated per-turn queries and one K and one V
 * tensor per turn ("fragment"), each [B_f, Hkv, rows_f, E] with B_f = 1 (shared by all W
 * workers) or W.  Key l of turn f is visible to (w, s) iff l <= locations[f,w,s],
 * l < fragment_lengths[f] and l < rows_f.
 */
typedef struct dvattn_sdpa_args {
    int dtype;
    int F, W, Hq, Hkv, E, Ev, S;
    float scale;
    void* out;                          /* [W,Hq,S,Ev] T                                   */
    const void* queries;                /* [F,W,Hq,S,E] T, rotated                         */
    const int* locations;               /* [F,W,S] i32 (device)                            */
    const int* fragment_lengths;        /* [F] i32 (device)                                */
    const void* const* key_fragments;   /* host array of F device pointers                 */
    const void* const* value_fragments; /* host array of F device pointers                 */
    const int* fragment_rows;           /* host array [F]: rows_f                          */
    const int* fragment_batch;          /* host array [F]: B_f (1 or W)                    */
    float* lse_out;                     /* optional [W,Hq,S] natural-log LSE               */
    float* out_f32;                     /* optional [W,Hq,S,Ev] f32 copy of the output     */
} dvattn_sdpa_args;

/*
 * Arguments of one paged KV append with fused K rotation (the step before the attention
 * path): the new tokens of worker w, keys rotated like apply_rotary_pos_emb, are written
 * at logical positions positions[w], positions[w]+1, ... of its block table.
 */
typedef struct dvattn_append_args {
    int dtype;
    int W, Hkv, E, Ev;
    int n;                        /* new tokens per worker in keys/values (with padding) */
    int R;                        /* rotary dim = cosines.size(2); 0: keys not rotated   */
    int block_size;
    int max_blocks_per_seq;
    long long num_blocks;
    void* k_cache;                /* [NB,BS,Hkv,E] T, written                            */
    void* v_cache;                /* [NB,BS,Hkv,Ev] T, written                           */
    const void* keys;             /* [W,Hkv,n,E] T, unrotated                            */
    const void* values;           /* [W,Hkv,n,Ev] T                                      */
    const float* cosines;         /* [W,n,R] f32, full width (both halves read)          */
    const float* sines;           /* [W,n,R] f32                                         */
    const int* block_tables;      /* [W,max_blocks] i32                                  */
    const int* positions;         /* [W] i32: logical position of worker w's first new token */
    const int* counts;            /* [W] i32 or null: only the last counts[w] of the n tokens
                                     are new (left padding); null = all n               */
} dvattn_append_args;

/*
 * Arguments of the turn/view metadata builder: for F cache segments shared by W workers
 * (each worker lists the segments in its own order) and n new tokens per worker.
 */
typedef struct dvattn_views_args {
    int F, W, n;
    int R;                        /* rotary dim of the cos/sin rows; 0: locations only    */
    float rope_base;              /* theta of the model's rotary embedding                */
    float attention_scaling;      /* factor on cos/sin (1 for the default rotary)         */
    int round_dtype;              /* DVATTN_*: cos/sin rounded through the model dtype    */
    const int* seg_lengths;       /* [F] i32: length of each segment                      */
    const int* seg_order;         /* [W,F] i32: index of segment f in worker w's list     */
    const float* inv_freq;        /* [R/2] f32 or null: the model's inverse frequencies
                                     (null: 1 / rope_base^(2j/R) computed on the device) */
    int* locations;               /* out [F,W,n] i32                                      */
    float* cosines;               /* out [F,W,n,R] f32 (both halves equal)                */
    float* sines;                 /* out [F,W,n,R] f32                                    */
} dvattn_views_args;

/*
 * The model's rotary embedding, for the attention entry points that compute the query
 * rotation tables on the device from the locations instead of taking cosines/sines.
 */
typedef struct dvattn_rotary_args {
    float rope_base;              /* theta                                                */
    float attention_scaling;      /* factor on cos/sin (1 for the default rotary)         */
    int round_dtype;              /* DVATTN_*: cos/sin rounded through the model dtype    */
    const float* inv_freq;        /* [R/2] f32 or null (1 / rope_base^(2j/R) on device)  */
} dvattn_rotary_args;

/* ABI version of this header (bumped on any layout change of the structs above). */
int dvattn_abi_version(void);

/* Human-readable name of a status code. */
const char* dvattn_status_string(int status);

/*
 * Bytes of device workspace `dvattn_paged_sdpa` needs for these arguments on the
 * current device (split-KV partials, per-sequence prefix sums).  Replaces the
 * function-static workspace of paged_v21::dvattn_paged_attention_gpu
 * (src/kernels/paged_kernel_v21.cuh:397-408).  Returns 0 when the arguments are invalid.
 */
size_t dvattn_paged_sdpa_workspace_size(const dvattn_paged_args* args);

/*
 * Paged decode: rotate q per turn (fused), attend over the paged cache, merge split-KV
 * partials.  Replaces dvattn_paged_attention_tpl + rope_gpu + paged_v21::
 * dvattn_paged_attention_gpu (src/binding.cu:151-203, src/rope.cuh:2-65,
 * src/kernels/paged_kernel_v21.cuh:377-431).  `workspace` is caller-owned device
 * memory of at least dvattn_paged_sdpa_workspace_size() bytes, 256-byte aligned; it
 * need not be zeroed.  Calls on the same workspace must be stream-ordered.
 */
int dvattn_paged_sdpa(const dvattn_paged_args* args, void* workspace, size_t workspace_bytes,
                      dvattn_stream_t stream);

/* Phases of dvattn_paged_sdpa (all three run on one stream, in this order). */
#define DVATTN_PHASE_ALL 0
#define DVATTN_PHASE_SCHEDULE 1 /* visible-key prefix sums and the per-CTA work split   */
#define DVATTN_PHASE_ATTEND 2   /* the split-KV attention kernel (the HBM stream)       */
#define DVATTN_PHASE_MERGE 3    /* log-sum-exp merge of segments split across CTAs      */

/*
 * One phase of dvattn_paged_sdpa on the same arguments and workspace; running SCHEDULE,
 * ATTEND, MERGE in order is exactly dvattn_paged_sdpa (PHASE_ALL).  Lets a caller put
 * events or other work between the phases (e.g. timing the attention kernel alone).
 * No reference counterpart: the reference launches its kernels back to back inside
 * paged_v21::dvattn_paged_attention_gpu (src/kernels/paged_kernel_v21.cuh:408-425).
 */
int dvattn_paged_sdpa_phase(const dvattn_paged_args* args, void* workspace, size_t workspace_bytes, int phase,
                            dvattn_stream_t stream);

/*
 * dvattn_paged_sdpa without a caller-supplied workspace, for callers that cannot allocate
 * device memory (an engine whose pool owns all of the GPU's memory and forbids
 * cudaMalloc after start-up, or a plain C host with no device allocator).  No
 * counterpart in the reference.  The split-KV scratch is one fixed array of
 * dvattn_paged_sdpa_noalloc_max_workspace() bytes (32 MiB) inside the library, held on
 * every GPU that loads it until the process exits; this entry point calls no
 * cudaMalloc/cudaFree.  Problems whose dvattn_paged_sdpa_workspace_size() exceeds that
 * return DVATTN_ERR_WORKSPACE.  The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress); make that first call before any stream capture.  All
 * calls on one device share the array, so calls that may overlap on the GPU (different
 * streams without ordering) race: serialise them.
 */
size_t dvattn_paged_sdpa_noalloc_max_workspace(void);
int dvattn_paged_sdpa_noalloc(const dvattn_paged_args* args, dvattn_stream_t stream);

/*
 * Error word of the last attention call that used `workspace` (dvattn_paged_sdpa,
 * dvattn_varlen_paged_sdpa, dvattn_sdpa and their *_rope / *_phase forms), or, with
 * workspace == NULL, of the last dvattn_paged_sdpa_noalloc call on the current device.
 * Waits for `stream` (call it after the attention call, before the next call on the same
 * workspace).  *error_word == 0: the call completed.  Nonzero: a bounded wait inside a
 * kernel gave up (~2 s; bit 1 loader, bit 2 / 8 compute warps, bit 4 bad shared-memory
 * alignment) and that call's outputs are invalid; the paged decode writes NaN to all of
 * them, the tensor-core prefill to the rows of the items that gave up.  The reference
 * reports kernel failures as a RuntimeError from C10_CUDA_CHECK (src/binding.cu:200,
 * src/cuda_check.cuh:16-29); its kernels have no waits that can give up.
 */
int dvattn_workspace_status(const void* workspace, dvattn_stream_t stream, int* error_word);

/* Workspace bytes of dvattn_varlen_paged_sdpa (see dvattn_paged_sdpa_workspace_size). */
size_t dvattn_varlen_paged_sdpa_workspace_size(const dvattn_varlen_args* args);

/*
 * Varlen chunked prefill over the paged cache.  Replaces dvattn_varlen_paged_attention_tpl
 * + rope_varlen_gpu + varlen_paged_v21::dvattn_varlen_paged_attention_gpu
 * (src/binding.cu:249-296, src/rope.cuh:67-114, src/kernels/varlen_paged_kernel_v21.cuh:373-428).
 * A turn whose location is negative for a token is skipped for that token.
 */
int dvattn_varlen_paged_sdpa(const dvattn_varlen_args* args, void* workspace,
                             size_t workspace_bytes, dvattn_stream_t stream);

/*
 * One phase of dvattn_varlen_paged_sdpa (see dvattn_paged_sdpa_phase).  On the tensor-core
 * prefill path SCHEDULE builds the work list, ATTEND runs the attention kernel and MERGE
 * has nothing to do.
 */
int dvattn_varlen_paged_sdpa_phase(const dvattn_varlen_args* args, void* workspace,
                                   size_t workspace_bytes, int phase, dvattn_stream_t stream);

/* Workspace bytes of dvattn_sdpa (0 on invalid arguments). */
size_t dvattn_sdpa_workspace_size(const dvattn_sdpa_args* args);

/*
 * Attention over contiguous per-turn K/V fragments: the `dvattn_sdpa` op
 * (`dvattn_attention_tpl` + `v21::dvattn_attention_gpu`, src/binding.cu:79-149,
 * src/kernels/kernel_v21.cuh:17-431).  The fragment descriptors are copied to the
 * workspace with one host-to-device copy on `stream`.  `dvattn_fused`
 * (src/binding.cu:356-372) is dvattn_rope into the rotated-query buffer followed by this.
 */
int dvattn_sdpa(const dvattn_sdpa_args* args, void* workspace, size_t workspace_bytes, dvattn_stream_t stream);

/*
 * Paged KV append with fused K rotation.  Replaces the reference's PyTorch cache update
 * (apply_rotary_pos_emb on the new keys + DynamicCache append, python/dvattn/attention.py:
 * 131-149, 302-304; the re-rotation of merge_caches, :245-251, is the same call with the
 * cos/sin of the target offset).  Positions outside the block table and pages outside
 * [0, num_blocks) are skipped.
 */
int dvattn_paged_append(const dvattn_append_args* args, dvattn_stream_t stream);

/*
 * Turn/view metadata on the GPU: replaces the host loops of DVAttnCache.update
 * (python/dvattn/attention.py:161-191: per-(segment, worker) locations, then the model's
 * rotary embedding of them).  Writes the locations, cosines and sines the attention ops take.
 */
int dvattn_build_views(const dvattn_views_args* args, dvattn_stream_t stream);

/*
 * dvattn_paged_sdpa / dvattn_varlen_paged_sdpa with the query rotation tables computed on
 * the device: the rotation of turn f for query (w, s) (token t) is the model's rotary
 * embedding at its location loc[f, w, s] (loc[f, t]), as DVAttnCache.update builds the
 * cos/sin it passes (python/dvattn/attention.py:161-191).  args->cosines / sines are
 * ignored; args->R is the rotary dim.  The tables live in the workspace (one small
 * kernel before the attention).
 */
size_t dvattn_paged_sdpa_rope_workspace_size(const dvattn_paged_args* args, const dvattn_rotary_args* rotary);
int dvattn_paged_sdpa_rope(const dvattn_paged_args* args, const dvattn_rotary_args* rotary, void* workspace,
                           size_t workspace_bytes, dvattn_stream_t stream);
size_t dvattn_varlen_paged_sdpa_rope_workspace_size(const dvattn_varlen_args* args, const dvattn_rotary_args* rotary);
int dvattn_varlen_paged_sdpa_rope(const dvattn_varlen_args* args, const dvattn_rotary_args* rotary, void* workspace,
                                  size_t workspace_bytes, dvattn_stream_t stream);

/*
 * Standalone query rotation, schema `dvattn_rope` (src/binding.cu:41-77, src/rope.cuh:2-65):
 * out [F,W,Hq,S,E] T = rotate(queries [W,Hq,S,E] T, cos/sin [F,W,S,R] f32).
 */
int dvattn_rope(int dtype, int F, int W, int Hq, int S, int E, int R, void* out,
                const void* queries, const float* cosines, const float* sines,
                dvattn_stream_t stream);

/*
 * Standalone varlen query rotation, schema `dvattn_varlen_rope` (src/binding.cu:205-247,
 * src/rope.cuh:67-114): out [F,T,H,E] T from queries [T,H,E] and cos/sin [F,T,R/2] f32.
 */
int dvattn_varlen_rope(int dtype, int F, int T, int H, int E, int R, void* out,
                       const void* queries, const float* cosines, const float* sines,
                       dvattn_stream_t stream);

/*
 * Log-sum-exp merge of `num_parts` partial attention results over disjoint key sets
 * (the split-KV reduce of src/kernels/paged_kernel_v21.cuh:307-374, exposed so that
 * partials gathered from several GPUs can be merged):
 *   part_out [num_parts][rows][Ev] f32 (each normalised), part_lse [num_parts][rows]
 *   natural-log LSE (-inf = empty part)  ->  out [rows][Ev] T, optional lse_out [rows].
 * Rows whose parts are all empty get zeros.
 */
int dvattn_lse_merge(int dtype, int num_parts, long long rows, int Ev, const float* part_out,
                     const float* part_lse, void* out, float* lse_out, dvattn_stream_t stream);

/*
 * dvattn_lse_merge over packed parts, as one collective gathers them: part i starts at
 * packed + i * rows * (Ev + 1) floats and holds its [rows][Ev] outputs followed by its
 * [rows] LSEs.  Lets each rank of a KV-sharded call exchange outputs and LSEs in a single
 * all-gather (no reference counterpart: the reference runs on one GPU).
 */
int dvattn_lse_merge_packed(int dtype, int num_parts, long long rows, int Ev, const float* packed,
                            void* out, float* lse_out, dvattn_stream_t stream);

/*
 * KV-sharded partials exchanged over peer memory (NVLink) instead of a collective: one
 * kernel per rank signals that its partial is complete, waits (bounded, ~2 s) for every
 * rank's signal, and merges all ranks' partials read straight from their memory.  No
 * reference counterpart (the reference runs on one GPU); the merge arithmetic is its
 * split-KV reduce (src/kernels/paged_kernel_v21.cuh:347-363).
 *
 * Each rank allocates one exchange region of dvattn_peer_region_bytes(rows, Ev)
 * (dvattn_peer_region_alloc: cudaMalloc, zeroed, plus its 64-byte CUDA IPC handle), sends
 * the handle to the other ranks, and maps theirs (dvattn_peer_region_open).  A region has
 * two slots; slot s holds a rank's packed partial at dvattn_peer_slot_offset(rows, Ev, s):
 * [rows][Ev] f32 outputs, then [rows] f32 natural-log LSEs (pass them as the attention
 * call's out_f32 / lse_out).  Consecutive calls must alternate slots.
 * dvattn_lse_merge_peers(dtype, world, rank, slot, rows, Ev, regions, out, lse_out,
 * stream): regions[j] = rank j's region as mapped on this rank (regions[rank] = own);
 * out [rows][Ev] T, optional lse_out [rows].  All ranks make the same sequence of calls.
 * A wait that runs out sets the error word (dvattn_workspace_status(own region, ...))
 * and writes NaN to this call's outputs.  world <= 8.
 */
size_t dvattn_peer_region_bytes(long long rows, int Ev);
size_t dvattn_peer_slot_offset(long long rows, int Ev, int slot);
int dvattn_peer_region_alloc(size_t bytes, void** region, void* ipc_handle);
int dvattn_peer_region_open(const void* ipc_handle, void** region);
int dvattn_peer_region_close(void* region);
int dvattn_peer_region_free(void* region);
int dvattn_lse_merge_peers(int dtype, int world, int rank, int slot, long long rows, int Ev, void* const* regions,
                           void* out, float* lse_out, dvattn_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* DVATTN_B200_H */
