// torch.ops.libdvatt.* registration for the B200 build: the schemas of the reference
// extension (src/binding.cu:407-430), implemented on top of the C ABI in
// libdvattn_b200.so.  Shapes are read and checked here exactly as the reference reads
// them; the kernels run on the current torch stream of the output's device, and the
// split-KV workspace comes from the torch caching allocator (no process-wide statics).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <vector>

#include "../../include/dvattn_b200.h"

namespace {

int dtype_code(const at::Tensor& t) {
    switch (t.scalar_type()) {
        case at::kFloat: return DVATTN_FLOAT32;
        case at::kHalf: return DVATTN_FLOAT16;
        case at::kBFloat16: return DVATTN_BFLOAT16;
        default:
            // The reference silently does nothing for other dtypes (src/binding.cu:318-324).
            TORCH_CHECK(false, "dvattn: unsupported dtype ", t.scalar_type(), " (float32, float16 or bfloat16)");
    }
}

void check_status(int st, const char* what) {
    TORCH_CHECK(st == DVATTN_OK, "dvattn: ", what, " failed: ", dvattn_status_string(st));
}

// DVATTN_CHECK_STATUS=1: after every attention call, wait for the stream and raise if a
// bounded wait inside a kernel gave up (dvattn_workspace_status).  Off by default: the
// check synchronises the stream.
bool check_status_enabled() {
    static const bool on = [] {
        const char* e = getenv("DVATTN_CHECK_STATUS");
        return e && e[0] && e[0] != '0';
    }();
    return on;
}

void check_call_status(const at::Tensor& ws, dvattn_stream_t stream, const char* what) {
    if (!check_status_enabled()) return;
    int word = 0;
    check_status(dvattn_workspace_status(ws.data_ptr(), stream, &word), what);
    TORCH_CHECK(word == 0, "dvattn: ", what, ": a bounded wait in the kernel gave up (error word ", word,
                "); the outputs of this call are invalid");
}

void check_cuda_tensor(const at::Tensor& t, const char* name, const at::Tensor& out) {
    TORCH_CHECK(t.is_cuda(), "dvattn: ", name, " must be a CUDA tensor");
    TORCH_CHECK(t.device() == out.device(), "dvattn: ", name, " is on ", t.device(), " but output is on ", out.device());
    TORCH_CHECK(t.is_contiguous(), "dvattn: ", name, " must be contiguous");
}

using Named = std::pair<const at::Tensor*, const char*>;
void check_all(const at::Tensor& out, std::initializer_list<Named> ts) {
    for (const Named& n : ts) check_cuda_tensor(*n.first, n.second, out);
}

void check_i32(const at::Tensor& t, const char* name) {
    TORCH_CHECK(t.scalar_type() == at::kInt, "dvattn: ", name, " must be int32");
}

dvattn_stream_t cur_stream(const at::Tensor& out) {
    return reinterpret_cast<dvattn_stream_t>(at::cuda::getCurrentCUDAStream(out.device().index()).stream());
}

// ---------------------------------------------------------------------------------
// dvattn_paged_sdpa (src/binding.cu:151-203 / 312-325)
// ---------------------------------------------------------------------------------
// Rotary parameters of the *_rope ops (cos/sin tables built on the device from the
// locations); null for the ops that take cosines/sines.
struct RotaryOpt {
    int R;
    double base, scaling;
    const c10::optional<at::Tensor>* inv_freq;
};

dvattn_rotary_args rotary_args(const RotaryOpt& r, const at::Tensor& out, int round_dtype) {
    dvattn_rotary_args ra{};
    ra.rope_base = static_cast<float>(r.base);
    ra.attention_scaling = static_cast<float>(r.scaling);
    ra.round_dtype = round_dtype;
    TORCH_CHECK(r.R >= 0 && r.R % 2 == 0, "dvattn rope: rotary_dim must be even and >= 0");
    if (r.inv_freq && r.inv_freq->has_value()) {
        const at::Tensor& t = **r.inv_freq;
        check_cuda_tensor(t, "inv_freq", out);
        TORCH_CHECK(t.scalar_type() == at::kFloat && t.numel() == r.R / 2, "dvattn rope: inv_freq must be f32 [rotary_dim/2]");
        ra.inv_freq = t.const_data_ptr<float>();
    }
    return ra;
}

void paged_impl(at::Tensor& out, double scale, const at::Tensor& locations, const at::Tensor& queries,
                const at::Tensor& cosines, const at::Tensor& sines, const at::Tensor& fragment_lengths,
                const at::Tensor& k_cache, const at::Tensor& v_cache, const at::Tensor& block_tables,
                const c10::optional<at::Tensor>& lse, const c10::optional<at::Tensor>& out_f32,
                const RotaryOpt* rot = nullptr) {
    const c10::cuda::CUDAGuard guard(out.device());
    const int dt = dtype_code(out);
    TORCH_CHECK(out.dim() == 4, "dvattn_paged_sdpa: output must be [W, Hq, S, Ev]");
    TORCH_CHECK(queries.dim() == 4 && locations.dim() == 3 && (rot || (cosines.dim() == 4 && sines.dim() == 4)) &&
                    k_cache.dim() == 4 && v_cache.dim() == 4 && block_tables.dim() == 2 && fragment_lengths.dim() == 1,
                "dvattn_paged_sdpa: wrong tensor ranks");
    for (auto* pr : {&queries, &k_cache, &v_cache})
        TORCH_CHECK(pr->scalar_type() == out.scalar_type(), "dvattn_paged_sdpa: queries/k_cache/v_cache must have the output dtype");
    TORCH_CHECK(rot || (cosines.scalar_type() == at::kFloat && sines.scalar_type() == at::kFloat),
                "dvattn_paged_sdpa: cosines/sines must be float32");
    check_i32(locations, "locations");
    check_i32(fragment_lengths, "fragment_lengths");
    check_i32(block_tables, "block_tables");
    check_cuda_tensor(out, "output", out);
    check_cuda_tensor(queries, "queries", out);
    check_cuda_tensor(locations, "locations", out);
    if (!rot) {
        check_cuda_tensor(cosines, "cosines", out);
        check_cuda_tensor(sines, "sines", out);
    }
    check_cuda_tensor(fragment_lengths, "fragment_lengths", out);
    check_cuda_tensor(k_cache, "k_cache", out);
    check_cuda_tensor(v_cache, "v_cache", out);
    check_cuda_tensor(block_tables, "block_tables", out);

    const int W = out.size(0), Hq = out.size(1), S = out.size(2), Ev = out.size(3);
    const int F = locations.size(0);
    TORCH_CHECK(locations.size(1) == W && locations.size(2) == S, "dvattn_paged_sdpa: locations must be [F, W, S]");
    TORCH_CHECK(queries.size(0) == W && queries.size(1) == Hq && queries.size(2) == S,
                "dvattn_paged_sdpa: queries must be [W, Hq, S, E]");
    const int E = queries.size(3);
    const int R = rot ? rot->R : cosines.size(3);
    if (!rot) {
        TORCH_CHECK(cosines.size(0) == F && cosines.size(1) == W && cosines.size(2) == S,
                    "dvattn_paged_sdpa: cosines must be [F, W, S, R]");
        TORCH_CHECK(sines.sizes() == cosines.sizes(), "dvattn_paged_sdpa: sines must match cosines");
    }
    TORCH_CHECK(fragment_lengths.size(0) == F, "dvattn_paged_sdpa: fragment_lengths must be [F]");
    const int BS = k_cache.size(1), Hkv = k_cache.size(2);
    TORCH_CHECK(k_cache.size(3) == E, "dvattn_paged_sdpa: k_cache must be [NB, BS, Hkv, E]");
    TORCH_CHECK(v_cache.size(0) == k_cache.size(0) && v_cache.size(1) == BS && v_cache.size(2) == Hkv && v_cache.size(3) == Ev,
                "dvattn_paged_sdpa: v_cache must be [NB, BS, Hkv, Ev]");
    TORCH_CHECK(block_tables.size(0) == W, "dvattn_paged_sdpa: block_tables must be [W, max_blocks]");

    dvattn_paged_args a{};
    a.dtype = dt;
    a.F = F; a.W = W; a.Hq = Hq; a.Hkv = Hkv; a.E = E; a.Ev = Ev; a.S = S; a.R = R;
    a.block_size = BS;
    a.max_blocks_per_seq = block_tables.size(1);
    a.num_blocks = k_cache.size(0);
    a.scale = static_cast<float>(scale);
    a.out = out.data_ptr();
    a.queries = queries.const_data_ptr();
    a.cosines = rot ? nullptr : cosines.const_data_ptr<float>();
    a.sines = rot ? nullptr : sines.const_data_ptr<float>();
    a.locations = locations.const_data_ptr<int>();
    a.fragment_lengths = fragment_lengths.const_data_ptr<int>();
    a.k_cache = k_cache.const_data_ptr();
    a.v_cache = v_cache.const_data_ptr();
    a.block_tables = block_tables.const_data_ptr<int>();
    if (lse.has_value()) {
        check_cuda_tensor(*lse, "lse", out);
        TORCH_CHECK(lse->scalar_type() == at::kFloat && lse->numel() == (int64_t)W * Hq * S, "dvattn: lse must be f32 [W, Hq, S]");
        a.lse_out = lse->data_ptr<float>();
    }
    if (out_f32.has_value()) {
        check_cuda_tensor(*out_f32, "out_f32", out);
        TORCH_CHECK(out_f32->scalar_type() == at::kFloat && out_f32->numel() == out.numel(), "dvattn: out_f32 must be f32 like output");
        a.out_f32 = out_f32->data_ptr<float>();
    }
    if (rot) {
        const dvattn_rotary_args ra = rotary_args(*rot, out, dt);
        const size_t wsb = dvattn_paged_sdpa_rope_workspace_size(&a, &ra);
        TORCH_CHECK(wsb > 0, "dvattn_paged_sdpa_rope: could not size the workspace (unsupported or invalid shape)");
        at::Tensor ws = at::empty({(int64_t)wsb}, out.options().dtype(at::kByte));
        check_status(dvattn_paged_sdpa_rope(&a, &ra, ws.data_ptr(), wsb, cur_stream(out)), "dvattn_paged_sdpa_rope");
        check_call_status(ws, cur_stream(out), "dvattn_paged_sdpa_rope");
        return;
    }
    int st = dvattn_paged_sdpa(&a, nullptr, 0, cur_stream(out));  // validation only when nothing to do
    if (st == DVATTN_ERR_WORKSPACE) {
        const size_t wsb = dvattn_paged_sdpa_workspace_size(&a);
        TORCH_CHECK(wsb > 0, "dvattn_paged_sdpa: could not size the workspace");
        at::Tensor ws = at::empty({(int64_t)wsb}, out.options().dtype(at::kByte));
        st = dvattn_paged_sdpa(&a, ws.data_ptr(), wsb, cur_stream(out));
        check_status(st, "dvattn_paged_sdpa");
        check_call_status(ws, cur_stream(out), "dvattn_paged_sdpa");
    }
    check_status(st, "dvattn_paged_sdpa");
}

void dvattn_paged_sdpa_op(at::Tensor& out, double scale, const at::Tensor& locations, const at::Tensor& queries,
                          const at::Tensor& cosines, const at::Tensor& sines, const at::Tensor& fragment_lengths,
                          const at::Tensor& k_cache, const at::Tensor& v_cache, const at::Tensor& block_tables) {
    paged_impl(out, scale, locations, queries, cosines, sines, fragment_lengths, k_cache, v_cache, block_tables,
               c10::nullopt, c10::nullopt);
}

void dvattn_paged_sdpa_ex_op(at::Tensor& out, const c10::optional<at::Tensor>& lse,
                             const c10::optional<at::Tensor>& out_f32, double scale, const at::Tensor& locations,
                             const at::Tensor& queries, const at::Tensor& cosines, const at::Tensor& sines,
                             const at::Tensor& fragment_lengths, const at::Tensor& k_cache, const at::Tensor& v_cache,
                             const at::Tensor& block_tables) {
    paged_impl(out, scale, locations, queries, cosines, sines, fragment_lengths, k_cache, v_cache, block_tables, lse,
               out_f32);
}

// ---------------------------------------------------------------------------------
// dvattn_varlen_paged_sdpa (src/binding.cu:249-296 / 327-342)
// ---------------------------------------------------------------------------------
void varlen_impl(at::Tensor& out, double scale, const at::Tensor& locations, const at::Tensor& queries,
                 const at::Tensor& cosines, const at::Tensor& sines, const at::Tensor& fragment_lengths,
                 const at::Tensor& k_cache, const at::Tensor& v_cache, const at::Tensor& block_tables,
                 const at::Tensor& cu_seqlens_q, const at::Tensor& cu_seqlens_k, const c10::optional<at::Tensor>& lse,
                 const c10::optional<at::Tensor>& out_f32, const RotaryOpt* rot = nullptr) {
    const c10::cuda::CUDAGuard guard(out.device());
    const int dt = dtype_code(out);
    TORCH_CHECK(queries.dim() == 3 && out.dim() == 3 && locations.dim() == 2 && (rot || (cosines.dim() == 3 && sines.dim() == 3)) &&
                    k_cache.dim() == 4 && v_cache.dim() == 4 && block_tables.dim() == 2 && cu_seqlens_q.dim() == 1,
                "dvattn_varlen_paged_sdpa: wrong tensor ranks");
    for (auto* pr : {&queries, &k_cache, &v_cache})
        TORCH_CHECK(pr->scalar_type() == out.scalar_type(), "dvattn_varlen_paged_sdpa: queries/k_cache/v_cache must have the output dtype");
    TORCH_CHECK(rot || (cosines.scalar_type() == at::kFloat && sines.scalar_type() == at::kFloat),
                "dvattn_varlen_paged_sdpa: cosines/sines must be float32");
    check_i32(locations, "locations");
    check_i32(fragment_lengths, "fragment_lengths");
    check_i32(block_tables, "block_tables");
    check_i32(cu_seqlens_q, "cu_seqlens_q");
    if (!rot) check_all(out, {Named{&cosines, "cosines"}, Named{&sines, "sines"}});
    check_all(out, {Named{&queries, "queries"}, Named{&locations, "locations"},
                    Named{&fragment_lengths, "fragment_lengths"}, Named{&k_cache, "k_cache"},
                    Named{&v_cache, "v_cache"}, Named{&block_tables, "block_tables"},
                    Named{&cu_seqlens_q, "cu_seqlens_q"}, Named{&out, "output"}});
    (void)cu_seqlens_k;  // accepted and unused, as in the reference

    const int T = queries.size(0), Hq = queries.size(1), E = queries.size(2);
    const int F = locations.size(0);
    const int W = cu_seqlens_q.size(0) - 1;
    const int Ev = v_cache.size(3);
    TORCH_CHECK(W >= 0, "dvattn_varlen_paged_sdpa: cu_seqlens_q must have W+1 entries");
    TORCH_CHECK(locations.size(1) == T, "dvattn_varlen_paged_sdpa: locations must be [F, T]");
    if (!rot) {
        TORCH_CHECK(cosines.size(0) == F && cosines.size(1) == T, "dvattn_varlen_paged_sdpa: cosines must be [F, T, R/2]");
        TORCH_CHECK(sines.sizes() == cosines.sizes(), "dvattn_varlen_paged_sdpa: sines must match cosines");
    }
    TORCH_CHECK(fragment_lengths.size(0) == F, "dvattn_varlen_paged_sdpa: fragment_lengths must be [F]");
    TORCH_CHECK(out.size(0) == T && out.size(1) == Hq && out.size(2) == Ev, "dvattn_varlen_paged_sdpa: output must be [T, Hq, Ev]");
    TORCH_CHECK(k_cache.size(3) == E, "dvattn_varlen_paged_sdpa: k_cache must be [NB, BS, Hkv, E]");
    TORCH_CHECK(v_cache.size(0) == k_cache.size(0) && v_cache.size(1) == k_cache.size(1) && v_cache.size(2) == k_cache.size(2),
                "dvattn_varlen_paged_sdpa: v_cache must match k_cache");

    dvattn_varlen_args a{};
    a.dtype = dt;
    a.F = F; a.W = W; a.Hq = Hq; a.Hkv = k_cache.size(2); a.E = E; a.Ev = Ev; a.T = T;
    a.R = rot ? rot->R : cosines.size(2) * 2;
    a.block_size = k_cache.size(1);
    a.max_blocks_per_seq = block_tables.size(1);
    a.num_blocks = k_cache.size(0);
    a.scale = static_cast<float>(scale);
    a.out = out.data_ptr();
    a.queries = queries.const_data_ptr();
    a.cosines = rot ? nullptr : cosines.const_data_ptr<float>();
    a.sines = rot ? nullptr : sines.const_data_ptr<float>();
    a.locations = locations.const_data_ptr<int>();
    a.fragment_lengths = fragment_lengths.const_data_ptr<int>();
    a.k_cache = k_cache.const_data_ptr();
    a.v_cache = v_cache.const_data_ptr();
    a.block_tables = block_tables.const_data_ptr<int>();
    a.cu_seqlens_q = cu_seqlens_q.const_data_ptr<int>();
    a.cu_seqlens_k = nullptr;
    if (lse.has_value()) {
        check_cuda_tensor(*lse, "lse", out);
        TORCH_CHECK(lse->scalar_type() == at::kFloat && lse->numel() == (int64_t)T * Hq, "dvattn: lse must be f32 [T, Hq]");
        a.lse_out = lse->data_ptr<float>();
    }
    if (out_f32.has_value()) {
        check_cuda_tensor(*out_f32, "out_f32", out);
        TORCH_CHECK(out_f32->scalar_type() == at::kFloat && out_f32->numel() == out.numel(), "dvattn: out_f32 must be f32 like output");
        a.out_f32 = out_f32->data_ptr<float>();
    }
    if (rot) {
        const dvattn_rotary_args ra = rotary_args(*rot, out, dt);
        const size_t wsb = dvattn_varlen_paged_sdpa_rope_workspace_size(&a, &ra);
        TORCH_CHECK(wsb > 0, "dvattn_varlen_paged_sdpa_rope: could not size the workspace (unsupported or invalid shape)");
        at::Tensor ws = at::empty({(int64_t)wsb}, out.options().dtype(at::kByte));
        check_status(dvattn_varlen_paged_sdpa_rope(&a, &ra, ws.data_ptr(), wsb, cur_stream(out)),
                     "dvattn_varlen_paged_sdpa_rope");
        check_call_status(ws, cur_stream(out), "dvattn_varlen_paged_sdpa_rope");
        return;
    }
    int st = dvattn_varlen_paged_sdpa(&a, nullptr, 0, cur_stream(out));
    if (st == DVATTN_ERR_WORKSPACE) {
        const size_t wsb = dvattn_varlen_paged_sdpa_workspace_size(&a);
        TORCH_CHECK(wsb > 0, "dvattn_varlen_paged_sdpa: could not size the workspace");
        at::Tensor ws = at::empty({(int64_t)wsb}, out.options().dtype(at::kByte));
        st = dvattn_varlen_paged_sdpa(&a, ws.data_ptr(), wsb, cur_stream(out));
        check_status(st, "dvattn_varlen_paged_sdpa");
        check_call_status(ws, cur_stream(out), "dvattn_varlen_paged_sdpa");
    }
    check_status(st, "dvattn_varlen_paged_sdpa");
}

void dvattn_varlen_paged_sdpa_op(at::Tensor& out, double scale, const at::Tensor& locations, const at::Tensor& queries,
                                 const at::Tensor& cosines, const at::Tensor& sines, const at::Tensor& fragment_lengths,
                                 const at::Tensor& k_cache, const at::Tensor& v_cache, const at::Tensor& block_tables,
                                 const at::Tensor& cu_seqlens_q, const at::Tensor& cu_seqlens_k) {
    varlen_impl(out, scale, locations, queries, cosines, sines, fragment_lengths, k_cache, v_cache, block_tables,
                cu_seqlens_q, cu_seqlens_k, c10::nullopt, c10::nullopt);
}

void dvattn_varlen_paged_sdpa_ex_op(at::Tensor& out, const c10::optional<at::Tensor>& lse,
                                    const c10::optional<at::Tensor>& out_f32, double scale,
                                    const at::Tensor& locations, const at::Tensor& queries, const at::Tensor& cosines,
                                    const at::Tensor& sines, const at::Tensor& fragment_lengths,
                                    const at::Tensor& k_cache, const at::Tensor& v_cache,
                                    const at::Tensor& block_tables, const at::Tensor& cu_seqlens_q,
                                    const at::Tensor& cu_seqlens_k) {
    varlen_impl(out, scale, locations, queries, cosines, sines, fragment_lengths, k_cache, v_cache, block_tables,
                cu_seqlens_q, cu_seqlens_k, lse, out_f32);
}

// The same two ops with the rotation tables built on the device from the locations
// (the model's rotary embedding: theta, scaling, optional inv_freq; cos/sin rounded
// through the output dtype as the model returns them).
void dvattn_paged_sdpa_rope_op(at::Tensor& out, double scale, const at::Tensor& locations, const at::Tensor& queries,
                               const at::Tensor& fragment_lengths, const at::Tensor& k_cache, const at::Tensor& v_cache,
                               const at::Tensor& block_tables, int64_t rotary_dim, double rope_base,
                               double attention_scaling, const c10::optional<at::Tensor>& inv_freq) {
    const RotaryOpt rot{(int)rotary_dim, rope_base, attention_scaling, &inv_freq};
    const at::Tensor none;
    paged_impl(out, scale, locations, queries, none, none, fragment_lengths, k_cache, v_cache, block_tables,
               c10::nullopt, c10::nullopt, &rot);
}

void dvattn_varlen_paged_sdpa_rope_op(at::Tensor& out, double scale, const at::Tensor& locations,
                                      const at::Tensor& queries, const at::Tensor& fragment_lengths,
                                      const at::Tensor& k_cache, const at::Tensor& v_cache,
                                      const at::Tensor& block_tables, const at::Tensor& cu_seqlens_q,
                                      const at::Tensor& cu_seqlens_k, int64_t rotary_dim, double rope_base,
                                      double attention_scaling, const c10::optional<at::Tensor>& inv_freq) {
    const RotaryOpt rot{(int)rotary_dim, rope_base, attention_scaling, &inv_freq};
    const at::Tensor none;
    varlen_impl(out, scale, locations, queries, none, none, fragment_lengths, k_cache, v_cache, block_tables,
                cu_seqlens_q, cu_seqlens_k, c10::nullopt, c10::nullopt, &rot);
}

// ---------------------------------------------------------------------------------
// dvattn_rope / dvattn_varlen_rope (src/binding.cu:41-77, 205-247)
// ---------------------------------------------------------------------------------
void dvattn_rope_op(at::Tensor& out, const at::Tensor& queries, const at::Tensor& cosines, const at::Tensor& sines) {
    const c10::cuda::CUDAGuard guard(out.device());
    const int dt = dtype_code(out);
    TORCH_CHECK(out.dim() == 5 && queries.dim() == 4 && cosines.dim() == 4 && sines.dim() == 4, "dvattn_rope: wrong tensor ranks");
    TORCH_CHECK(queries.scalar_type() == out.scalar_type(), "dvattn_rope: queries must have the output dtype");
    TORCH_CHECK(cosines.scalar_type() == at::kFloat && sines.scalar_type() == at::kFloat, "dvattn_rope: cosines/sines must be float32");
    check_all(out, {Named{&queries, "queries"}, Named{&cosines, "cosines"},
                    Named{&sines, "sines"}, Named{&out, "output"}});
    const int F = out.size(0), W = out.size(1), Hq = out.size(2), S = out.size(3), E = out.size(4);
    const int R = cosines.size(3);
    TORCH_CHECK(queries.size(0) == W && queries.size(1) == Hq && queries.size(2) == S && queries.size(3) == E,
                "dvattn_rope: queries must be [W, Hq, S, E]");
    TORCH_CHECK(cosines.size(0) == F && cosines.size(1) == W && cosines.size(2) == S, "dvattn_rope: cosines must be [F, W, S, R]");
    TORCH_CHECK(sines.sizes() == cosines.sizes(), "dvattn_rope: sines must match cosines");
    check_status(dvattn_rope(dt, F, W, Hq, S, E, R, out.data_ptr(), queries.const_data_ptr(),
                             cosines.const_data_ptr<float>(), sines.const_data_ptr<float>(), cur_stream(out)),
                 "dvattn_rope");
}

void dvattn_varlen_rope_op(at::Tensor& out, const at::Tensor& queries, const at::Tensor& cosines, const at::Tensor& sines) {
    const c10::cuda::CUDAGuard guard(out.device());
    const int dt = dtype_code(out);
    TORCH_CHECK(out.dim() == 4 && queries.dim() == 3 && cosines.dim() == 3 && sines.dim() == 3, "dvattn_varlen_rope: wrong tensor ranks");
    TORCH_CHECK(queries.scalar_type() == out.scalar_type(), "dvattn_varlen_rope: queries must have the output dtype");
    TORCH_CHECK(cosines.scalar_type() == at::kFloat && sines.scalar_type() == at::kFloat, "dvattn_varlen_rope: cosines/sines must be float32");
    check_all(out, {Named{&queries, "queries"}, Named{&cosines, "cosines"},
                    Named{&sines, "sines"}, Named{&out, "output"}});
    const int F = out.size(0), T = out.size(1), H = out.size(2), E = out.size(3);
    const int R = cosines.size(2) * 2;
    TORCH_CHECK(queries.size(0) == T && queries.size(1) == H && queries.size(2) == E, "dvattn_varlen_rope: queries must be [T, H, E]");
    TORCH_CHECK(cosines.size(0) == F && cosines.size(1) == T, "dvattn_varlen_rope: cosines must be [F, T, R/2]");
    TORCH_CHECK(sines.sizes() == cosines.sizes(), "dvattn_varlen_rope: sines must match cosines");
    check_status(dvattn_varlen_rope(dt, F, T, H, E, R, out.data_ptr(), queries.const_data_ptr(),
                                    cosines.const_data_ptr<float>(), sines.const_data_ptr<float>(), cur_stream(out)),
                 "dvattn_varlen_rope");
}

// ---------------------------------------------------------------------------------
// LSE merge of per-GPU partials (no reference counterpart as a public op)
// ---------------------------------------------------------------------------------
void dvattn_lse_merge_op(at::Tensor& out, const c10::optional<at::Tensor>& lse_out, const at::Tensor& part_out,
                         const at::Tensor& part_lse) {
    const c10::cuda::CUDAGuard guard(out.device());
    const int dt = dtype_code(out);
    TORCH_CHECK(part_out.scalar_type() == at::kFloat && part_lse.scalar_type() == at::kFloat, "dvattn_lse_merge: partials must be float32");
    check_cuda_tensor(part_out, "part_out", out);
    check_cuda_tensor(part_lse, "part_lse", out);
    check_cuda_tensor(out, "output", out);
    TORCH_CHECK(part_out.dim() >= 2, "dvattn_lse_merge: part_out must be [parts, ..., Ev]");
    const int parts = part_out.size(0);
    const int Ev = part_out.size(-1);
    const int64_t rows = out.numel() / Ev;
    TORCH_CHECK(part_out.numel() == (int64_t)parts * rows * Ev && part_lse.numel() == (int64_t)parts * rows,
                "dvattn_lse_merge: part_out [parts, rows.., Ev] / part_lse [parts, rows..] do not match output");
    float* lp = nullptr;
    if (lse_out.has_value()) {
        check_cuda_tensor(*lse_out, "lse_out", out);
        TORCH_CHECK(lse_out->scalar_type() == at::kFloat && lse_out->numel() == rows, "dvattn_lse_merge: lse_out must be f32 [rows]");
        lp = lse_out->data_ptr<float>();
    }
    check_status(dvattn_lse_merge(dt, parts, rows, Ev, part_out.const_data_ptr<float>(), part_lse.const_data_ptr<float>(),
                                  out.data_ptr(), lp, cur_stream(out)),
                 "dvattn_lse_merge");
}

// ---------------------------------------------------------------------------------
// dvattn_build_views (B200 addition): locations and cos/sin of the turn/view structure
// ---------------------------------------------------------------------------------
void dvattn_build_views_op(at::Tensor& locations, at::Tensor& cosines, at::Tensor& sines, const at::Tensor& seg_lengths,
                           const at::Tensor& seg_order, const c10::optional<at::Tensor>& inv_freq, double rope_base,
                           double attention_scaling, int64_t round_dtype) {
    const c10::cuda::CUDAGuard guard(locations.device());
    TORCH_CHECK(locations.dim() == 3 && cosines.dim() == 4 && sines.dim() == 4 && seg_lengths.dim() == 1 &&
                    seg_order.dim() == 2, "dvattn_build_views: wrong tensor ranks");
    check_i32(locations, "locations");
    check_i32(seg_lengths, "seg_lengths");
    check_i32(seg_order, "seg_order");
    TORCH_CHECK(cosines.scalar_type() == at::kFloat && sines.scalar_type() == at::kFloat,
                "dvattn_build_views: cosines/sines must be float32");
    check_all(locations, {Named{&locations, "locations"}, Named{&cosines, "cosines"}, Named{&sines, "sines"},
                          Named{&seg_lengths, "seg_lengths"}, Named{&seg_order, "seg_order"}});
    const int F = locations.size(0), W = locations.size(1), n = locations.size(2), R = cosines.size(3);
    TORCH_CHECK(seg_lengths.size(0) == F && seg_order.size(0) == W && seg_order.size(1) == F,
                "dvattn_build_views: seg_lengths [F], seg_order [W, F]");
    TORCH_CHECK(cosines.size(0) == F && cosines.size(1) == W && cosines.size(2) == n && sines.sizes() == cosines.sizes(),
                "dvattn_build_views: cosines/sines must be [F, W, n, R]");
    dvattn_views_args a{};
    a.F = F; a.W = W; a.n = n; a.R = R;
    a.rope_base = static_cast<float>(rope_base);
    a.attention_scaling = static_cast<float>(attention_scaling);
    a.round_dtype = static_cast<int>(round_dtype);
    a.seg_lengths = seg_lengths.const_data_ptr<int>();
    a.seg_order = seg_order.const_data_ptr<int>();
    if (inv_freq.has_value()) {
        check_cuda_tensor(*inv_freq, "inv_freq", locations);
        TORCH_CHECK(inv_freq->scalar_type() == at::kFloat && inv_freq->numel() == R / 2,
                    "dvattn_build_views: inv_freq must be f32 [R/2]");
        a.inv_freq = inv_freq->const_data_ptr<float>();
    }
    a.locations = locations.data_ptr<int>();
    a.cosines = cosines.data_ptr<float>();
    a.sines = sines.data_ptr<float>();
    check_status(dvattn_build_views(&a, cur_stream(locations)), "dvattn_build_views");
}

// ---------------------------------------------------------------------------------
// dvattn_paged_append (B200 addition): the new tokens' keys rotated as
// apply_rotary_pos_emb and written with their values into the workers' pages
// ---------------------------------------------------------------------------------
void dvattn_paged_append_op(at::Tensor& k_cache, at::Tensor& v_cache, const at::Tensor& keys, const at::Tensor& values,
                            const at::Tensor& cosines, const at::Tensor& sines, const at::Tensor& block_tables,
                            const at::Tensor& positions, const c10::optional<at::Tensor>& counts) {
    const c10::cuda::CUDAGuard guard(k_cache.device());
    const int dt = dtype_code(k_cache);
    TORCH_CHECK(k_cache.dim() == 4 && v_cache.dim() == 4 && keys.dim() == 4 && values.dim() == 4 &&
                    cosines.dim() == 3 && sines.dim() == 3 && block_tables.dim() == 2 && positions.dim() == 1,
                "dvattn_paged_append: wrong tensor ranks");
    for (const at::Tensor* t : {(const at::Tensor*)&v_cache, &keys, &values})
        TORCH_CHECK(t->scalar_type() == k_cache.scalar_type(), "dvattn_paged_append: caches and new tokens must share the dtype");
    TORCH_CHECK(cosines.scalar_type() == at::kFloat && sines.scalar_type() == at::kFloat,
                "dvattn_paged_append: cosines/sines must be float32");
    check_i32(block_tables, "block_tables");
    check_i32(positions, "positions");
    check_all(k_cache, {Named{&k_cache, "k_cache"}, Named{&v_cache, "v_cache"}, Named{&keys, "keys"},
                        Named{&values, "values"}, Named{&cosines, "cosines"}, Named{&sines, "sines"},
                        Named{&block_tables, "block_tables"}, Named{&positions, "positions"}});
    const int W = keys.size(0), Hkv = keys.size(1), n = keys.size(2), E = keys.size(3);
    const int Ev = values.size(3), R = cosines.size(2);
    TORCH_CHECK(values.size(0) == W && values.size(1) == Hkv && values.size(2) == n, "dvattn_paged_append: values must be [W, Hkv, n, Ev]");
    TORCH_CHECK(k_cache.size(2) == Hkv && k_cache.size(3) == E, "dvattn_paged_append: k_cache must be [NB, BS, Hkv, E]");
    TORCH_CHECK(v_cache.size(0) == k_cache.size(0) && v_cache.size(1) == k_cache.size(1) && v_cache.size(2) == Hkv &&
                    v_cache.size(3) == Ev, "dvattn_paged_append: v_cache must be [NB, BS, Hkv, Ev]");
    TORCH_CHECK(cosines.size(0) == W && cosines.size(1) == n && sines.sizes() == cosines.sizes(),
                "dvattn_paged_append: cosines/sines must be [W, n, R]");
    TORCH_CHECK(block_tables.size(0) == W && positions.size(0) == W, "dvattn_paged_append: block_tables [W, max_blocks], positions [W]");
    dvattn_append_args a{};
    a.dtype = dt;
    a.W = W; a.Hkv = Hkv; a.E = E; a.Ev = Ev; a.n = n; a.R = R;
    a.block_size = k_cache.size(1);
    a.max_blocks_per_seq = block_tables.size(1);
    a.num_blocks = k_cache.size(0);
    a.k_cache = k_cache.data_ptr();
    a.v_cache = v_cache.data_ptr();
    a.keys = keys.const_data_ptr();
    a.values = values.const_data_ptr();
    a.cosines = cosines.const_data_ptr<float>();
    a.sines = sines.const_data_ptr<float>();
    a.block_tables = block_tables.const_data_ptr<int>();
    a.positions = positions.const_data_ptr<int>();
    if (counts.has_value()) {
        check_cuda_tensor(*counts, "counts", k_cache);
        check_i32(*counts, "counts");
        TORCH_CHECK(counts->numel() == W, "dvattn_paged_append: counts must be [W]");
        a.counts = counts->const_data_ptr<int>();
    }
    check_status(dvattn_paged_append(&a, cur_stream(k_cache)), "dvattn_paged_append");
}

// ---------------------------------------------------------------------------------
// dvattn_sdpa / dvattn_fused: contiguous per-turn fragments (src/binding.cu:79-149,
// 356-372).  key_fragments[f] is [Hkv, L_f, E] or [B, Hkv, L_f, E] with B = 1 (one
// fragment shared by the W workers) or B = W; queries are [F, W, Hq, S, E], rotated.
// ---------------------------------------------------------------------------------
void sdpa_impl(at::Tensor& out, double scale, const at::Tensor& locations, const at::Tensor& queries,
               const at::Tensor& fragment_lengths, const std::vector<at::Tensor>& keys,
               const std::vector<at::Tensor>& values, const char* name) {
    const c10::cuda::CUDAGuard guard(out.device());
    const int dt = dtype_code(out);
    TORCH_CHECK(out.dim() == 4, name, ": output must be [W, Hq, S, Ev]");
    TORCH_CHECK(queries.dim() == 5 && locations.dim() == 3 && fragment_lengths.dim() == 1, name, ": wrong tensor ranks");
    TORCH_CHECK(queries.scalar_type() == out.scalar_type(), name, ": queries must have the output dtype");
    check_i32(locations, "locations");
    check_i32(fragment_lengths, "fragment_lengths");
    check_all(out, {Named{&out, "output"}, Named{&queries, "queries"}, Named{&locations, "locations"},
                    Named{&fragment_lengths, "fragment_lengths"}});
    const int W = out.size(0), Hq = out.size(1), S = out.size(2), Ev = out.size(3);
    const int F = locations.size(0), E = queries.size(4);
    TORCH_CHECK(locations.size(1) == W && locations.size(2) == S, name, ": locations must be [F, W, S]");
    TORCH_CHECK(queries.size(0) == F && queries.size(1) == W && queries.size(2) == Hq && queries.size(3) == S,
                name, ": queries must be [F, W, Hq, S, E]");
    TORCH_CHECK(fragment_lengths.size(0) == F, name, ": fragment_lengths must be [F]");
    TORCH_CHECK((int)keys.size() == F && (int)values.size() == F, name, ": need one key and one value fragment per turn");
    TORCH_CHECK(F > 0, name, ": at least one fragment");
    const bool batched = keys[0].dim() == 4;
    const int fo = batched ? 1 : 0;
    const int Hkv = keys[0].size(fo);
    std::vector<const void*> kp(F), vp(F);
    std::vector<int> rows(F), batch(F);
    for (int f = 0; f < F; ++f) {
        const at::Tensor& k = keys[f];
        const at::Tensor& v = values[f];
        TORCH_CHECK(k.dim() == 3 + fo && v.dim() == 3 + fo, name, ": fragments must all be [Hkv, L, E] or all [B, Hkv, L, E]");
        TORCH_CHECK(k.scalar_type() == out.scalar_type() && v.scalar_type() == out.scalar_type(), name,
                    ": fragments must have the output dtype");
        check_cuda_tensor(k, "key fragment", out);
        check_cuda_tensor(v, "value fragment", out);
        TORCH_CHECK(k.size(fo) == Hkv && v.size(fo) == Hkv, name, ": fragments must have Hkv heads");
        TORCH_CHECK(v.size(fo + 1) == k.size(fo + 1), name, ": key and value fragment lengths differ");
        TORCH_CHECK(k.size(fo + 2) == E && v.size(fo + 2) == Ev, name, ": fragment head dims must be E / Ev");
        const int B = batched ? (int)k.size(0) : 1;
        TORCH_CHECK(B == 1 || B == W, name, ": fragment batch must be 1 or W");
        TORCH_CHECK(!batched || v.size(0) == B, name, ": key and value fragment batches differ");
        kp[f] = k.const_data_ptr();
        vp[f] = v.const_data_ptr();
        rows[f] = (int)k.size(fo + 1);
        batch[f] = B;
    }
    dvattn_sdpa_args a{};
    a.dtype = dt;
    a.F = F; a.W = W; a.Hq = Hq; a.Hkv = Hkv; a.E = E; a.Ev = Ev; a.S = S;
    a.scale = static_cast<float>(scale);
    a.out = out.data_ptr();
    a.queries = queries.const_data_ptr();
    a.locations = locations.const_data_ptr<int>();
    a.fragment_lengths = fragment_lengths.const_data_ptr<int>();
    a.key_fragments = kp.data();
    a.value_fragments = vp.data();
    a.fragment_rows = rows.data();
    a.fragment_batch = batch.data();
    int st = dvattn_sdpa(&a, nullptr, 0, cur_stream(out));  // validation only when nothing to do
    if (st == DVATTN_ERR_WORKSPACE) {
        const size_t wsb = dvattn_sdpa_workspace_size(&a);
        TORCH_CHECK(wsb > 0, name, ": could not size the workspace");
        at::Tensor ws = at::empty({(int64_t)wsb}, out.options().dtype(at::kByte));
        st = dvattn_sdpa(&a, ws.data_ptr(), wsb, cur_stream(out));
        check_status(st, name);
        check_call_status(ws, cur_stream(out), name);
    }
    check_status(st, name);
}

void dvattn_sdpa_op(at::Tensor& out, double scale, const at::Tensor& locations, const at::Tensor& queries,
                    const at::Tensor& fragment_lengths, const std::vector<at::Tensor>& keys,
                    const std::vector<at::Tensor>& values) {
    sdpa_impl(out, scale, locations, queries, fragment_lengths, keys, values, "dvattn_sdpa");
}

// rope into rq, then attention over the (made contiguous) fragments, as the reference
void dvattn_fused_op(at::Tensor& out, at::Tensor& rq, double scale, const at::Tensor& locations, const at::Tensor& queries,
                     const at::Tensor& fragment_lengths, const std::vector<at::Tensor>& keys,
                     const std::vector<at::Tensor>& values, const at::Tensor& cosines, const at::Tensor& sines) {
    std::vector<at::Tensor> kc, vc;
    kc.reserve(keys.size());
    vc.reserve(values.size());
    for (const at::Tensor& k : keys) kc.push_back(k.contiguous());
    for (const at::Tensor& v : values) vc.push_back(v.contiguous());
    dvattn_rope_op(rq, queries, cosines, sines);
    sdpa_impl(out, scale, locations, rq, fragment_lengths, kc, vc, "dvattn_fused");
}

}  // namespace

TORCH_LIBRARY(libdvatt, m) {
    std::vector<at::Tag> tags{at::Tag::needs_fixed_stride_order};
    m.def("dvattn_sdpa(Tensor(a!) output, float scale, Tensor locations, Tensor queries, "
          "Tensor fragment_lengths, Tensor[] key_fragments, Tensor[] value_fragments) -> ()", tags, torch::_RegisterOrVerify::REGISTER);
    m.def("dvattn_paged_sdpa(Tensor(a!) output, float scale, Tensor locations, Tensor queries, "
          "Tensor cosines, Tensor sines, Tensor fragment_lengths, Tensor k_cache, Tensor v_cache, Tensor block_tables) -> ()", tags, torch::_RegisterOrVerify::REGISTER);
    m.def("dvattn_rope(Tensor(a!) output, Tensor queries, Tensor cosines, Tensor sines) -> ()", tags, torch::_RegisterOrVerify::REGISTER);
    m.def("dvattn_fused(Tensor(a!) output, Tensor(b!) rq, float scale, Tensor locations, Tensor queries, "
          "Tensor fragment_lengths, Tensor[] key_fragments, Tensor[] value_fragments, Tensor cosines, Tensor sines) -> ()", tags, torch::_RegisterOrVerify::REGISTER);
    m.def("dvattn_varlen_rope(Tensor(a!) output, Tensor queries, Tensor cosines, Tensor sines) -> ()", tags, torch::_RegisterOrVerify::REGISTER);
    m.def("dvattn_varlen_paged_sdpa(Tensor(a!) output, float scale, Tensor locations, Tensor queries, "
          "Tensor cosines, Tensor sines, Tensor fragment_lengths, Tensor k_cache, Tensor v_cache, "
          "Tensor block_tables, Tensor cu_seqlens_q, Tensor cu_seqlens_k) -> ()", tags, torch::_RegisterOrVerify::REGISTER);
    // B200 additions: optional natural-log LSE and f32 output (for cross-GPU merges), and the merge itself.
    m.def("dvattn_paged_sdpa_ex(Tensor(a!) output, Tensor(b!)? lse, Tensor(c!)? out_f32, float scale, Tensor locations, "
          "Tensor queries, Tensor cosines, Tensor sines, Tensor fragment_lengths, Tensor k_cache, Tensor v_cache, "
          "Tensor block_tables) -> ()", tags, torch::_RegisterOrVerify::REGISTER);
    m.def("dvattn_varlen_paged_sdpa_ex(Tensor(a!) output, Tensor(b!)? lse, Tensor(c!)? out_f32, float scale, "
          "Tensor locations, Tensor queries, Tensor cosines, Tensor sines, Tensor fragment_lengths, Tensor k_cache, "
          "Tensor v_cache, Tensor block_tables, Tensor cu_seqlens_q, Tensor cu_seqlens_k) -> ()", tags, torch::_RegisterOrVerify::REGISTER);
    m.def("dvattn_lse_merge(Tensor(a!) output, Tensor(b!)? lse_out, Tensor part_out, Tensor part_lse) -> ()", tags, torch::_RegisterOrVerify::REGISTER);
    m.def("dvattn_paged_sdpa_rope(Tensor(a!) output, float scale, Tensor locations, Tensor queries, "
          "Tensor fragment_lengths, Tensor k_cache, Tensor v_cache, Tensor block_tables, int rotary_dim, "
          "float rope_base, float attention_scaling, Tensor? inv_freq) -> ()", tags, torch::_RegisterOrVerify::REGISTER);
    m.def("dvattn_varlen_paged_sdpa_rope(Tensor(a!) output, float scale, Tensor locations, Tensor queries, "
          "Tensor fragment_lengths, Tensor k_cache, Tensor v_cache, Tensor block_tables, Tensor cu_seqlens_q, "
          "Tensor cu_seqlens_k, int rotary_dim, float rope_base, float attention_scaling, Tensor? inv_freq) -> ()",
          tags, torch::_RegisterOrVerify::REGISTER);
    m.def("dvattn_build_views(Tensor(a!) locations, Tensor(b!) cosines, Tensor(c!) sines, Tensor seg_lengths, "
          "Tensor seg_order, Tensor? inv_freq, float rope_base, float attention_scaling, int round_dtype) -> ()", tags, torch::_RegisterOrVerify::REGISTER);
    m.def("dvattn_paged_append(Tensor(a!) k_cache, Tensor(b!) v_cache, Tensor keys, Tensor values, Tensor cosines, "
          "Tensor sines, Tensor block_tables, Tensor positions, Tensor? counts) -> ()", tags, torch::_RegisterOrVerify::REGISTER);
}

TORCH_LIBRARY_IMPL(libdvatt, CUDA, m) {
    m.impl("dvattn_sdpa", dvattn_sdpa_op);
    m.impl("dvattn_paged_sdpa", dvattn_paged_sdpa_op);
    m.impl("dvattn_rope", dvattn_rope_op);
    m.impl("dvattn_fused", dvattn_fused_op);
    m.impl("dvattn_varlen_rope", dvattn_varlen_rope_op);
    m.impl("dvattn_varlen_paged_sdpa", dvattn_varlen_paged_sdpa_op);
    m.impl("dvattn_paged_sdpa_ex", dvattn_paged_sdpa_ex_op);
    m.impl("dvattn_varlen_paged_sdpa_ex", dvattn_varlen_paged_sdpa_ex_op);
    m.impl("dvattn_lse_merge", dvattn_lse_merge_op);
    m.impl("dvattn_paged_append", dvattn_paged_append_op);
    m.impl("dvattn_build_views", dvattn_build_views_op);
    m.impl("dvattn_paged_sdpa_rope", dvattn_paged_sdpa_rope_op);
    m.impl("dvattn_varlen_paged_sdpa_rope", dvattn_varlen_paged_sdpa_rope_op);
}
