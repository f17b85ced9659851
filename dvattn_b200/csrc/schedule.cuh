// Balanced split-KV schedule shared by the paged-decode kernels and their merge.
//
// Work unit = one visible key token of one (query row, KV head) "segment" (or of one
// query row with all its KV heads, when hsplit == 1).  Segment g = ws * Hkv + hkv, where
// ws = w * S + s indexes the query rows of the paged op.
// The visible keys of a segment are the concatenation over turns f of the keys
// l < V_f(ws) = min(L_f, loc[f,ws] + 1) (clipped to the block table), so masked turn
// padding is never scheduled.  Units are ordered segment-major; with P[ws] the
// exclusive prefix of V(ws) = sum_f V_f(ws), segment g starts at unit
// P[ws] * Hkv + hkv * V(ws).  CTA c of n owns units [c*U/n, (c+1)*U/n): every CTA streams
// the same number of key bytes whatever the sequence lengths are, and a segment is
// split only where a CTA boundary falls inside it.  A CTA that covers a whole segment
// writes the final output; the pieces of a split segment go to partial slots
// (slot 2c for the CTA's first segment, 2c+1 for its last) and are merged by
// `decode_merge_kernel`.
//
// This replaces the reference's uniform split (grid.z = max(2, SMs / (Hkv*W*S)) CTAs
// striding over every key position, src/kernels/paged_kernel_v21.cuh:385-392).
#pragma once

#include "common.cuh"

namespace dvb {

// One contiguous K/V fragment of the dvattn_sdpa op: K of turn f, KV head h, worker w,
// key l at k + ((w * wmul * Hkv + h) * rows + l) * E (wmul = 0: one fragment shared by
// all workers, 1: a batch dimension of W); keys l >= rows read as zeros.
struct FragDesc {
    const void* k;
    const void* v;
    int rows;
    int wmul;
};

struct DecodeSched {
    long long U;  // total units
    int n_eff;    // CTAs that own units (<= n_launch)
    int error;    // nonzero: a bounded wait gave up (the outputs of this call are invalid)
};
static_assert(offsetof(DecodeSched, error) == 12, "the error word is read at byte 12 (kErrorWordOffset)");

// Device-side view of one paged decode call (passed by value).
struct PagedParams {
    int F, W, Hq, Hkv, E, S, R, BS, maxb, WS, gqa, cap;
    long long NB;
    float scale_log2;  // scale * log2(e)
    void* out;
    const void* q;
    const float* cos;
    const float* sin;
    const int* loc;
    const int* L;
    const void* k;
    const void* v;
    const int* bt;
    float* lse_out;
    float* out_f32;
    DecodeSched* sched;
    long long* P;      // [WS + 1]
    float* part_o;     // [n_launch * 2][16][E]
    float* part_lse;   // [n_launch * 2][16]
    int n_launch;
    int min_units;
    // varlen: query row ws is packed token t (S == 1); its block-table row is the
    // sequence containing t, found once by the prep kernel from cu_seqlens_q.
    const int* cu_q;   // [nseq + 1] or null (decode: block-table row = ws / S)
    int nseq;
    int* row_seq;      // [WS] workspace, valid when cu_q != null
    int cs_stride;     // floats per cos/sin row: R (decode) or R/2 (varlen)
    // Unit ordering: a row's visible keys form `hsplit` segments (one per KV head, hsplit
    // = Hkv) for kernels that stream one head per CTA, or one segment covering all heads
    // (hsplit = 1) for the row kernel; a partial slot holds `slot_heads` heads.
    int hsplit;
    int slot_heads;
    int bs_shift;      // log2(block_size) when it is a power of two, else -1
    long long* cstart; // [n_launch + 1] first unit of each CTA's range (written by the prep kernel)
    int rot_units;     // units charged for a turn start (its query rotation) in the balanced split
    // 1: no prep kernel; every attention CTA computes the split itself (cta_prefix /
    // cta_boundary) and publishes its share of P / cstart / the header for the merge
    int fused;
    // contiguous fragments (dvattn_sdpa): nfrag = F descriptors in device memory, keys
    // addressed per turn instead of through the block table; the queries are per turn
    // (q_turn_stride elements apart) and already rotated (R = 0)
    int nfrag;
    long long q_turn_stride;
    const FragDesc* frag;
    // row kernel on fragments: 2 * nfrag 128-byte tensor maps (K then V of each turn) in
    // the workspace
    const char* fmaps;
    // Test hook (DVATTN_TEST_STALL_TILE): the row kernel's CTA 0 never issues the loads of
    // this tile, so a bounded wait runs out and the call reports its error word; -1: off.
    int stall_tile;
    int n_sm;        // SMs of the device (0: no one-wave cap)
    long long unit_bytes;  // K+V bytes streamed per unit
    int rotate;  // row kernel: walk each CTA's range from its first segment start (RotTileIter)
};



__device__ __forceinline__ int row_block_table(const PagedParams& p, int ws) {
    return p.cu_q ? p.row_seq[ws] : ws / p.S;
}

// Visible keys of turn f (offset `off` in the sequence's logical cache) for a query with
// location `loc`: l < L, l <= loc, and off + l inside the block table (`cap` positions).
__device__ __forceinline__ int turn_vis(int L, int loc, int off, int cap) {
    int v = min(L, loc + 1);
    v = min(v, cap - off);
    return v > 0 ? v : 0;
}

// Units of one row segment: each turn with visible keys counts its keys plus
// rot_units for its query rotation, so the balanced split charges CTAs for the
// rotations they do, not only for the keys they stream.
__device__ __forceinline__ int turn_units(int vis, int rot) { return vis > 0 ? vis + rot : 0; }
__device__ __forceinline__ int seg_visible(const PagedParams& p, int ws) {
    int off = 0, tot = 0;
    for (int f = 0; f < p.F; ++f) {
        int L = __ldg(p.L + f);
        tot += turn_units(turn_vis(L, __ldg(p.loc + (size_t)f * p.WS + ws), off, p.cap), p.rot_units);
        off += L;
    }
    return tot;
}

// CTA whose (non-empty) unit range contains u: the largest c < n with cstart[c] <= u.
__device__ __forceinline__ int cta_of(const long long* cstart, long long u, int n) {
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (cstart[mid] <= u) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// One pass over the schedule: fills P and the header.  Single CTA of 1024 threads.
// First unit of CTA c of n: c * U / n, moved back to the start of a turn when it falls
// inside the rotation units of that turn, so every turn's rotation is done by the CTA that
// streams the turn's first keys.  Pq: the prefix sums P (shared or global memory).
__device__ __forceinline__ long long cta_boundary(const PagedParams& p, const long long* Pq, long long U, int n, int c) {
    if (c >= n) return U;
    long long u = (n > 0) ? (long long)c * U / n : 0;
    if (c > 0) {
        int lo = 0, hi = p.WS - 1;  // row: largest ws with P[ws] * hsplit <= u
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (Pq[mid] * p.hsplit <= u) lo = mid; else hi = mid - 1;
        }
        const int ws = lo;
        const long long V = Pq[ws + 1] - Pq[ws];
        if (V > 0) {
            const long long r = u - Pq[ws] * p.hsplit;
            long long acc = (r / V) * V;  // start of the segment (KV head) within the row
            int off = 0;
            for (int f = 0; f < p.F; ++f) {
                const int L = __ldg(p.L + f);
                const int tu = turn_units(turn_vis(L, __ldg(p.loc + (size_t)f * p.WS + ws), off, p.cap), p.rot_units);
                // (turn start, end of its rotation units]: snap to the turn start, so a
                // non-empty range holding a turn's rotation units also holds its first key
                if (tu > 0 && r <= acc + p.rot_units) {
                    u -= r - acc;
                    break;
                }
                if (r < acc + tu) break;
                acc += tu;
                off += L;
            }
        }
    }
    return u;
}

// Number of CTAs that own units: ceil(U / min_units) capped at n_launch (>= 1 if U > 0).
// A call streaming less than kOneWaveBytes is further capped at one CTA per SM (p.n_sm):
// with two per SM its rows split into twice as many pieces whose partials and merge cost
// more than the second CTA's overlap gains (config 2 at 8 sequences: 36.3 -> 29.7 µs per
// call; at 4: 33.0 -> 22-27 µs; from 16 sequences up, 2 per SM is as fast or faster).
constexpr long long kOneWaveBytes = 96ll << 20;
__device__ __forceinline__ int sched_ctas(const PagedParams& p, long long U) {
    const long long want = (U + p.min_units - 1) / p.min_units;
    int cap = p.n_launch;
    if (p.n_sm > 0 && p.unit_bytes > 0 && U * p.unit_bytes < kOneWaveBytes && p.n_sm < cap) cap = p.n_sm;
    int n = (int)(want < cap ? want : cap);
    return U > 0 ? (n > 0 ? n : 1) : 0;
}

// In-kernel schedule (PagedParams::fused): block-wide exclusive scan of the row unit
// counts into sP[0..WS] (shared memory), then U and the CTA count.  All threads of the
// block call it; sP must hold WS + 1 entries.
template <int NT>
__device__ __forceinline__ void cta_prefix(const PagedParams& p, long long* sP, long long* sScratch, long long& U,
                                           int& n) {
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    constexpr int NW = NT / 32;
    long long carry = 0;
    for (int base = 0; base < p.WS; base += NT) {
        const int ws = base + tid;
        const long long v = ws < p.WS ? (long long)seg_visible(p, ws) : 0;
        long long x = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const long long y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) sScratch[wid] = x;
        __syncthreads();
        long long before = carry;
        for (int w2 = 0; w2 < wid; ++w2) before += sScratch[w2];
        if (ws < p.WS) sP[ws] = before + x - v;
        long long tot = carry;
        for (int w2 = 0; w2 < NW; ++w2) tot += sScratch[w2];
        carry = tot;
        __syncthreads();
    }
    if (tid == 0) sP[p.WS] = carry;
    U = carry * p.hsplit;
    n = sched_ctas(p, U);
    __syncthreads();
}

__global__ void __launch_bounds__(1024) decode_prep_kernel(PagedParams p) {
    __shared__ long long warp_tot[32];
    __shared__ long long carry_s;
    constexpr int kSharedRows = 2048;  // rows whose prefix sums are also kept in shared memory
    __shared__ long long sP[kSharedRows + 1];
    constexpr int kSharedCtas = 2048;  // CTA boundaries computed before the wait below
    __shared__ long long sC[kSharedCtas + 1];
    // let the attention kernel launch now; it waits (griddepcontrol.wait) for our results
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // This kernel is itself a programmatic dependent of the previous call's merge, which
    // still reads the workspace: everything up to the writes is computed before waiting
    // for it (when the rows fit in shared memory), so that work overlaps the merge.
    const bool early = p.WS <= kSharedRows;
    if (!early) asm volatile("griddepcontrol.wait;" ::: "memory");
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    if (tid == 0) carry_s = 0;
    __syncthreads();
    for (int base = 0; base < p.WS; base += 1024) {
        const int ws = base + tid;
        long long v = ws < p.WS ? (long long)seg_visible(p, ws) : 0;
        // inclusive warp scan
        long long x = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            long long y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) warp_tot[wid] = x;
        __syncthreads();
        if (wid == 0) {
            long long t = warp_tot[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                long long y = __shfl_up_sync(0xffffffffu, t, o);
                if (lane >= o) t += y;
            }
            warp_tot[lane] = t;  // inclusive prefix of warp totals
        }
        __syncthreads();
        const long long carry = carry_s;
        const long long excl = carry + (wid ? warp_tot[wid - 1] : 0) + x - v;
        if (ws < p.WS) {
            if (!early) p.P[ws] = excl;
            if (ws <= kSharedRows) sP[ws] = excl;
        }
        __syncthreads();
        if (tid == 1023) carry_s = excl + v;
        __syncthreads();
    }
    __shared__ int n_s;
    __shared__ long long U_s;
    if (tid == 0) {
        const long long tot = carry_s;
        if (!early) p.P[p.WS] = tot;
        if (p.WS <= kSharedRows) sP[p.WS] = tot;
        const long long U = tot * p.hsplit;
        const int n = sched_ctas(p, U);
        n_s = n;
        U_s = U;
    }
    __syncthreads();
    // CTA boundaries: c * U / n, moved back to the start of a turn when they fall inside
    // the rotation units of that turn (cta_boundary).
    const int n = n_s;
    const long long U = U_s;
    const long long* Pq = p.WS <= kSharedRows ? sP : p.P;
    if (early && n > kSharedCtas) asm volatile("griddepcontrol.wait;" ::: "memory");
    for (int c = tid; c <= n; c += 1024) {
        const long long cs = cta_boundary(p, Pq, U, n, c);
        if (early && n <= kSharedCtas) sC[c] = cs; else p.cstart[c] = cs;
        if (c == 0 && !early) {
            p.sched->U = U;
            p.sched->error = 0;
            p.sched->n_eff = n;
        }
    }
    if (early) {
        __syncthreads();
        asm volatile("griddepcontrol.wait;" ::: "memory");
        for (int ws = tid; ws <= p.WS; ws += 1024) p.P[ws] = sP[ws];
        if (n <= kSharedCtas)
            for (int c = tid; c <= n; c += 1024) p.cstart[c] = sC[c];
        if (tid == 0) {
            p.sched->U = U;
            p.sched->error = 0;
            p.sched->n_eff = n;
        }
    }
    if (p.cu_q) {  // after the wait in both modes
        // sequence of each packed token: the first w with t < cu[w+1]
        // (src/kernels/varlen_paged_kernel_v21.cuh:40-47), 0 if there is none.
        for (int t = tid; t < p.WS; t += 1024) {
            int lo = 0, hi = p.nseq;  // search in [lo, hi)
            while (lo < hi) {
                const int mid = (lo + hi) >> 1;
                if (t < __ldg(p.cu_q + mid + 1)) hi = mid; else lo = mid + 1;
            }
            p.row_seq[t] = lo < p.nseq ? lo : 0;
        }
    }
}

// Walks the tiles of one CTA's unit range in order.  Each tile lies inside one turn of
// one segment and holds at most TILE keys.  Producer (loads) and consumer (math) each
// run their own copy in lock step.
struct TileDesc {
    int ws, hkv, f, pos0, n;
    int off;  // logical position of the turn's first key
    bool new_seg, new_turn, seg_last, seg_complete, first_piece;
};

// With `align` > 0 (a power of two <= TILE) tiles also never cross an align-sized window
// of logical positions, so a tile's keys sit at fixed window rows, as the TMA kernels'
// page boxes need.
template <int TILE> struct TileIter {
    int ws, hkv, f, t, off, vis;
    long long rem;
    int seg_left;
    bool from_start, pend_seg, pend_turn, first_seg;
    int align;

    // units of row w (= P[w + 1] - P[w]), from the inputs: the iterator never reads P, so
    // it also runs under the in-kernel schedule, where P is published only at the end
    __device__ __forceinline__ int seg_len(const PagedParams& p, int w) const { return seg_visible(p, w); }

    // ws0: segment row containing u0 and P0 = P[ws0] (found by the caller); u0/u1: unit range.
    __device__ __forceinline__ void init(const PagedParams& p, int ws0, long long P0, long long u0, long long u1) {
        ws = ws0;
        const int V = seg_len(p, ws);
        long long r = u0 - P0 * p.hsplit;
        hkv = (int)(r / V);
        int ts = (int)(r - (long long)hkv * V);
        seg_left = V - ts;
        from_start = (ts == 0);
        f = 0;
        off = 0;
        vis = turn_vis(__ldg(p.L), __ldg(p.loc + ws), 0, p.cap);
        while (ts >= turn_units(vis, p.rot_units)) {
            ts -= turn_units(vis, p.rot_units);
            off += __ldg(p.L + f);
            ++f;
            vis = turn_vis(__ldg(p.L + f), __ldg(p.loc + (size_t)f * p.WS + ws), off, p.cap);
        }
        t = ts - p.rot_units;  // negative while inside the turn's rotation units
        rem = u1 - u0;
        pend_seg = pend_turn = true;
        first_seg = true;
        align = 0;
    }

    __device__ __forceinline__ bool next(const PagedParams& p, TileDesc& d) {
        if (rem <= 0) return false;
        for (;;) {
            if (t < 0) {  // rotation units: cost only, no keys
                const int k = (long long)(-t) < rem ? -t : (int)rem;
                t += k;
                rem -= k;
                seg_left -= k;
                if (rem <= 0) return false;
                continue;
            }
            if (t < vis) break;
            off += __ldg(p.L + f);
            ++f;
            pend_turn = true;
            if (f == p.F) {
                f = 0;
                off = 0;
                if (++hkv == p.hsplit) {
                    hkv = 0;
                    do { ++ws; } while (seg_visible(p, ws) == 0);
                }
                seg_left = seg_len(p, ws);
                from_start = true;
                pend_seg = true;
                first_seg = false;
            }
            vis = turn_vis(__ldg(p.L + f), __ldg(p.loc + (size_t)f * p.WS + ws), off, p.cap);
            t = vis > 0 ? -p.rot_units : 0;
        }
        int n = vis - t;
        if (n > TILE) n = TILE;
        if (align) {
            const int room = align - ((off + t) & (align - 1));
            if (n > room) n = room;
        }
        if ((long long)n > rem) n = (int)rem;
        d.ws = ws;
        d.hkv = hkv;
        d.f = f;
        d.pos0 = off + t;
        d.off = off;
        d.n = n;
        d.new_seg = pend_seg;
        d.new_turn = pend_turn;
        d.first_piece = first_seg;
        t += n;
        rem -= n;
        seg_left -= n;
        d.seg_last = (seg_left == 0) || (rem == 0);
        d.seg_complete = from_start && (seg_left == 0);
        pend_seg = pend_turn = false;
        return true;
    }
};

// A CTA's unit range [u0, u1) walked from the first segment start b inside it: first
// [b, u1), then [u0, b).  The piece [u0, b) -- the tail of a segment an earlier CTA began --
// comes last, so every piece whose result is only a partial ends at the end of the CTA's
// work, and its first global write comes after nearly all its streaming (the writes wait
// for the previous grid, which may still be merging the previous call).  Slots keep their
// meaning: [u0, b) is the CTA's first segment (first_piece), the rest are not.  Without a
// segment start strictly inside the range this is the plain walk of [u0, u1).
template <int TILE> struct RotTileIter {
    TileIter<TILE> it;
    int phase, ws0, align;
    long long P0, u0, b;
    __device__ __forceinline__ void init(const PagedParams& p, int ws0_, long long P0_, long long u0_, long long u1,
                                         int wsb, long long b_, int align_) {
        ws0 = ws0_;
        P0 = P0_;
        u0 = u0_;
        b = b_;
        align = align_;
        if (b > u0 && b < u1) {
            phase = 0;
            it.init(p, wsb, b / p.hsplit, b, u1);
            it.first_seg = false;
        } else {
            phase = 1;
            it.init(p, ws0, P0, u0, u1);
        }
        it.align = align;
    }
    __device__ __forceinline__ bool next(const PagedParams& p, TileDesc& d) {
        if (it.next(p, d)) return true;
        if (phase != 0) return false;
        phase = 1;
        it.init(p, ws0, P0, u0, b);
        it.align = align;
        return it.next(p, d);
    }
};

// Segment row containing unit u0: the largest ws with P[ws] * Hkv <= u0 (so empty rows
// before a non-empty one are skipped).  Block-wide; all threads get the result.
__device__ __forceinline__ int find_row_in(const long long* Pq, int WS, int hsplit, long long u0) {
    int lo = 0, hi = WS - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (Pq[mid] * hsplit <= u0) lo = mid; else hi = mid - 1;
    }
    return lo;
}
template <int NT>
__device__ __forceinline__ int find_row(const PagedParams& p, long long u0) {
    int cnt = 0;
    for (int base = 0; base < p.WS; base += NT) {
        const int i = base + (int)threadIdx.x;
        const int pred = (i < p.WS) && (p.P[i] * p.hsplit <= u0);
        const int c = __syncthreads_count(pred);
        cnt += c;
        if (c < NT) break;
    }
    return cnt - 1;
}

}  // namespace dvb
