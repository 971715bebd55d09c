// decode.cu -- decode-time kernels of the IMI KV-cache path (sm_100a).
//
//   imi_similarity_kernel   reference-compatible cell scorer over merged fp32
//                           centroids (compute_impl.cu:62-103)
//   imi_select_kernel       separable cell scoring + top-nprobe + token budget
//                           + page truncation + execution row list, one CTA per
//                           KV group (retrieval.py:295-303,
//                           wave_buffer_cpu_hotcold.cpp:303-371,
//                           gather_copy.cu:100-213, async_update.py:20-76)
//   imi_attn_kernel         split-K gather attention over the row list
//                           (weighted_flash_decoding semantics, retrieval.py:439-447)
//   imi_combine_kernel      log-sum-exp merge of the split partials
//   imi_append_kernel       steady-zone append (runtime.py:378-392)
//   imi_async_assign_kernel batched decode-time cell assignment and running
//                           mean update (async_update.py:77-162)
//   imi_apply_kernel        publish updated cell centroids (async_update.py:7-19)
#include "common.cuh"
#include "imi_internal.h"

#include <float.h>

namespace imi {

// ----------------------------------------------------------------------------
// Reference-compatible scorer: sim[h, c] = fma chain over d of q_sum[d]*C[c,d]
// with q_sum[d] = sum_g float(q[h, g, d]) in g order.  One thread per cell; the
// grid spans (cells / 256, heads) instead of the reference's one CTA per head.
// ----------------------------------------------------------------------------
__global__ void imi_similarity_kernel(const uint16_t* __restrict__ q, const float* __restrict__ cent,
                                      float* __restrict__ out, int G, int n_cells, int dim, long long out_stride) {
    extern __shared__ float qs[];
    const int h = blockIdx.y;
    for (int d = threadIdx.x; d < dim; d += blockDim.x) {
        float acc = 0.0f;
        for (int g = 0; g < G; ++g) acc = __fadd_rn(acc, bf16_bits_to_f32(q[(size_t)(h * G + g) * dim + d]));
        qs[d] = acc;
    }
    __syncthreads();
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= n_cells) return;
    const float* row = cent + ((size_t)h * n_cells + c) * dim;
    float s = 0.0f;
    for (int d = 0; d < dim; d += 4) {
        const float4 v = *reinterpret_cast<const float4*>(row + d);
        s = __fmaf_rn(qs[d + 0], v.x, s);
        s = __fmaf_rn(qs[d + 1], v.y, s);
        s = __fmaf_rn(qs[d + 2], v.z, s);
        s = __fmaf_rn(qs[d + 3], v.w, s);
    }
    out[(size_t)h * out_stride + c] = s;
}

// ----------------------------------------------------------------------------
// Block-wide helpers (blockDim.x == SEL_THREADS).
// ----------------------------------------------------------------------------
constexpr int SEL_THREADS = 1024;
constexpr int SEL_CAP = 2048;      // candidates that are sorted exactly
constexpr int SEL_BUCKETS = 2048;  // histogram buckets per refinement round

__device__ int block_reduce_sum_i(int v, int* red) {
    v = warp_sum_i(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    if (w == 0) {
        v = (l < (int)(blockDim.x >> 5)) ? red[l] : 0;
        v = warp_sum_i(v);
        if (l == 0) red[0] = v;
    }
    __syncthreads();
    int r = red[0];
    __syncthreads();
    return r;
}

__device__ uint32_t block_reduce_u32(uint32_t v, bool is_max, uint32_t* red) {
    for (int o = 16; o > 0; o >>= 1) {
        uint32_t t = __shfl_xor_sync(0xffffffffu, v, o);
        v = is_max ? max(v, t) : min(v, t);
    }
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    if (w == 0) {
        v = (l < (int)(blockDim.x >> 5)) ? red[l] : (is_max ? 0u : 0xffffffffu);
        for (int o = 16; o > 0; o >>= 1) {
            uint32_t t = __shfl_xor_sync(0xffffffffu, v, o);
            v = is_max ? max(v, t) : min(v, t);
        }
        if (l == 0) red[0] = v;
    }
    __syncthreads();
    uint32_t r = red[0];
    __syncthreads();
    return r;
}

// Inclusive scan of one int per thread across the block.  Returns the inclusive
// value; *total receives the block total.
__device__ int block_scan_incl(int v, int* red, int* total) {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    int x = v;
    for (int o = 1; o < 32; o <<= 1) {
        int t = __shfl_up_sync(0xffffffffu, x, o);
        if (l >= o) x += t;
    }
    __syncthreads();
    if (l == 31) red[w] = x;
    __syncthreads();
    if (w == 0) {
        const int nw = blockDim.x >> 5;
        int y = (l < nw) ? red[l] : 0;
        for (int o = 1; o < 32; o <<= 1) {
            int t = __shfl_up_sync(0xffffffffu, y, o);
            if (l >= o) y += t;
        }
        if (l < nw) red[l] = y;
    }
    __syncthreads();
    const int base = (w > 0) ? red[w - 1] : 0;
    if (total) *total = red[(blockDim.x >> 5) - 1];
    __syncthreads();
    return x + base;
}

// ----------------------------------------------------------------------------
// Separable cell scoring + selection + execution row list.  One CTA per KV
// group.  Shared memory: scores[n_slots] | qsum[dim] | prefix table |
// last-subspace centroids (transposed) | hist | sort keys | kept bitmap | misc.
// ----------------------------------------------------------------------------
struct SelectSmem {
    static __host__ __device__ size_t bytes(int n_slots, int dim, int table, int sub, int k_last) {
        size_t b = 0;
        b += sizeof(float) * ((size_t)n_slots + 4);            // scores
        b += sizeof(float) * (size_t)dim;                      // q_sum
        b += sizeof(float) * ((size_t)table + 4);              // prefix partial sums
        b += sizeof(float) * (size_t)sub * (size_t)(k_last + 1);  // last-subspace centroids, transposed (S > 1)
        b += sizeof(int) * SEL_BUCKETS;                        // histogram
        b += sizeof(unsigned long long) * SEL_CAP;             // sort keys
        b += sizeof(uint32_t) * (((size_t)n_slots + 31) / 32 + 1);  // kept-before-truncation bitmap
        b += 256 * sizeof(int);                                // reductions / misc
        return b + 64;
    }
};

__global__ void __launch_bounds__(SEL_THREADS, 1) imi_select_kernel(SelectArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int h = blockIdx.x;
    const int tid = threadIdx.x;
    const int S = a.parts == 0 ? 1 : a.parts;
    const int sub = a.dim / S;
    const int k_last = a.ks[S - 1];
    int table = 1;
    for (int s = 0; s < S - 1; ++s) table *= a.ks[s];

    unsigned char* p = smem_raw;
    float* sc = reinterpret_cast<float*>(p); p += sizeof(float) * ((size_t)a.n_slots + 4);
    float* qs = reinterpret_cast<float*>(p); p += sizeof(float) * a.dim;
    float* tab = reinterpret_cast<float*>(p); p += sizeof(float) * ((size_t)table + 4);
    float* cT = reinterpret_cast<float*>(p); p += sizeof(float) * (size_t)(S > 1 ? sub : 0) * (k_last + 1);
    int* hist = reinterpret_cast<int*>(p); p += sizeof(int) * SEL_BUCKETS;
    p = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(p) + 7) & ~uintptr_t(7));
    unsigned long long* keys = reinterpret_cast<unsigned long long*>(p); p += sizeof(unsigned long long) * SEL_CAP;
    uint32_t* kept_bits = reinterpret_cast<uint32_t*>(p); p += sizeof(uint32_t) * ((a.n_slots + 31) / 32 + 1);
    int* misc = reinterpret_cast<int*>(p);  // misc[0..63] scalars, misc[64..] reduction scratch
    int* red = misc + 64;

    const size_t hs = (size_t)h;
    const int32_t* sizes = a.cell_sizes + hs * a.n_slots;
    const uint8_t* mask = a.cell_mask + hs * a.n_slots;
    const int32_t* code = a.cell_code + hs * a.n_slots;
    const uint8_t* dirty = a.cell_dirty ? a.cell_dirty + hs * a.n_slots : nullptr;
    const float* merged = a.centroids + hs * a.n_slots * (size_t)a.dim;
    const float* subc = a.sub_centroids + hs * (size_t)S * a.kmax * sub;

    // ---- q_sum (compute_impl.cu:80-88): sum of the group's query heads in g order
    for (int d = tid; d < a.dim; d += blockDim.x) {
        float acc = 0.0f;
        for (int g = 0; g < a.G; ++g) acc = __fadd_rn(acc, bf16_bits_to_f32(a.q[(hs * a.G + g) * a.dim + d]));
        qs[d] = acc;
    }
    // last-subspace centroids, transposed [d][i]
    if (S > 1) {
        const float* cl = subc + (size_t)(S - 1) * a.kmax * sub;
        for (int e = tid; e < k_last * sub; e += blockDim.x) {
            const int i = e / sub, d = e - i * sub;
            cT[d * (k_last + 1) + i] = cl[(size_t)i * sub + d];
        }
    }
    for (int w = tid; w < (a.n_slots + 31) / 32 + 1; w += blockDim.x) kept_bits[w] = 0;
    __syncthreads();
    // ---- prefix partial sums over the first S-1 subspaces, level by level
    if (S > 1) {
        if (tid == 0) tab[0] = 0.0f;
        __syncthreads();
        int width = 1;
        for (int s = 0; s < S - 1; ++s) {
            const int ks = a.ks[s];
            const float* cs = subc + (size_t)s * a.kmax * sub;
            // new table entries: prefix index p (width), digit i (ks); written
            // after all reads of the previous level (double pass through regs)
            const int total = width * ks;
            float vals[8];
            int cnt = 0;
            for (int e = tid; e < total && cnt < 8; e += blockDim.x, ++cnt) {
                const int pi = e / ks, i = e - pi * ks;
                float acc = tab[pi];
                const float* cr = cs + (size_t)i * sub;
                for (int d = 0; d < sub; ++d) acc = __fmaf_rn(qs[s * sub + d], cr[d], acc);
                vals[cnt] = acc;
            }
            __syncthreads();
            cnt = 0;
            for (int e = tid; e < total && cnt < 8; e += blockDim.x, ++cnt) tab[e] = vals[cnt];
            __syncthreads();
            width = total;
        }
    }
    // ---- cell scores (compute_impl.cu:93-101 arithmetic, separable evaluation)
    const float NEG_INF = -INFINITY;
    for (int c = tid; c < a.n_slots; c += blockDim.x) {
        float s;
        const int cc = code[c];
        if (mask[c] || cc < 0) {
            s = NEG_INF;
        } else if (S == 1 || (dirty && dirty[c])) {
            const float* row = merged + (size_t)c * a.dim;
            s = 0.0f;
            for (int d = 0; d < a.dim; d += 4) {
                const float4 v = *reinterpret_cast<const float4*>(row + d);
                s = __fmaf_rn(qs[d], v.x, s);
                s = __fmaf_rn(qs[d + 1], v.y, s);
                s = __fmaf_rn(qs[d + 2], v.z, s);
                s = __fmaf_rn(qs[d + 3], v.w, s);
            }
        } else {
            int pidx = 0;
            for (int t = 0; t < S - 1; ++t) pidx = pidx * a.ks[t] + ((cc >> (8 * t)) & 0xff);
            const int il = (cc >> (8 * (S - 1))) & 0xff;
            s = tab[pidx];
            const float* q2 = qs + (S - 1) * sub;
#pragma unroll 8
            for (int d = 0; d < sub; ++d) s = __fmaf_rn(q2[d], cT[d * (k_last + 1) + il], s);
        }
        sc[c] = s;
        if (a.scores_out) a.scores_out[hs * a.n_slots + c] = s;
    }
    __syncthreads();

    // ---- candidate statistics
    int mycnt = 0;
    uint32_t mn = 0xffffffffu, mx = 0u;
    for (int c = tid; c < a.n_slots; c += blockDim.x) {
        const float s = sc[c];
        if (s != NEG_INF) {
            ++mycnt;
            const uint32_t o = ord_f32(s);
            mn = min(mn, o);
            mx = max(mx, o);
        }
    }
    const int ncand = block_reduce_sum_i(mycnt, red);
    uint32_t lo = block_reduce_u32(mn, false, reinterpret_cast<uint32_t*>(red));
    uint32_t hi = block_reduce_u32(mx, true, reinterpret_cast<uint32_t*>(red));
    const int want = min(a.nprobe, ncand);

    // ---- collect the top `want` candidates (exact order decided by the sort)
    // Invariant: every candidate with ord > hi is collected (`above` of them),
    // and the boundary candidate (rank want-1) has ord in [lo, hi].
    int* ncol = misc + 0;
    if (tid == 0) {
        *ncol = 0;
        misc[1] = 0;
    }
    __syncthreads();
    int above = 0;
    bool done = (want == 0);
    while (!done) {
        if (lo == hi) {
            // equal scores: the lowest slot indices rank first
            const int need = want - above;
            for (int base = 0; base < a.n_slots; base += blockDim.x) {
                const int c = base + tid;
                const int f = (c < a.n_slots && sc[c] != NEG_INF && ord_f32(sc[c]) == lo) ? 1 : 0;
                int tot;
                const int incl = block_scan_incl(f, red, &tot);
                const int before = misc[1];
                if (f && before + incl - 1 < need) {
                    const int at = atomicAdd(ncol, 1);
                    if (at < SEL_CAP) keys[at] = ((unsigned long long)lo << 32) | (0xffffffffu - (uint32_t)c);
                }
                __syncthreads();
                if (tid == 0) misc[1] = before + tot;
                __syncthreads();
            }
            break;
        }
        for (int b = tid; b < SEL_BUCKETS; b += blockDim.x) hist[b] = 0;
        __syncthreads();
        const unsigned long long range = (unsigned long long)(hi - lo) + 1ull;
        for (int c = tid; c < a.n_slots; c += blockDim.x) {
            const float s = sc[c];
            if (s == NEG_INF) continue;
            const uint32_t o = ord_f32(s);
            if (o < lo || o > hi) continue;
            atomicAdd(&hist[(int)(((unsigned long long)(o - lo) * SEL_BUCKETS) / range)], 1);
        }
        __syncthreads();
        // highest bucket b* with above + sum_{b >= b*} hist[b] >= want (one warp)
        if (tid < 32) {
            int carry = above, bstar = 0, incl_at = 0;
            for (int base = SEL_BUCKETS - 32; base >= 0; base -= 32) {
                const int b = base + (31 - tid);  // lane 0 = highest bucket of this chunk
                int x = hist[b];
                for (int o = 1; o < 32; o <<= 1) {
                    const int t = __shfl_up_sync(0xffffffffu, x, o);
                    if (tid >= o) x += t;
                }
                const int incl = carry + x;
                const unsigned hitm = __ballot_sync(0xffffffffu, incl >= want);
                if (hitm) {
                    const int ln = __ffs(hitm) - 1;
                    bstar = base + (31 - ln);
                    incl_at = __shfl_sync(0xffffffffu, incl, ln);
                    break;
                }
                carry = __shfl_sync(0xffffffffu, incl, 31);
            }
            if (tid == 0) {
                misc[2] = bstar;
                misc[3] = incl_at;
            }
        }
        __syncthreads();
        const int bstar = misc[2];
        const int incl_at = misc[3];
        const uint32_t b_lo = lo + (uint32_t)(((unsigned long long)bstar * range + SEL_BUCKETS - 1) / SEL_BUCKETS);
        const uint32_t b_hi =
            lo + (uint32_t)(((unsigned long long)(bstar + 1) * range + SEL_BUCKETS - 1) / SEL_BUCKETS) - 1u;
        const int in_b = hist[bstar];
        const bool finish = incl_at <= SEL_CAP;
        // finish: take [b_lo, hi]; otherwise take the buckets above b*, (b_hi, hi]
        const unsigned long long take_lo = finish ? (unsigned long long)b_lo : (unsigned long long)b_hi + 1ull;
        for (int c = tid; c < a.n_slots; c += blockDim.x) {
            const float s = sc[c];
            if (s == NEG_INF) continue;
            const uint32_t o = ord_f32(s);
            if ((unsigned long long)o >= take_lo && o <= hi) {
                const int at = atomicAdd(ncol, 1);
                if (at < SEL_CAP) keys[at] = ((unsigned long long)o << 32) | (0xffffffffu - (uint32_t)c);
            }
        }
        __syncthreads();
        if (finish) {
            done = true;
        } else {
            above = incl_at - in_b;
            lo = b_lo;
            hi = b_hi;
        }
        __syncthreads();
    }
    __syncthreads();
    const int nkeys = min(*ncol, SEL_CAP);
    // ---- bitonic sort, descending
    int npow = 2;
    while (npow < nkeys) npow <<= 1;
    for (int i = nkeys + tid; i < npow; i += blockDim.x) keys[i] = 0ull;
    __syncthreads();
    for (int k = 2; k <= npow; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = tid; i < (npow >> 1); i += blockDim.x) {
                const int x = 2 * j * (i / j) + (i % j);
                const int y = x + j;
                const unsigned long long kx = keys[x], ky = keys[y];
                const bool desc = ((x & k) == 0);
                if (desc ? (kx < ky) : (kx > ky)) {
                    keys[x] = ky;
                    keys[y] = kx;
                }
            }
            __syncthreads();
        }
    }
    // ---- budget rule (retrieval.py:295-303) + page truncation
    // (wave_buffer_cpu_hotcold.cpp:320-330) over the first `want` sorted entries
    const int m = min(want, nkeys);
    int* sel_slot = hist;                 // [SEL_CAP], histogram no longer needed
    int* sel_start = reinterpret_cast<int*>(keys) + 0;  // reused after reading keys (see below)
    int run_size = 0, run_pages = 0, run_sel = 0, run_kept = 0;
    const int* offs = a.cell_offsets + hs * (a.n_slots + 1);
    int32_t* rows = a.row_index + hs * (size_t)a.exec_capacity;
    const int static_len = a.static_len;
    // read the sorted slots into registers first so `keys` can be reused
    int my_slot[SEL_CAP / SEL_THREADS];
#pragma unroll
    for (int q = 0; q < SEL_CAP / SEL_THREADS; ++q) {
        const int r = q * SEL_THREADS + tid;
        my_slot[q] = (r < m) ? (int)(0xffffffffu - (uint32_t)(keys[r] & 0xffffffffull)) : -1;
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < SEL_CAP / SEL_THREADS; ++q) {
        const int r = q * SEL_THREADS + tid;
        if (q * SEL_THREADS >= m) break;
        const int slot = my_slot[q];
        const int sz = (r < m) ? sizes[slot] : 0;
        const int pg = sz > 0 ? (sz + a.page_size - 1) / a.page_size : 0;
        int tot_s, tot_p, tot_k, tot_f;
        const int incl_s = block_scan_incl(sz, red, &tot_s) + run_size;
        const int incl_p = block_scan_incl(pg, red, &tot_p) + run_pages;
        const bool kept = (r < m) && sz > 0 && (incl_s - sz) < a.max_tokens;
        const bool fin = kept && incl_p <= a.buffer_pages;
        block_scan_incl(kept ? 1 : 0, red, &tot_k);
        const int rank_f = block_scan_incl(fin ? 1 : 0, red, &tot_f) + run_sel;
        if (kept) atomicOr(&kept_bits[slot >> 5], 1u << (slot & 31));
        if (fin) {
            a.sel_cells[hs * a.nprobe + (rank_f - 1)] = slot;
            sel_slot[rank_f - 1] = slot;
            sel_start[rank_f - 1] = static_len + (incl_s - sz);
        }
        run_size += tot_s;
        run_pages += tot_p;
        run_sel += tot_f;
        run_kept += tot_k;
    }
    __syncthreads();
    const int nsel = run_sel;
    // execution row list: static zone, then the selected cells' list rows in
    // selection order (gather_copy.cu:100-213 with every page a miss)
    for (int r = tid; r < static_len; r += blockDim.x) rows[r] = (1 << 30) | r;
    {
        const int w = tid >> 5, ln = tid & 31;
        for (int i = w; i < nsel; i += (SEL_THREADS >> 5)) {
            const int slot = sel_slot[i];
            const int st = sel_start[i];
            const int off = offs[slot];
            const int sz = sizes[slot];
            for (int j = ln; j < sz; j += 32) rows[st + j] = off + j;
        }
    }
    int sel_rows = 0;
    if (nsel > 0) sel_rows = sel_start[nsel - 1] - static_len + sizes[sel_slot[nsel - 1]];
    __syncthreads();
    // delta rows that belong to a kept cell (async_update.py:46-76); the padding
    // id matches when the nprobe list holds any dropped entry
    int total = static_len + sel_rows;
    if (a.delta_count) {
        const int dcount = min(a.delta_count[h], a.delta_capacity);
        const bool has_pad = run_kept < a.nprobe;
        const int32_t* dids = a.delta_cell_ids + hs * a.delta_capacity;
        int appended = 0;
        for (int base = 0; base < dcount; base += blockDim.x) {
            const int pidx = base + tid;
            int f = 0;
            if (pidx < dcount) {
                const int cid = dids[pidx];
                if (cid >= 0 && cid < a.n_slots) f = (kept_bits[cid >> 5] >> (cid & 31)) & 1;
                if (cid == a.padding_id && has_pad) f = 1;
            }
            int tot;
            const int incl = block_scan_incl(f, red, &tot);
            if (f) {
                const int at = total + appended + incl - 1;
                if (at < a.exec_capacity) rows[at] = (2 << 30) | pidx;
            }
            appended += tot;
        }
        total = min(total + appended, a.exec_capacity);
    }
    if (tid == 0) {
        a.sel_count[h] = nsel;
        a.row_count[h] = total;
        if (a.kept_count) a.kept_count[h] = run_kept;
    }
}

// ----------------------------------------------------------------------------
// Split-K gather attention.  Grid (splits, groups), 4 warps.  Each warp streams
// 16-row tiles of the group's row list through a cp.async ring in shared memory
// (XOR-swizzled 16-byte chunks so ldmatrix is conflict-free), computes
// S = Q K^T and O += P V with mma.sync m16n8k16 (query heads on M), and keeps an
// online softmax.  Warps merge in shared memory; each CTA writes one partial.
// ----------------------------------------------------------------------------
constexpr int ATT_WARPS = 4;
constexpr int ATT_STAGES = 4;
constexpr int ATT_TILE = 16;                 // rows per tile
constexpr int ATT_ROWB = 256;                // bytes per row (dim 128, bf16)
constexpr int ATT_STAGE_BYTES = 2 * ATT_TILE * ATT_ROWB;  // K + V

IMI_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

IMI_DEV void cp_async16(uint32_t dst, const void* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes));
}
IMI_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
IMI_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

IMI_DEV void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
IMI_DEV void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
IMI_DEV void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
IMI_DEV uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

IMI_DEV const unsigned char* row_src(const AttnArgs& a, int h, int idx, bool is_v) {
    const int src = (unsigned)idx >> 30;
    const int row = idx & 0x3fffffff;
    if (src == 0) {
        const unsigned char* b = reinterpret_cast<const unsigned char*>(is_v ? a.list_values : a.list_keys);
        return b + ((size_t)h * a.list_rows + row) * ATT_ROWB;
    } else if (src == 1) {
        const unsigned char* b = reinterpret_cast<const unsigned char*>(is_v ? a.static_values : a.static_keys);
        return b + ((size_t)h * a.static_rows + row) * ATT_ROWB;
    }
    const unsigned char* b = reinterpret_cast<const unsigned char*>(is_v ? a.delta_values : a.delta_keys);
    if (!b) return nullptr;
    return b + ((size_t)h * a.delta_rows + row) * ATT_ROWB;
}

__global__ void __launch_bounds__(ATT_WARPS * 32) imi_attn_kernel(AttnArgs a) {
    extern __shared__ __align__(128) unsigned char att_smem[];
    const int h = blockIdx.y;
    const int split = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;
    const int rows_total = a.row_count[h];
    int chunk = (rows_total + a.splits - 1) / a.splits;
    chunk = (chunk + ATT_TILE - 1) & ~(ATT_TILE - 1);
    const int r0 = split * chunk;
    const int r1 = min(rows_total, r0 + chunk);
    const int ntiles = r1 > r0 ? (r1 - r0 + ATT_TILE - 1) / ATT_TILE : 0;
    const int32_t* ridx = a.row_index + (size_t)h * a.exec_capacity;

    unsigned char* wbuf = att_smem + (size_t)warp * ATT_STAGES * ATT_STAGE_BYTES;
    const uint32_t wbuf_s = smem_u32(wbuf);

    // Q fragments (query heads on M; heads >= G are zero rows)
    uint32_t qa[8][2];
    {
        const uint16_t* qh = a.q + (size_t)h * a.G * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (g < a.G) {
                const uint32_t* q32 = reinterpret_cast<const uint32_t*>(qh + (size_t)g * 128);
                qa[j][0] = q32[(16 * j + 2 * c) >> 1];
                qa[j][1] = q32[(16 * j + 8 + 2 * c) >> 1];
            } else {
                qa[j][0] = 0u;
                qa[j][1] = 0u;
            }
        }
    }
    const float sl2 = a.scale * 1.4426950408889634f;
    float m_run = -INFINITY, l_run = 0.0f;
    float o[16][4];
#pragma unroll
    for (int u = 0; u < 16; ++u) o[u][0] = o[u][1] = o[u][2] = o[u][3] = 0.0f;

    // tiles handled by this warp: t = warp, warp + ATT_WARPS, ...
    const int my_tiles = ntiles > warp ? (ntiles - warp + ATT_WARPS - 1) / ATT_WARPS : 0;

    auto issue = [&](int it) {
        const int t = warp + it * ATT_WARPS;
        const int stage = it % ATT_STAGES;
        const uint32_t sb = wbuf_s + stage * ATT_STAGE_BYTES;
        const int rbase = r0 + t * ATT_TILE;
        const int myrow = rbase + (lane & 15);
        const int myidx = (myrow < r1) ? ridx[myrow] : -1;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const int tensor = k >> 3;
            const int i = 2 * (k & 7) + (lane >> 4);
            const int ch = lane & 15;
            const int idx = __shfl_sync(0xffffffffu, myidx, i);
            const uint32_t dst = sb + tensor * (ATT_TILE * ATT_ROWB) + i * ATT_ROWB + ((ch ^ (i & 7)) << 4);
            const unsigned char* src = idx >= 0 ? row_src(a, h, idx, tensor == 1) : nullptr;
            if (src) {
                cp_async16(dst, src + ch * 16, 16);
            } else {
                cp_async16(dst, a.q, 0);  // zero-fill
            }
        }
    };

    // prologue: always ATT_STAGES-1 groups (some possibly empty) so that the
    // wait below always retires the group of the tile being consumed
    for (int it = 0; it < ATT_STAGES - 1; ++it) {
        if (it < my_tiles) issue(it);
        cp_async_commit();
    }
    for (int it = 0; it < my_tiles; ++it) {
        if (it + ATT_STAGES - 1 < my_tiles) issue(it + ATT_STAGES - 1);
        cp_async_commit();
        cp_async_wait<ATT_STAGES - 1>();
        __syncwarp();
        const int t = warp + it * ATT_WARPS;
        const int stage = it % ATT_STAGES;
        const uint32_t kb = wbuf_s + stage * ATT_STAGE_BYTES;
        const uint32_t vb = kb + ATT_TILE * ATT_ROWB;
        // S = Q K^T  (two n-tiles of 8 rows)
        float s0[4] = {0, 0, 0, 0}, s1[4] = {0, 0, 0, 0};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int row = (lane & 7) + ((lane >> 4) << 3);
            const int ch = 2 * j + ((lane >> 3) & 1);
            uint32_t b0, b1, b2, b3;
            ldsm_x4(kb + row * ATT_ROWB + ((ch ^ (row & 7)) << 4), b0, b1, b2, b3);
            mma_bf16(s0, qa[j][0], 0u, qa[j][1], 0u, b0, b1);
            mma_bf16(s1, qa[j][0], 0u, qa[j][1], 0u, b2, b3);
        }
        const int rbase = r0 + t * ATT_TILE;
        float x[4];
        x[0] = (rbase + 2 * c < r1) ? s0[0] * sl2 : -INFINITY;
        x[1] = (rbase + 2 * c + 1 < r1) ? s0[1] * sl2 : -INFINITY;
        x[2] = (rbase + 8 + 2 * c < r1) ? s1[0] * sl2 : -INFINITY;
        x[3] = (rbase + 9 + 2 * c < r1) ? s1[1] * sl2 : -INFINITY;
        float tmax = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
        const float m_new = fmaxf(m_run, tmax);
        float pr[4];
        if (m_new == -INFINITY) {
            pr[0] = pr[1] = pr[2] = pr[3] = 0.0f;
        } else {
            const float alpha = exp2f(m_run - m_new);
#pragma unroll
            for (int e = 0; e < 4; ++e) pr[e] = exp2f(x[e] - m_new);
            l_run = l_run * alpha + (pr[0] + pr[1] + pr[2] + pr[3]);
#pragma unroll
            for (int u = 0; u < 16; ++u) {
                o[u][0] *= alpha;
                o[u][1] *= alpha;
            }
            m_run = m_new;
        }
        const uint32_t pa0 = pack_bf16(pr[0], pr[1]);
        const uint32_t pa2 = pack_bf16(pr[2], pr[3]);
        // O += P V
#pragma unroll
        for (int u = 0; u < 16; u += 2) {
            const int row = (lane & 7) + (((lane >> 3) & 1) << 3);
            const int ch = u + (lane >> 4);
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(vb + row * ATT_ROWB + ((ch ^ (row & 7)) << 4), b0, b1, b2, b3);
            mma_bf16(o[u], pa0, 0u, pa2, 0u, b0, b1);
            mma_bf16(o[u + 1], pa0, 0u, pa2, 0u, b2, b3);
        }
        __syncwarp();
    }
    cp_async_wait<0>();
    // per-group l: sum the four lanes of the group
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
    __syncthreads();
    // merge warps through shared memory
    float* sm_m = reinterpret_cast<float*>(att_smem);           // [warps][8]
    float* sm_l = sm_m + ATT_WARPS * 8;                          // [warps][8]
    float* sm_o = sm_l + ATT_WARPS * 8;                          // [warps][8][128]
    if (c == 0) {
        sm_m[warp * 8 + g] = m_run;
        sm_l[warp * 8 + g] = l_run;
    }
#pragma unroll
    for (int u = 0; u < 16; ++u) {
        sm_o[(warp * 8 + g) * 128 + 8 * u + 2 * c] = o[u][0];
        sm_o[(warp * 8 + g) * 128 + 8 * u + 2 * c + 1] = o[u][1];
    }
    __syncthreads();
    const size_t pbase = ((size_t)h * a.splits + split) * a.G;
    for (int e = threadIdx.x; e < a.G * 128; e += blockDim.x) {
        const int gg = e >> 7, d = e & 127;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < ATT_WARPS; ++w) M = fmaxf(M, sm_m[w * 8 + gg]);
        float acc = 0.0f, L = 0.0f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < ATT_WARPS; ++w) {
                const float f = exp2f(sm_m[w * 8 + gg] - M);
                acc += sm_o[(w * 8 + gg) * 128 + d] * f;
                L += sm_l[w * 8 + gg] * f;
            }
        }
        a.part_o[(pbase + gg) * 128 + d] = acc;
        if (d == 0) {
            a.part_ml[(pbase + gg) * 2 + 0] = M;
            a.part_ml[(pbase + gg) * 2 + 1] = L;
        }
    }
}

__global__ void imi_combine_kernel(AttnArgs a) {
    const int h = blockIdx.x;
    for (int e = threadIdx.x; e < a.G * 128; e += blockDim.x) {
        const int gg = e >> 7, d = e & 127;
        float M = -INFINITY;
        for (int s = 0; s < a.splits; ++s) M = fmaxf(M, a.part_ml[(((size_t)h * a.splits + s) * a.G + gg) * 2]);
        float acc = 0.0f, L = 0.0f;
        if (M != -INFINITY) {
            for (int s = 0; s < a.splits; ++s) {
                const size_t pb = ((size_t)h * a.splits + s) * a.G + gg;
                const float f = exp2f(a.part_ml[pb * 2] - M);
                acc += a.part_o[pb * 128 + d] * f;
                L += a.part_ml[pb * 2 + 1] * f;
            }
        }
        const float r = L > 0.0f ? acc / L : 0.0f;
        reinterpret_cast<__nv_bfloat16*>(a.out)[((size_t)h * a.G + gg) * 128 + d] = __float2bfloat16_rn(r);
    }
}

// ----------------------------------------------------------------------------
// Steady-zone append: zone[h, pos, :] = new[h, :] for keys and values, and
// (optionally) the async-update batch slot (runtime.py:378-392,
// async_update.py:115-117).  One warp per (group, tensor).
// ----------------------------------------------------------------------------
__global__ void imi_append_kernel(AppendArgs a) {
    const int h = blockIdx.x;
    const int t = threadIdx.x >> 5;  // 0 = keys, 1 = values
    const int lane = threadIdx.x & 31;
    if (t > 1) return;
    const uint4* src = reinterpret_cast<const uint4*>(
        reinterpret_cast<const unsigned char*>(t ? a.new_values : a.new_keys) + (size_t)h * a.src_head_stride * 2);
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(t ? a.zone_values : a.zone_keys) +
                                          ((size_t)h * a.zone_rows + a.pos) * a.dim * 2);
    const int n16 = a.dim * 2 / 16;
    for (int i = lane; i < n16; i += 32) {
        const uint4 v = src[i];
        dst[i] = v;
        if (a.batch_keys) {
            uint4* bd = reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(t ? a.batch_values : a.batch_keys) +
                                                 ((size_t)h * a.batch_cap + a.batch_slot) * a.dim * 2);
            bd[i] = v;
        }
    }
}

// ----------------------------------------------------------------------------
// Batched decode-time cell assignment and running-mean update, one CTA per
// group (async_update.py:122-161).  Inner products follow the d-ordered fma
// chain (separable for unchanged cells, full row for updated cells); ties go
// to the lowest slot (torch.argmax).  Delta sums are added in token order.
// ----------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) imi_async_assign_kernel(AsyncArgs a) {
    extern __shared__ __align__(16) unsigned char as_smem[];
    const int h = blockIdx.x;
    const int tid = threadIdx.x;
    const int S = a.parts == 0 ? 1 : a.parts;
    const int sub = a.dim / S;
    const int B = a.batch;
    const size_t hs = h;
    float* kf = reinterpret_cast<float*>(as_smem);                 // [B][dim]
    float* tab = kf + (size_t)B * a.dim;                           // [B][table]
    int table = 1;
    for (int s = 0; s < S - 1; ++s) table *= a.ks[s];
    unsigned long long* best = reinterpret_cast<unsigned long long*>(tab + (size_t)B * table + 2);  // [B]
    int* ids = reinterpret_cast<int*>(best + B);                   // [B]
    for (int e = tid; e < B * a.dim; e += blockDim.x)
        kf[e] = bf16_bits_to_f32(a.batch_keys[(hs * a.batch_cap) * a.dim + e]);
    if (tid < B) best[tid] = 0ull;
    __syncthreads();
    const float* subc = a.sub_centroids + hs * (size_t)S * a.kmax * sub;
    const float* shadow = a.shadow + hs * a.n_slots * (size_t)a.dim;
    // prefix tables per key
    if (S > 1) {
        for (int b = 0; b < B; ++b) {
            if (tid == 0) tab[(size_t)b * table] = 0.0f;
        }
        __syncthreads();
        int width = 1;
        for (int s = 0; s < S - 1; ++s) {
            const int ks = a.ks[s];
            const int total = width * ks;
            const float* cs = subc + (size_t)s * a.kmax * sub;
            float vals[16];
            int cnt = 0;
            for (int e = tid; e < B * total && cnt < 16; e += blockDim.x, ++cnt) {
                const int b = e / total, r = e - b * total;
                const int pi = r / ks, i = r - pi * ks;
                float acc = tab[(size_t)b * table + pi];
                for (int d = 0; d < sub; ++d) acc = __fmaf_rn(kf[b * a.dim + s * sub + d], cs[(size_t)i * sub + d], acc);
                vals[cnt] = acc;
            }
            __syncthreads();
            cnt = 0;
            for (int e = tid; e < B * total && cnt < 16; e += blockDim.x, ++cnt) {
                const int b = e / total, r = e - b * total;
                tab[(size_t)b * table + r] = vals[cnt];
            }
            __syncthreads();
            width = total;
        }
    }
    // argmax over every slot (padding slots have zero centroids and score 0)
    for (int e = tid; e < B * a.n_slots; e += blockDim.x) {
        const int b = e / a.n_slots, cslot = e - b * a.n_slots;
        const int cc = a.cell_code[hs * a.n_slots + cslot];
        float s;
        if (S == 1 || cc < 0 || (a.shadow_dirty && a.shadow_dirty[hs * a.n_slots + cslot])) {
            const float* row = shadow + (size_t)cslot * a.dim;
            s = 0.0f;
            for (int d = 0; d < a.dim; ++d) s = __fmaf_rn(kf[b * a.dim + d], row[d], s);
        } else {
            int pidx = 0;
            for (int t = 0; t < S - 1; ++t) pidx = pidx * a.ks[t] + ((cc >> (8 * t)) & 0xff);
            const int il = (cc >> (8 * (S - 1))) & 0xff;
            s = (S > 1) ? tab[(size_t)b * table + pidx] : 0.0f;
            const float* cl = subc + ((size_t)(S - 1) * a.kmax + il) * sub;
            for (int d = 0; d < sub; ++d) s = __fmaf_rn(kf[b * a.dim + (S - 1) * sub + d], cl[d], s);
        }
        const unsigned long long key = ((unsigned long long)ord_f32(s) << 32) | (0xffffffffu - (uint32_t)cslot);
        atomicMax(&best[b], key);
    }
    __syncthreads();
    if (tid < B) ids[tid] = (int)(0xffffffffu - (uint32_t)(best[tid] & 0xffffffffull));
    __syncthreads();
    // delta counts / sums in token order (one warp walks the batch)
    if (tid < 32) {
        for (int b = 0; b < B; ++b) {
            const int cid = ids[b];
            float* ds = a.delta_sums + (hs * a.n_slots + cid) * (size_t)a.dim;
            for (int d = tid; d < a.dim; d += 32) ds[d] = __fadd_rn(ds[d], kf[b * a.dim + d]);
            if (tid == 0) a.delta_counts[hs * a.n_slots + cid] += 1;
            __syncwarp();
        }
    }
    __syncthreads();
    // running-mean update for cells that reached the threshold (each touched
    // cell once: the first batch entry that names it does the work)
    for (int b = 0; b < B; ++b) {
        const int cid = ids[b];
        bool first = true;
        for (int e = 0; e < b; ++e)
            if (ids[e] == cid) first = false;
        if (!first) continue;
        const size_t cs = hs * a.n_slots + cid;
        const int dc = a.delta_counts[cs];
        __syncthreads();
        if (dc >= a.threshold) {
            const int cnt = a.counts[cs];
            const int nc = cnt + dc;
            const float denom = (float)max(nc, 1);
            const float fc = (float)cnt;
            float* row = a.shadow + cs * a.dim;
            float* ds = a.delta_sums + cs * a.dim;
            for (int d = tid; d < a.dim; d += blockDim.x) {
                row[d] = __fdiv_rn(__fadd_rn(__fmul_rn(row[d], fc), ds[d]), denom);
                ds[d] = 0.0f;
            }
            __syncthreads();
            if (tid == 0) {
                a.counts[cs] = nc;
                a.delta_counts[cs] = 0;
                if (a.shadow_dirty) a.shadow_dirty[cs] = 1;
                if (a.pending) a.pending[cs] = 1;
            }
        }
        __syncthreads();
    }
    // delta ring (async_update.py:146-161)
    const int wp = a.ring_write_pos[h];
    for (int e = tid; e < B * (a.dim / 8); e += blockDim.x) {
        const int b = e / (a.dim / 8), q8 = e - b * (a.dim / 8);
        const int pos = (wp + b) % a.ring_cap;
        const uint4* sk = reinterpret_cast<const uint4*>(a.batch_keys + (hs * a.batch_cap + b) * a.dim) + q8;
        const uint4* sv = reinterpret_cast<const uint4*>(a.batch_values + (hs * a.batch_cap + b) * a.dim) + q8;
        reinterpret_cast<uint4*>(a.ring_keys + (hs * a.ring_cap + pos) * a.dim)[q8] = *sk;
        reinterpret_cast<uint4*>(a.ring_values + (hs * a.ring_cap + pos) * a.dim)[q8] = *sv;
    }
    if (tid < B) a.ring_cell_ids[hs * a.ring_cap + (wp + tid) % a.ring_cap] = ids[tid];
    __syncthreads();
    if (tid == 0) {
        a.ring_write_pos[h] = (wp + B) % a.ring_cap;
        a.ring_count[h] = min(a.ring_count[h] + B, a.ring_cap);
    }
    if (a.ids_out && tid < B) a.ids_out[hs * B + tid] = ids[tid];
}

// Publish the updated cells: live[c] = shadow[c] for slots flagged pending
// (async_update.py:7-19 copies the whole shadow; only changed rows differ).
__global__ void imi_apply_kernel(ApplyArgs a) {
    const int h = blockIdx.y;
    const size_t hs = h;
    for (int c = blockIdx.x; c < a.n_slots; c += gridDim.x) {
        const size_t cs = hs * a.n_slots + c;
        if (!a.pending[cs]) continue;
        for (int d = threadIdx.x; d < a.dim; d += blockDim.x) a.live[cs * a.dim + d] = a.shadow[cs * a.dim + d];
        __syncthreads();
        if (threadIdx.x == 0) {
            a.pending[cs] = 0;
            a.live_dirty[cs] = 1;
        }
    }
}

// ----------------------------------------------------------------------------
// host launchers
// ----------------------------------------------------------------------------
size_t select_smem_bytes(const SelectArgs& a) {
    const int S = a.parts == 0 ? 1 : a.parts;
    int table = 1;
    for (int s = 0; s < S - 1; ++s) table *= a.ks[s];
    return SelectSmem::bytes(a.n_slots, a.dim, table, S > 1 ? a.dim / S : 0, a.ks[S - 1]);
}

cudaError_t launch_similarity(const uint16_t* q, const float* cent, float* out, int bg, int G, int n_cells, int dim,
                              long long out_stride, cudaStream_t st) {
    dim3 grid((n_cells + 255) / 256, bg);
    imi_similarity_kernel<<<grid, 256, dim * sizeof(float), st>>>(q, cent, out, G, n_cells, dim, out_stride);
    return cudaGetLastError();
}

cudaError_t launch_select(const SelectArgs& a, cudaStream_t st) {
    const size_t sm = select_smem_bytes(a);
    cudaError_t e = cudaFuncSetAttribute(imi_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) return e;
    imi_select_kernel<<<a.bg, SEL_THREADS, sm, st>>>(a);
    return cudaGetLastError();
}

size_t attn_smem_bytes() { return (size_t)ATT_WARPS * ATT_STAGES * ATT_STAGE_BYTES; }

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t st) {
    const size_t sm = attn_smem_bytes();
    cudaError_t e = cudaFuncSetAttribute(imi_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) return e;
    imi_attn_kernel<<<dim3(a.splits, a.bg), ATT_WARPS * 32, sm, st>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    imi_combine_kernel<<<a.bg, 512, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_append(const AppendArgs& a, cudaStream_t st) {
    imi_append_kernel<<<a.bg, 64, 0, st>>>(a);
    return cudaGetLastError();
}

size_t async_smem_bytes(const AsyncArgs& a) {
    const int S = a.parts == 0 ? 1 : a.parts;
    int table = 1;
    for (int s = 0; s < S - 1; ++s) table *= a.ks[s];
    return sizeof(float) * ((size_t)a.batch * a.dim + (size_t)a.batch * table + 2) + 8 * a.batch + 4 * a.batch + 64;
}

cudaError_t launch_async_assign(const AsyncArgs& a, cudaStream_t st) {
    const size_t sm = async_smem_bytes(a);
    cudaError_t e = cudaFuncSetAttribute(imi_async_assign_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) return e;
    imi_async_assign_kernel<<<a.bg, 1024, sm, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_apply(const ApplyArgs& a, cudaStream_t st) {
    imi_apply_kernel<<<dim3(min(a.n_slots, 256), a.bg), 128, 0, st>>>(a);
    return cudaGetLastError();
}

}  // namespace imi
