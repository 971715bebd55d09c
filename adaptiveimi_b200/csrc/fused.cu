// fused.cu -- one decode layer's retrieval and attention in a single launch
// (sm_100a): cell scoring, the selection, the execution-row layout and the
// split-K gather attention with its split merge.
//
// Semantics: those of the select kernel (select.cu; retrieval.py:295-303,
// wave_buffer_cpu_hotcold.cpp:303-371, async_update.py:46-76) followed by the
// attention kernel (attention.cu; weighted_flash_decoding as retrieval.py:439-447
// calls it), with one difference in order only: the selected cells, and so their
// rows, come out in rank order (descending score), the order of the
// reference's own top-k list and of its page walk, rather than slot order.
//
// Grid (clusters x 8, groups) with clusters of 8 CTAs, one CTA per SM.  Every
// cluster of a group computes the group's selection (the clusters of a group
// agree, so no CTA ever waits for another cluster), then every CTA of the group
// streams its share of the rows:
//  1. each CTA scores one eighth of the occupied slots (the separable fma chains
//     of the select kernel, bit-identical to compute_impl.cu:62-103) and sorts
//     its slice's ranking keys (bitonic, shared memory);
//  2. through distributed shared memory the sorted slices, and each slot's key,
//     size and list offset, reach the cluster's leader;
//  3. the leader merges the eight sorted slices (a merge-path tree, only the
//     first nprobe + 1 ranks), scans their tokens and pages in rank order and
//     finds the selection (all three rules) and the kept list (rank and token
//     rules); it lays the execution rows out as runs -- the steady zone, each
//     selected cell's list rows, each matching delta row -- and the cluster's
//     CTAs copy that run table;
//  4. each CTA streams its contiguous share of the group's 16-row tiles through
//     the attention loop of attention.cu (a row's source is a binary search in
//     the run table away) and writes one (m, l, o) partial; the last CTA of the
//     group (an atomic ticket) merges the partials into the output.
// The first cluster of a group writes the selection outputs; every CTA writes
// the row-list entries of its own tiles when a row list is given.  Every wait
// is a hardware cluster barrier; the split merge is a ticket, not a wait.
#include <cooperative_groups.h>

#include "attn_core.cuh"
#include "common.cuh"
#include "imi_internal.h"
#include "select_core.cuh"

namespace cg = cooperative_groups;

namespace imi {

constexpr int FC_CL = 8;                    // CTAs per cluster
constexpr int FC_THREADS = AT_WARPS * 32;   // the streaming warps do the selection too
constexpr int FC_WARPS = AT_WARPS;
constexpr int FC_CPT = 8;                   // slots per thread of a slice
constexpr int FC_SLICE_MAX = FC_THREADS * FC_CPT;  // 2048 slots per CTA, 16384 per cluster
constexpr int FC_RANKS_MAX = 2048;          // merged ranks the leader scans (nprobe + 1)

struct FusedArgs {
    SelectArgs s;
    AttnArgs a;
    AppendArgs ap;   // ap.new_keys set: the step's steady-zone append
    int runs_cap;    // run-table entries: steady zone + nprobe + delta capacity
};

struct FcHdr {
    unsigned long long red64[FC_WARPS];
    unsigned int red32[FC_WARPS];
    int redi[FC_WARPS];
    int cnt[FC_CL];        // candidates in each CTA's sorted slice (leader)
    int len1[4], len2[2];  // merge-tree level lengths (leader)
    int A, B;              // first rank out of the selection / of the kept list
    int tokA;              // tokens of the selected cells
};

struct FcLayout {
    size_t sizes, kept, lists, sortbuf, b1, qs, tab, tables, runs, total;
};

__host__ __device__ inline size_t fc_align(size_t x) { return (x + 127) & ~size_t(127); }
__host__ __device__ inline int fc_pow2(int x) {
    int p = 1;
    while (p < x) p <<= 1;
    return p;
}
__host__ __device__ inline int fc_ne(const SelectArgs& a) {
    return (a.slot_bound > 0 && a.slot_bound < a.n_slots) ? a.slot_bound : a.n_slots;
}
__host__ __device__ inline int fc_ranks(const SelectArgs& a) {
    const int ne = fc_ne(a);
    return ne < a.nprobe + 1 ? ne : a.nprobe + 1;
}

// Shared-memory regions (identical offsets in every CTA: DSMEM addresses are
// offsets).  The selection area is reused as the attention ring once the run
// table (past both) is built.
__host__ __device__ inline FcLayout fc_layout(const SelectArgs& a, int runs_cap) {
    const int S = a.parts == 0 ? 1 : a.parts;
    const int sub = a.dim / S;
    int table = 1;
    for (int s = 0; s < S - 1; ++s) table *= a.ks[s];
    const int ne = fc_ne(a);
    const int chunk = (ne + FC_CL - 1) / FC_CL;
    const int M = fc_ranks(a);
    FcLayout L;
    size_t o = fc_align(sizeof(FcHdr));
    L.sizes = o;  // [ne] leader: size by slot
    o = fc_align(o + 4 * (size_t)ne);
    L.kept = o;  // [ne / 32] leader: kept-list membership by slot
    o = fc_align(o + 4 * (((size_t)ne + 31) / 32));
    L.lists = o;  // [8 * chunk] leader: the sorted slices; later merge level 2 ([2 * M])
    const size_t nl = (size_t)FC_CL * chunk > 2 * (size_t)M ? (size_t)FC_CL * chunk : 2 * (size_t)M;
    o = fc_align(o + 8 * nl);
    L.sortbuf = o;  // [pow2(chunk)] this CTA's slice being sorted
    o = fc_align(o + 8 * (size_t)fc_pow2(chunk));
    L.b1 = o;  // [4 * M] merge level 1; later the merged ranks ([M])
    o = fc_align(o + 8 * 4 * (size_t)M);
    L.qs = o;
    o = fc_align(o + 4 * (size_t)a.dim);
    L.tab = o;
    o = fc_align(o + 4 * ((size_t)table + 4));
    L.tables = o;
    size_t tables = 0;
    if (S > 1) {
        for (int s = 0; s < S; ++s) tables += (size_t)sub * sl_ld(a.ks[s]) * sizeof(float);
        if (S > 2) tables += (256 + (size_t)a.ks[0] * a.ks[1]) * sizeof(float);
    }
    o = fc_align(o + tables);
    const size_t ring = (size_t)AT_RING_BYTES;
    L.runs = fc_align(o > ring ? o : ring);  // [4] run count and rows, then the run table
    L.total = L.runs + 16 + 4 * (2 * (size_t)runs_cap + 1);
    return L;
}

IMI_DEV void fc_stamp(const SelectArgs& a, int h, int k, bool on) {
#ifdef FC_DEBUG_STAMPS  // every rank of the first cluster: phase_ns[(h * 8 + rank) * 8 + k]
    if (a.phase_ns && threadIdx.x == 0 && blockIdx.x < FC_CL) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        a.phase_ns[((size_t)h * 8 + blockIdx.x) * 8 + k] = t;
    }
#else
    if (on) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        a.phase_ns[(size_t)h * 8 + k] = t;
    }
#endif
}

// Bitonic sort of buf[0, P) (P a power of two), descending, all threads.
// Stages whose pairs stay inside one warp's 64-element chunks sync the warp
// only.
IMI_DEV void fc_sort_desc(unsigned long long* buf, int P) {
    const int tid = threadIdx.x;
    for (int k = 2; k <= P; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            const int lj = __ffs(j) - 1;  // j is a power of two
            for (int p = tid; p < (P >> 1); p += FC_THREADS) {
                const int i = ((p >> lj) << (lj + 1)) + (p & (j - 1)), l = i + j;
                const unsigned long long x = buf[i], y = buf[l];
                const bool desc = (i & k) == 0;
                if (desc ? (x < y) : (x > y)) {
                    buf[i] = y;
                    buf[l] = x;
                }
            }
            const int nj = j > 1 ? (j >> 1) : (k << 1 <= P ? k : 0);
            if (j >= 64 || nj >= 64 || nj == 0)
                __syncthreads();
            else
                __syncwarp();
        }
    }
    __syncthreads();
}

// Output ranks [o0, o1) of the descending merge of X[0, nx) and Y[0, ny)
// (unique keys): the merge-path split of diagonal o0, then a sequential merge.
IMI_DEV void fc_merge_range(const unsigned long long* X, int nx, const unsigned long long* Y, int ny,
                            unsigned long long* out, int o0, int o1) {
    if (o0 >= o1) return;
    int lo = max(0, o0 - ny), hi = min(o0, nx);
    while (lo < hi) {  // the smallest i whose X[i] ranks after Y[o0 - 1 - i]
        const int i = (lo + hi) >> 1;
        const int j = o0 - 1 - i;
        if (j < 0 || X[i] < Y[j])
            hi = i;
        else
            lo = i + 1;
    }
    int i = lo, j = o0 - lo;
    for (int o = o0; o < o1; ++o) {
        const bool takeX = j >= ny || (i < nx && X[i] > Y[j]);
        out[o] = takeX ? X[i++] : Y[j++];
    }
}

// One level of the merge tree: `pairs` merges of (in + 2m * stride_in, len[2m])
// with (in + (2m+1) * stride_in, len[2m+1]) into out + m * stride_out, each
// keeping its first M ranks; lengths into len_out.
IMI_DEV void fc_merge_level(const unsigned long long* in, const int* len_in, int stride_in, unsigned long long* out,
                            int* len_out, int stride_out, int pairs, int M) {
    const int per = FC_THREADS / pairs;
    const int m = threadIdx.x / per, t = threadIdx.x - m * per;
    if (m < pairs) {
        const int nx = len_in[2 * m], ny = len_in[2 * m + 1];
        const int L = min(nx + ny, M);
        const int step = (L + per - 1) / per;
        fc_merge_range(in + (size_t)(2 * m) * stride_in, nx, in + (size_t)(2 * m + 1) * stride_in, ny,
                       out + (size_t)m * stride_out, min(L, t * step), min(L, (t + 1) * step));
        if (t == 0) len_out[m] = L;
    }
    __syncthreads();
}

__global__ void __cluster_dims__(FC_CL, 1, 1) __launch_bounds__(FC_THREADS, 1)
    imi_decode_fused_kernel(const __grid_constant__ FusedArgs f) {
    extern __shared__ __align__(128) unsigned char fsm[];
    const SelectArgs& a = f.s;
    const AttnArgs& at = f.a;
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int cl = blockIdx.x / FC_CL;  // this cluster among the group's clusters
    const int h = blockIdx.y;
    const int tid = threadIdx.x, wid = tid >> 5, lid = tid & 31;
    const size_t hs = (size_t)h;
    const int S = a.parts == 0 ? 1 : a.parts;
    const int sub = a.dim / S;
    const int sub_shift = __ffs(sub) - 1;
    const int k_last = a.ks[S - 1];
    const int n = a.n_slots;
    const int ne = fc_ne(a);
    const int M = fc_ranks(a);
    const FcLayout Lo = fc_layout(a, f.runs_cap);
    FcHdr& hd = *reinterpret_cast<FcHdr*>(fsm);
    int* ssz = reinterpret_cast<int*>(fsm + Lo.sizes);
    unsigned int* kept = reinterpret_cast<unsigned int*>(fsm + Lo.kept);
    unsigned long long* lists = reinterpret_cast<unsigned long long*>(fsm + Lo.lists);
    unsigned long long* sortbuf = reinterpret_cast<unsigned long long*>(fsm + Lo.sortbuf);
    unsigned long long* b1 = reinterpret_cast<unsigned long long*>(fsm + Lo.b1);
    unsigned long long* b2 = lists;  // the slices are consumed by level 1
    unsigned long long* fin = b1;    // level 1 is consumed by level 2
    float* qs = reinterpret_cast<float*>(fsm + Lo.qs);
    float* tab = reinterpret_cast<float*>(fsm + Lo.tab);
    float* cT = reinterpret_cast<float*>(fsm + Lo.tables);
    const int ldT = sl_ld(k_last);
    float* cP = cT + (S > 1 ? sub * ldT : 0);
    float* bufA = cP + (S > 1 ? prefix_table_offset(a, S - 1, sub) : 0);
    float* bufB = bufA + 256;
    // outside the ring, so other CTAs may read the leader's copy while it streams
    int* run_hdr = reinterpret_cast<int*>(fsm + Lo.runs);  // [0] runs, [1] execution rows
    int* run_start = run_hdr + 4;                          // [runs + 1] first execution row of each run
    int* run_src = run_start + f.runs_cap + 1;             // [runs] row-list entry of the run's first row
    const bool stamping = a.phase_ns != nullptr && tid == 0 && rank == 0 && cl == 0;

    fc_stamp(a, h, 0, stamping);
    // the next kernel may be scheduled once every CTA here runs; it waits for
    // this grid's completion before touching memory
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    // first half of the cluster barrier that guards the DSMEM stores
    asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory");
    const int chunk = (ne + FC_CL - 1) / FC_CL;
    const int c0 = min(ne, rank * chunk), c1 = min(ne, c0 + chunk);
    {  // warm L2 for this CTA's inputs while the previous kernel drains
        auto pf = [](const void* ptr) { asm volatile("prefetch.global.L2 [%0];" ::"l"(ptr)); };
        const size_t base = hs * n;
        for (int i = c0 + tid * 32; i < c1; i += FC_THREADS * 32) {
            pf(a.cell_code + base + i);
            pf(a.cell_sizes + base + i);
            pf(a.cell_offsets + hs * (n + 1) + i);
            if ((i & 127) == 0) pf(a.cell_mask + base + i);
        }
        if (S > 1) {
            const char* sc = reinterpret_cast<const char*>(a.sub_centroids + hs * S * a.kmax * sub);
            const size_t bytes = (size_t)S * a.kmax * sub * 4;
            for (size_t o = (size_t)tid * 128; o < bytes; o += (size_t)FC_THREADS * 128) pf(sc + o);
        }
        if (tid < (a.G * a.dim * 2 + 127) / 128)
            pf(reinterpret_cast<const char*>(a.q + hs * a.G * a.dim) + tid * 128);
    }
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    if (f.ap.new_keys && cl == 0 && rank == FC_CL - 1 && wid < 2) append_group(f.ap, h, wid, lid);

    // ---------------- 1. score this CTA's slice ----------------
    const int32_t* sizes = a.cell_sizes + hs * n;
    const uint8_t* mask = a.cell_mask + hs * n;
    const int32_t* code = a.cell_code + hs * n;
    const int32_t* offs = a.cell_offsets + hs * (n + 1);
    const uint8_t* dirty = a.cell_dirty ? a.cell_dirty + hs * n : nullptr;
    const float* merged = a.centroids + hs * n * (size_t)a.dim;
    const float* subc = a.sub_centroids + hs * (size_t)S * a.kmax * sub;
    if (S > 1) {
        for (int s = 0; s < S; ++s) {
            const int k = a.ks[s];
            float* dst = s == S - 1 ? cT : cP + prefix_table_offset(a, s, sub);
            const int ld = sl_ld(k);
            const float* src = subc + (size_t)s * a.kmax * sub;
            for (int e = tid; e < k * sub; e += FC_THREADS) cp_async4(dst + (e & (sub - 1)) * ld + (e >> sub_shift), src + e);
        }
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
    int ccv[FC_CPT], szv[FC_CPT];
    bool mkv[FC_CPT], dkv[FC_CPT];
#pragma unroll
    for (int j = 0; j < FC_CPT; ++j) {
        const int c = c0 + tid + j * FC_THREADS;
        const bool in = c < c1;
        ccv[j] = in ? code[c] : -1;
        mkv[j] = in ? mask[c] != 0 : true;
        szv[j] = in ? sizes[c] : 0;
        dkv[j] = in && dirty ? dirty[c] != 0 : false;
    }
    if (tid < a.dim) {
        float acc = 0.0f;
        for (int g = 0; g < a.G; ++g) acc = __fadd_rn(acc, bf16_bits_to_f32(a.q[(hs * a.G + g) * a.dim + tid]));
        qs[tid] = acc;
    }
    asm volatile("cp.async.wait_all;\n" ::: "memory");
    __syncthreads();
    fc_stamp(a, h, 1, stamping);
    if (S > 1) {  // prefix table over the first S-1 subspaces (level s chains subspace s onto level s-1)
        int width = 1;
        for (int s = 0; s < S - 1; ++s) {
            const int ks = a.ks[s], ld = sl_ld(ks);
            const int total = width * ks;
            const float* cs = cP + prefix_table_offset(a, s, sub);
            const float* src = s == 0 ? nullptr : (((s - 1) & 1) ? bufB : bufA);
            float* dst = s == S - 2 ? tab : ((s & 1) ? bufB : bufA);
            const float* qq = qs + s * sub;
            for (int e = tid; e < total; e += FC_THREADS) {
                const int pi = e / ks, i = e - pi * ks;
                float acc = src ? src[pi] : 0.0f;
#pragma unroll 8
                for (int d = 0; d < sub; ++d) acc = __fmaf_rn(qq[d], cs[d * ld + i], acc);
                dst[e] = acc;
            }
            __syncthreads();
            width = total;
        }
    }
    unsigned long long kv[FC_CPT];
    {
        float acc[FC_CPT];
        int il[FC_CPT];
        bool sep[FC_CPT];
#pragma unroll
        for (int j = 0; j < FC_CPT; ++j) {
            acc[j] = 0.0f;
            il[j] = 0;
            const int cc = ccv[j];
            const bool cand = !mkv[j] && cc >= 0;
            sep[j] = cand && S > 1 && !dkv[j];
            if (sep[j]) {
                int pidx = 0;
                for (int t = 0; t < S - 1; ++t) pidx = pidx * a.ks[t] + ((cc >> (8 * t)) & 0xff);
                il[j] = (cc >> (8 * (S - 1))) & 0xff;
                acc[j] = tab[pidx];
            }
            kv[j] = cand ? 1ull : 0ull;  // candidate flag until the score is in
        }
        if (S > 1) {  // the last subspace's chain, several cells per thread interleaved
            const float* q2 = qs + (S - 1) * sub;
            float ch[FC_CPT];
#pragma unroll
            for (int j = 0; j < FC_CPT; ++j) ch[j] = acc[j];
            const int live = (c1 - c0 + FC_THREADS - 1) / FC_THREADS;  // uniform over the CTA
            for (int d0 = 0; d0 < sub; d0 += 4) {
                float qv[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) qv[u] = q2[d0 + u];
#pragma unroll
                for (int j = 0; j < FC_CPT; ++j) {
                    if (j < live) {
#pragma unroll
                        for (int u = 0; u < 4; ++u) ch[j] = __fmaf_rn(qv[u], cT[(d0 + u) * ldT + il[j]], ch[j]);
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < FC_CPT; ++j)
                if (sep[j]) acc[j] = ch[j];
        }
#pragma unroll
        for (int j = 0; j < FC_CPT; ++j) {
            const int c = c0 + tid + j * FC_THREADS;
            float sc = -INFINITY;
            if (kv[j]) {
                if (sep[j]) {
                    sc = acc[j];
                } else {  // an updated (or IVF) centroid: the chain over the live merged row
                    const float* row = merged + (size_t)c * a.dim;
                    sc = 0.0f;
                    for (int d = 0; d < a.dim; d += 4) {
                        const float4 v = *reinterpret_cast<const float4*>(row + d);
                        sc = __fmaf_rn(qs[d], v.x, sc);
                        sc = __fmaf_rn(qs[d + 1], v.y, sc);
                        sc = __fmaf_rn(qs[d + 2], v.z, sc);
                        sc = __fmaf_rn(qs[d + 3], v.w, sc);
                    }
                }
                kv[j] = ((unsigned long long)ord_f32(sc) << 32) | (0xffffffffu - (uint32_t)c);
            }
            if (a.scores_out && cl == 0 && c < c1) a.scores_out[hs * n + c] = sc;
        }
    }
    if (a.scores_out && cl == 0)
        for (int c = ne + rank * FC_THREADS + tid; c < n; c += FC_CL * FC_THREADS) a.scores_out[hs * n + c] = -INFINITY;

    // ---------------- 2. sort the slice; everything to the leader ----------------
    fc_stamp(a, h, 5, stamping);
    const int P = fc_pow2(max(chunk, 2));
#pragma unroll
    for (int j = 0; j < FC_CPT; ++j) {
        const int i = tid + j * FC_THREADS;
        if (i < P) sortbuf[i] = (c0 + i < c1) ? kv[j] : 0ull;
    }
    for (int i = tid + FC_CPT * FC_THREADS; i < P; i += FC_THREADS) sortbuf[i] = 0ull;
    __syncthreads();
    fc_sort_desc(sortbuf, P);
    int ncand = 0;  // the slice's candidates: they sort first (non-candidates are 0)
    {
        int mine = 0;
#pragma unroll
        for (int j = 0; j < FC_CPT; ++j) mine += kv[j] != 0ull ? 1 : 0;
        sl_scan<FC_THREADS>(mine, hd.redi, &ncand);
    }
    fc_stamp(a, h, 2, stamping);
    asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
#ifdef FC_DEBUG_STAMPS
    fc_stamp(a, h, 3, false);
#endif
    {
        FcHdr* lead = cluster.map_shared_rank(&hd, 0);
        int* lsz = cluster.map_shared_rank(ssz, 0);
        unsigned long long* llist = cluster.map_shared_rank(lists, 0) + (size_t)rank * chunk;
        for (int i = tid; i < ncand; i += FC_THREADS) llist[i] = sortbuf[i];
#pragma unroll
        for (int j = 0; j < FC_CPT; ++j) {
            const int c = c0 + tid + j * FC_THREADS;
            if (c < c1) lsz[c] = kv[j] ? szv[j] : 0;
        }
        if (tid == 0) lead->cnt[rank] = ncand;
    }
#ifdef FC_DEBUG_STAMPS
    fc_stamp(a, h, 4, false);
#endif
    cluster.sync();  // every slice is in the leader
#ifdef FC_DEBUG_STAMPS
    fc_stamp(a, h, 5, false);
#endif

    // ---------------- 3. the leader: merge, scan, runs ----------------
    const int static_len = a.static_len;
    const int base_run = static_len > 0 ? 1 : 0;
    if (rank == 0) {
#ifndef FC_DEBUG_STAMPS
        fc_stamp(a, h, 3, stamping);
#endif
        fc_merge_level(lists, hd.cnt, chunk, b1, hd.len1, M, 4, M);
        fc_merge_level(b1, hd.len1, M, b2, hd.len2, M, 2, M);
        fc_merge_level(b2, hd.len2, M, fin, &hd.A, 0, 1, M);  // hd.A temporarily holds the merged length
        const int Mt = hd.A;
        SelRules r;
        r.nprobe = a.nprobe;
        r.max_tokens = a.max_tokens;
        r.buffer_pages = a.buffer_pages;
        r.page_size = a.page_size;
        r.pg_shift = __ffs(a.page_size) - 1;
        r.pg_pow2 = (a.page_size & (a.page_size - 1)) == 0;
        // ranks [tid * E, tid * E + E): tokens and pages, then one scan
        const int E = (Mt + FC_THREADS - 1) / FC_THREADS;
        const int r0 = min(Mt, tid * E), r1 = min(Mt, r0 + E);
        unsigned int tk = 0;
        unsigned long long pg = 0;
        for (int i = r0; i < r1; ++i) {
            const int slot = (int)(0xffffffffu - (uint32_t)fin[i]);
            const int z = ssz[slot];
            tk += (unsigned)z;
            pg += (unsigned long long)sl_pages(z, r);
        }
        unsigned long long xp = pg;
        unsigned int yt = tk;
        __syncthreads();  // hd.A is read by every thread above before it is reset
        if (tid == 0) {
            hd.A = Mt;
            hd.B = Mt;
        }
        sl_scan_pair<FC_THREADS>(xp, yt, hd);
        long long tok_b = (long long)(yt - tk), pg_b = (long long)(xp - pg);
        for (int i = r0; i < r1; ++i) {  // the first rank where a rule fires
            const int slot = (int)(0xffffffffu - (uint32_t)fin[i]);
            const int z = ssz[slot];
            const int pz = sl_pages(z, r);
            const bool rc = (i >= r.nprobe) || (tok_b >= r.max_tokens);
            const bool rp = pg_b + pz > r.buffer_pages;
            if (rc || rp) atomicMin(&hd.A, i);
            if (rc) atomicMin(&hd.B, i);
            tok_b += z;
            pg_b += pz;
        }
        for (int w = tid; w < (ne + 31) / 32; w += FC_THREADS) kept[w] = 0u;
        __syncthreads();
        const int A = hd.A, B = hd.B;
        for (int i = r0; i < min(r1, B); ++i) {  // kept-list membership by slot (delta rows)
            const int slot = (int)(0xffffffffu - (uint32_t)fin[i]);
            atomicOr(&kept[slot >> 5], 1u << (slot & 31));
        }
        // the selected cells' runs (rank order) and the selection outputs
        tok_b = (long long)(yt - tk);
        for (int i = r0; i < r1; ++i) {
            const int slot = (int)(0xffffffffu - (uint32_t)fin[i]);
            const int z = ssz[slot];
            if (i < A) {
                run_start[base_run + i] = static_len + (int)tok_b;
                run_src[base_run + i] = __ldg(offs + slot);
                if (cl == 0) a.sel_cells[hs * a.nprobe + i] = slot;
            }
            if (i == A) hd.tokA = (int)tok_b;
            tok_b += z;
        }
        if (A == Mt && r1 == Mt && r0 < r1) hd.tokA = (int)tok_b;  // everything selected
        if (Mt == 0 && tid == 0) hd.tokA = 0;
        if (tid == 0 && static_len > 0) {
            run_start[0] = 0;
            run_src[0] = 1 << 30;
        }
        __syncthreads();
        const int sel_rows = hd.tokA;
        // delta rows whose cell is in the kept list (or the padding id when that
        // list holds a dropped entry), in ring order, after the cells
        const int dcount = a.delta_count ? min(a.delta_count[h], a.delta_capacity) : 0;
        int appended = 0;
        const int rd = base_run + A;
        if (dcount > 0) {
            const int32_t* dids = a.delta_cell_ids + hs * a.delta_capacity;
            const bool has_pad = B < a.nprobe;
            for (int base = 0; base < dcount; base += FC_THREADS) {
                const int pidx = base + tid;
                int fl = 0;
                if (pidx < dcount) {
                    const int cid = dids[pidx];
                    if (cid >= 0 && cid < ne) fl = (kept[cid >> 5] >> (cid & 31)) & 1u;
                    if (cid == a.padding_id && has_pad) fl = 1;
                }
                int tot;
                const int incl = sl_scan<FC_THREADS>(fl, hd.redi, &tot);
                if (fl) {
                    const int q = appended + incl - 1;
                    run_start[rd + q] = static_len + sel_rows + q;
                    run_src[rd + q] = (2 << 30) | pidx;
                }
                appended += tot;
            }
        }
        if (tid == 0) {
            const int total = min(static_len + sel_rows + appended, a.exec_capacity);
            run_hdr[0] = rd + appended;
            run_hdr[1] = total;
            run_start[rd + appended] = static_len + sel_rows + appended;
            if (cl == 0) {
                a.sel_count[h] = A;
                if (a.row_count) a.row_count[h] = total;
                if (a.kept_count) a.kept_count[h] = B;
            }
        }
#ifndef FC_DEBUG_STAMPS
        fc_stamp(a, h, 4, stamping);
#endif
    }
    cluster.sync();  // the leader's run table is complete
    int nruns, rows_total;
    {
        const int* lh = cluster.map_shared_rank(run_hdr, 0);
        nruns = lh[0];
        rows_total = lh[1];
        if (rank != 0) {
            const int* ls = cluster.map_shared_rank(run_start, 0);
            const int* lr = cluster.map_shared_rank(run_src, 0);
            for (int i = tid; i <= nruns; i += FC_THREADS) run_start[i] = ls[i];
            for (int i = tid; i < nruns; i += FC_THREADS) run_src[i] = lr[i];
        }
    }
    // nothing reads the leader's shared memory after this point; the matching
    // wait is just before the CTA exits
    asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory");
    __syncthreads();  // the local run table is complete; the selection area becomes the ring
    fc_stamp(a, h, 7, stamping);

    // ---------------- 4. attention over this CTA's tiles ----------------
    const int J = gridDim.x, split = blockIdx.x;
    const int gtiles = (rows_total + AT_TILE - 1) / AT_TILE;
    const int per = (gtiles + J - 1) / J;
    const int ct0 = min(gtiles, split * per), ct1 = min(gtiles, ct0 + per);
    int32_t* rlist = a.row_index ? a.row_index + hs * (size_t)a.exec_capacity : nullptr;
    uint32_t qa[8][2];
    attn_load_q(at, h, lid, qa);
    float m_run = -INFINITY, l_run = 0.0f;
    float o[16][4];
#pragma unroll
    for (int u = 0; u < 16; ++u) o[u][0] = o[u][1] = o[u][2] = o[u][3] = 0.0f;
    auto entry = [&](int t) -> int {
        const int rr = t * AT_TILE + (lid & 15);
        if (t >= ct1 || rr >= rows_total) return -1;
        int lo = 0, hi = nruns;  // the last run whose start is <= rr
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (run_start[mid] <= rr)
                lo = mid;
            else
                hi = mid;
        }
        const int e = run_src[lo] + (rr - run_start[lo]);
        if (rlist && lid < 16) rlist[rr] = e;
        return e;
    };
    attn_stream(at, h, wid, lid, smem_u32(fsm), ct0, ct1, rows_total, qa, entry, m_run, l_run, o);
    fc_stamp(a, h, 6, stamping);
    attn_write_partial(at, h, split, fsm, m_run, l_run, o);
    attn_ticket_merge(at, h, fsm);
    asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}

int fused_runs_cap(const SelectArgs& s) { return 1 + s.nprobe + (s.delta_count ? s.delta_capacity : 0); }

size_t fused_smem_bytes(const SelectArgs& s) { return fc_layout(s, fused_runs_cap(s)).total; }

// Whether this layer can run as one fused launch: the selection's shared
// memory and the run table fit next to the attention ring, the slices and
// ranks fit the leader's buffers, and the attention splits are whole clusters.
bool fused_eligible(const SelectArgs& s, const AttnArgs& a, const char** why) {
    if (s.cand_out || s.key_base != 0 || a.o_part || a.ml_part || !a.counters)
        return (*why = "sequence-sharding outputs or no merge counters"), false;
    if (a.splits % FC_CL != 0) return (*why = "splits not a multiple of 8"), false;
    if ((fc_ne(s) + FC_CL - 1) / FC_CL > FC_SLICE_MAX) return (*why = "too many slots"), false;
    if (fc_ranks(s) > FC_RANKS_MAX) return (*why = "nprobe too large"), false;
    if (fused_smem_bytes(s) > 227 * 1024) return (*why = "selection too large for one CTA"), false;
    return true;
}

cudaError_t launch_decode_fused(const SelectArgs& s, const AttnArgs& a, cudaStream_t st, const AppendArgs* app) {
    FusedArgs f{};
    f.s = s;
    f.a = a;
    if (app) f.ap = *app;
    f.runs_cap = fused_runs_cap(s);
    const size_t sm = fc_layout(s, f.runs_cap).total;
    static int smem_set[64] = {};
    cudaError_t e = ensure_smem(reinterpret_cast<const void*>(&imi_decode_fused_kernel), sm, smem_set, 64);
    if (e != cudaSuccess) return e;
    return launch_pdl(imi_decode_fused_kernel, dim3(a.splits, a.bg), dim3(FC_THREADS), sm, st, f);
}

}  // namespace imi
