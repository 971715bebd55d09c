// select.cu -- decode-time cell scoring and selection (sm_100a).
//
// Semantics (the reference's decode path, all on the device):
//   * cell scores: compute_impl.cu:62-103 (q_sum over the group's query heads
//     in g order, then an fma chain over d = 0..D-1 with the merged centroid);
//     evaluated separably: the chain over the first S-1 subspaces is shared by
//     every cell with the same digit prefix and the last subspace finishes it
//     per cell -- the same operations in the same order, so the same bits;
//     masked slots score -inf (retrieval.py:357);
//   * selection: top-nprobe by (score, lower slot first), keep while the
//     exclusive token prefix < max_tokens (retrieval.py:295-303), then stop
//     before the first cell whose pages ceil(size/page) push the running page
//     count above buffer_pages (wave_buffer_cpu_hotcold.cpp:320-330);
//   * execution rows: the steady zone, then the selected cells' list rows
//     (gather_copy.cu:100-213 with every page a miss), then the delta-ring rows
//     whose cell is in the kept list, or the padding id when that list holds a
//     dropped entry (async_update.py:46-76), truncated at the execution stride.
//
// Each rule is monotone in rank, so the selected set is the rank prefix that
// ends before the first element A violating a rule.  A is found by histogram
// refinement: a round histograms the candidates into 2048 buckets weighted by
// (count, pages) packed in one 64-bit word and by tokens, a block-wide
// descending scan finds the first bucket where a rule can fire, and once that
// bucket holds at most 32 elements one warp ranks them and walks the rules
// exactly.  The first round uses buckets linear in the score; the rare
// fallback refines power-of-two ranges of the 64-bit key (score bits, then the
// complement of the slot, so keys are unique).  The boundary with all three
// rules (the selected cells) and the boundary without the page rule (the kept
// list that delta rows match against) come out of the same pass.  Attention
// does not depend on row order, so the selected cells are emitted in slot
// order without a sort.
//
// The kernel sits on the decode critical path (attention waits on it), so it
// is written for latency.  A cluster of 8 CTAs serves one KV group.  Every
// CTA issues all of its global loads at once -- the subspace centroids
// (4-byte cp.async straight into a transposed shared-memory layout), its
// slice of the cell codes, masks and sizes, and the query -- and waits once.
// It then scores its slice (two to four interleaved fma chains per thread)
// and stores every key and size straight into the leader CTA's shared memory
// through DSMEM.  The first cluster barrier is split (arrive at entry, wait
// just before the first DSMEM store) so it costs nothing.  The leader alone
// runs the boundary search, ranks the selected cells by warp ballots in slot
// order, computes their row offsets with one block scan and writes the rows
// with every warp.
#include <cooperative_groups.h>

#include <type_traits>

#include "common.cuh"
#include "imi_internal.h"

namespace cg = cooperative_groups;

namespace imi {

constexpr int SL_CL = 8;                // CTAs per cluster: all score, the leader selects
constexpr int SL_THREADS = 512;
constexpr int SL_WARPS = SL_THREADS / 32;
constexpr int SL_NB = 2048;             // histogram buckets per refinement round (2^11)
constexpr int SL_NB_BITS = 11;
constexpr int SL_MAX_SLOTS = 16384;     // keys and sizes live in the leader's shared memory
constexpr int SL_CPT = SL_MAX_SLOTS / SL_CL / SL_THREADS;  // cells per thread when scoring (<= 4)
constexpr int SL_SEL_MAX = 2048;        // selected cells at most (nprobe <= 2048)

struct SelHdr {
    unsigned long long kmin, kmax;
    unsigned long long hcp[SL_NB];  // per bucket: (count << 32) | pages
    unsigned int hsz[SL_NB];        // per bucket: tokens
    unsigned long long red64[SL_WARPS];
    unsigned int red32[SL_WARPS];
    int redi[SL_WARPS];
    // boundary with all three rules
    unsigned long long bkeys[32];
    int bsz[32];
    int nb, first, bucket, bcnt;
    long long pre[3];
    unsigned long long T, flags;
    // boundary with the rank and token rules only
    unsigned long long bkeys2[32];
    int bsz2[32];
    int nb2, first2, bucket2, bcnt2;
    long long pre2[3];
    unsigned long long T2;
    int wsel[SL_WARPS], wkept[SL_WARPS];
    unsigned long long rscr[2][48];  // resolve scratch per warp: 32 keys, then 32 sizes
};

// Leading dimension of a transposed [sub][k] centroid table: odd, so that a
// warp reading one row at scattered columns spreads over the banks.
__host__ __device__ inline int sl_ld(int k) { return (k & 1) ? k + 2 : k + 1; }

IMI_DEV void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                 "l"(src)
                 : "memory");
}

// Block-wide inclusive scan of one int (all SL_THREADS threads call it).
__device__ __forceinline__ int sl_scan(int v, int* red, int* total) {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, x, o);
        if (l >= o) x += t;
    }
    if (l == 31) red[w] = x;
    __syncthreads();
    if (w == 0) {
        int y = l < SL_WARPS ? red[l] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, y, o);
            if (l >= o) y += t;
        }
        if (l < SL_WARPS) red[l] = y;
    }
    __syncthreads();
    const int base = (w > 0) ? red[w - 1] : 0;
    if (total) *total = red[SL_WARPS - 1];
    __syncthreads();
    return x + base;
}

// Block-wide inclusive scan of a (64-bit, 32-bit) pair under one set of barriers.
__device__ __forceinline__ void sl_scan_pair(unsigned long long& x, unsigned int& y, SelHdr& sm) {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long tx = __shfl_up_sync(0xffffffffu, x, o);
        const unsigned int ty = __shfl_up_sync(0xffffffffu, y, o);
        if (l >= o) {
            x += tx;
            y += ty;
        }
    }
    if (l == 31) {
        sm.red64[w] = x;
        sm.red32[w] = y;
    }
    __syncthreads();
    if (w == 0) {
        unsigned long long xx = l < SL_WARPS ? sm.red64[l] : 0ull;
        unsigned int yy = l < SL_WARPS ? sm.red32[l] : 0u;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned long long tx = __shfl_up_sync(0xffffffffu, xx, o);
            const unsigned int ty = __shfl_up_sync(0xffffffffu, yy, o);
            if (l >= o) {
                xx += tx;
                yy += ty;
            }
        }
        if (l < SL_WARPS) {
            sm.red64[l] = xx;
            sm.red32[l] = yy;
        }
    }
    __syncthreads();
    if (w > 0) {
        x += sm.red64[w - 1];
        y += sm.red32[w - 1];
    }
    __syncthreads();
}

__global__ void __cluster_dims__(SL_CL, 1, 1) __launch_bounds__(SL_THREADS, 1)
    imi_select_kernel(SelectArgs a) {
    extern __shared__ __align__(16) unsigned char dyn[];
    SelHdr& sm = *reinterpret_cast<SelHdr*>(dyn);
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = (int)cluster.block_rank();
    const int h = blockIdx.y;
    const int tid = threadIdx.x;
    const int wid = tid >> 5, lid = tid & 31;
    const int S = a.parts == 0 ? 1 : a.parts;
    const int sub = a.dim / S;
    const int sub_shift = __ffs(sub) - 1;  // sub is a power of two (128 / S)
    const int k_last = a.ks[S - 1];
    int table = 1;
    for (int s = 0; s < S - 1; ++s) table *= a.ks[s];
    const int n = a.n_slots;
    const int npad = (n + 1) & ~1;
    const bool pg_pow2 = (a.page_size & (a.page_size - 1)) == 0;
    const int pg_shift = __ffs(a.page_size) - 1;
    auto pages_of = [&](int sz) -> int {
        if (sz <= 0) return 0;
        return pg_pow2 ? (sz + a.page_size - 1) >> pg_shift : (sz + a.page_size - 1) / a.page_size;
    };

    // identical layout in every CTA (DSMEM addresses are offsets)
    unsigned char* p = dyn + ((sizeof(SelHdr) + 15) & ~size_t(15));
    unsigned long long* skey = reinterpret_cast<unsigned long long*>(p);  // [n] leader: 0 = not a candidate
    p += sizeof(unsigned long long) * npad;
    int* ssz = reinterpret_cast<int*>(p);  // [n] leader: sizes of candidates
    p += sizeof(int) * npad;
    float* qs = reinterpret_cast<float*>(p);
    p += sizeof(float) * a.dim;
    float* tab = reinterpret_cast<float*>(p);
    p += sizeof(float) * (table + 4);
    // transposed centroid tables: the last subspace [sub][ld(k_last)], then
    // the prefix subspaces back to back; the leader reuses the region for the
    // selected-cell lists once scoring is over
    float* cT = reinterpret_cast<float*>(p);
    const int ldT = sl_ld(k_last);
    float* cP = cT + (S > 1 ? sub * ldT : 0);
    int* sel_slot = reinterpret_cast<int*>(p);
    int* sel_start = sel_slot + SL_SEL_MAX;
    int* sel_off = sel_start + SL_SEL_MAX;

    const size_t hs = (size_t)h;
    auto stamp = [&](int k) {
        if (a.phase_ns && tid == 0 && rank == 0) {
            unsigned long long t;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
            a.phase_ns[hs * 8 + k] = t;
        }
    };
    stamp(0);
    // let the attention kernel that follows (a programmatic dependent launch)
    // start setting up on the SMs this kernel leaves free
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    if (rank == 0 && tid == 0) {
        sm.kmin = ~0ull;
        sm.kmax = 0ull;
    }
    // first half of the cluster barrier that guards the DSMEM stores: every
    // CTA is running and the leader's header is set
    asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory");

    const int32_t* sizes = a.cell_sizes + hs * n;
    const uint8_t* mask = a.cell_mask + hs * n;
    const int32_t* code = a.cell_code + hs * n;
    const uint8_t* dirty = a.cell_dirty ? a.cell_dirty + hs * n : nullptr;
    const float* merged = a.centroids + hs * n * (size_t)a.dim;
    const float* subc = a.sub_centroids + hs * (size_t)S * a.kmax * sub;

    // ---------------- every CTA: all global loads at once ----------------
    int poff[4] = {0, 0, 0, 0};  // offsets of the prefix tables within cP
    if (S > 1) {
        int off = 0;
        for (int s = 0; s < S - 1; ++s) {
            poff[s] = off;
            off += sub * sl_ld(a.ks[s]);
        }
        for (int s = 0; s < S; ++s) {
            const int k = a.ks[s];
            float* dst = s == S - 1 ? cT : cP + poff[s];
            const int ld = sl_ld(k);
            const float* src = subc + (size_t)s * a.kmax * sub;
            const int total = k * sub;
            for (int e = tid; e < total; e += SL_THREADS) {
                const int i = e >> sub_shift, d = e & (sub - 1);
                cp_async4(dst + d * ld + i, src + e);
            }
        }
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
    const int chunk = (n + SL_CL - 1) / SL_CL;
    const int c0 = rank * chunk;
    const int c1 = min(n, c0 + chunk);
    int ccv[SL_CPT], szv[SL_CPT];
    bool mkv[SL_CPT], dkv[SL_CPT];
#pragma unroll
    for (int j = 0; j < SL_CPT; ++j) {
        const int c = c0 + tid + j * SL_THREADS;
        const bool in = c < c1;
        ccv[j] = in ? code[c] : -1;
        mkv[j] = in ? mask[c] != 0 : true;
        szv[j] = in ? sizes[c] : 0;
        dkv[j] = in && dirty ? dirty[c] != 0 : false;
    }
    if (tid < a.dim) {
        float qv[8];
#pragma unroll
        for (int g = 0; g < 8; ++g) qv[g] = g < a.G ? bf16_bits_to_f32(a.q[(hs * a.G + g) * a.dim + tid]) : 0.0f;
        float acc = 0.0f;
        for (int g = 0; g < a.G; ++g) acc = __fadd_rn(acc, qv[g]);
        qs[tid] = acc;
    }
    asm volatile("cp.async.wait_all;\n" ::: "memory");
    __syncthreads();

    // ---------------- every CTA: prefix table over the first S-1 subspaces ----------------
    if (S > 1) {
        int width = 1;
        for (int s = 0; s < S - 1; ++s) {
            const int ks = a.ks[s];
            const float* cs = cP + poff[s];
            const int ld = sl_ld(ks);
            const int total = width * ks;
            const float* qq = qs + s * sub;
            float vals[16];
            int cnt = 0;
            for (int e = tid; e < total && cnt < 16; e += SL_THREADS, ++cnt) {
                const int pi = e / ks, i = e - pi * ks;
                float acc = s == 0 ? 0.0f : tab[pi];
#pragma unroll 8
                for (int d = 0; d < sub; ++d) acc = __fmaf_rn(qq[d], cs[d * ld + i], acc);
                vals[cnt] = acc;
            }
            if (s > 0) __syncthreads();  // every read of the previous level is done
            cnt = 0;
            for (int e = tid; e < total && cnt < 16; e += SL_THREADS, ++cnt) tab[e] = vals[cnt];
            __syncthreads();
            width = total;
        }
    }
    stamp(1);

    // ---------------- every CTA: score its slice ----------------
    const float* q2 = qs + (S - 1) * sub;
    float acc[SL_CPT];
    int il[SL_CPT];
    bool sep[SL_CPT], cand[SL_CPT];
#pragma unroll
    for (int j = 0; j < SL_CPT; ++j) {
        acc[j] = 0.0f;
        il[j] = 0;
        const int cc = ccv[j];
        cand[j] = !mkv[j] && cc >= 0;
        sep[j] = cand[j] && S > 1 && !dkv[j];
        if (sep[j]) {
            int pidx = 0;
            for (int t = 0; t < S - 1; ++t) pidx = pidx * a.ks[t] + ((cc >> (8 * t)) & 0xff);
            il[j] = (cc >> (8 * (S - 1))) & 0xff;
            acc[j] = tab[pidx];
        }
    }
    if (S > 1) {
        // interleaved chains over the last subspace; the number of live cells
        // per thread is uniform over the CTA
        // (a cell that is not separable runs the chain on column 0 and the
        // result is discarded)
        auto chains = [&](auto nj) {
            constexpr int J = decltype(nj)::value;
            float ch[J];
#pragma unroll
            for (int j = 0; j < J; ++j) ch[j] = acc[j];
            for (int d0 = 0; d0 < sub; d0 += 8) {
                float cv[8][J], qv[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    qv[u] = q2[d0 + u];
#pragma unroll
                    for (int j = 0; j < J; ++j) cv[u][j] = cT[(d0 + u) * ldT + il[j]];
                }
#pragma unroll
                for (int u = 0; u < 8; ++u)
#pragma unroll
                    for (int j = 0; j < J; ++j) ch[j] = __fmaf_rn(qv[u], cv[u][j], ch[j]);
            }
#pragma unroll
            for (int j = 0; j < J; ++j)
                if (sep[j]) acc[j] = ch[j];
        };
        const int live = (c1 - c0 + SL_THREADS - 1) / SL_THREADS;
        if (live <= 2)
            chains(std::integral_constant<int, 2>{});
        else
            chains(std::integral_constant<int, SL_CPT>{});
    }
    asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
    {
        SelHdr* lead = cluster.map_shared_rank(&sm, 0);
        unsigned long long* lkey = cluster.map_shared_rank(skey, 0);
        int* lsz = cluster.map_shared_rank(ssz, 0);
        unsigned long long kmn = ~0ull, kmx = 0ull;
#pragma unroll
        for (int j = 0; j < SL_CPT; ++j) {
            const int c = c0 + tid + j * SL_THREADS;
            if (c >= c1) continue;
            unsigned long long key = 0ull;
            float s = -INFINITY;
            if (cand[j]) {
                if (sep[j]) {
                    s = acc[j];
                } else {
                    const float* row = merged + (size_t)c * a.dim;
                    s = 0.0f;
                    for (int d = 0; d < a.dim; d += 4) {
                        const float4 v = *reinterpret_cast<const float4*>(row + d);
                        s = __fmaf_rn(qs[d], v.x, s);
                        s = __fmaf_rn(qs[d + 1], v.y, s);
                        s = __fmaf_rn(qs[d + 2], v.z, s);
                        s = __fmaf_rn(qs[d + 3], v.w, s);
                    }
                }
                key = ((unsigned long long)ord_f32(s) << 32) | (0xffffffffu - (uint32_t)c);
                kmn = min(kmn, key);
                kmx = max(kmx, key);
            }
            lkey[c] = key;
            lsz[c] = key ? szv[j] : 0;
            if (a.scores_out) a.scores_out[hs * n + c] = s;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            kmn = min(kmn, (unsigned long long)__shfl_xor_sync(0xffffffffu, kmn, o));
            kmx = max(kmx, (unsigned long long)__shfl_xor_sync(0xffffffffu, kmx, o));
        }
        if (lid == 0 && kmx != 0ull) {
            atomicMin(&lead->kmin, kmn);
            atomicMax(&lead->kmax, kmx);
        }
    }
    cluster.sync();  // every score is in the leader
    if (rank != 0) return;
    stamp(2);
    const unsigned long long key_lo0 = sm.kmin, key_hi0 = sm.kmax;
    const bool any_cand = key_hi0 != 0ull;

    // One warp resolves a boundary bucket exactly: rank its (<= 32) elements,
    // place them in rank order (lane r holds the element of rank r), scan their
    // tokens and pages, and let the first lane whose rule fires name the
    // boundary.  `scratch` holds 32 keys and 32 sizes for the warp.
    auto resolve = [&](const unsigned long long* bk, const int* bs, int m, long long xc, long long xs, long long xp,
                       bool use_pages, unsigned long long blo, unsigned long long* scratch, unsigned long long& T,
                       unsigned long long& fl) {
        const unsigned long long mk = lid < m ? bk[lid] : 0ull;
        const int msz = lid < m ? bs[lid] : 0;
        int rk = 0;
#pragma unroll 8
        for (int q = 0; q < 32; ++q) {
            const unsigned long long o = __shfl_sync(0xffffffffu, mk, q);
            rk += (q < m && o > mk) ? 1 : 0;
        }
        int* ssz2 = reinterpret_cast<int*>(scratch + 32);
        if (lid < m) {
            scratch[rk] = mk;
            ssz2[rk] = msz;
        }
        __syncwarp();
        const unsigned long long k = lid < m ? scratch[lid] : 0ull;
        const int sz = lid < m ? ssz2[lid] : 0;
        const int pg = pages_of(sz);
        int isz = sz, ipg = pg;  // inclusive scans over the ranked elements
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int ts = __shfl_up_sync(0xffffffffu, isz, o);
            const int tp = __shfl_up_sync(0xffffffffu, ipg, o);
            if (lid >= o) {
                isz += ts;
                ipg += tp;
            }
        }
        const long long bc = xc + lid, bsum = xs + (isz - sz), bpg = xp + (ipg - pg);
        const bool rc = (bc >= a.nprobe) || (bsum >= a.max_tokens);
        const bool rp = use_pages && (bpg + pg > a.buffer_pages);
        const unsigned fire = __ballot_sync(0xffffffffu, lid < m && (rc || rp));
        if (fire) {
            const int f = __ffs(fire) - 1;
            T = __shfl_sync(0xffffffffu, k, f);
            fl = __shfl_sync(0xffffffffu, rc ? 1u : 0u, f) ? 1ull : 0ull;
        } else {
            T = blo > 0 ? blo - 1 : 0ull;
            fl = 1ull;  // nothing fires here: the token rule fires just below this bucket
        }
        __syncwarp();
    };

    // Per-thread view of 4 buckets after a histogram round: thread t owns
    // buckets SL_NB-1-4t .. SL_NB-4-4t (descending), with the exclusive
    // (count, tokens, pages) prefixes of the candidates above them.
    struct Scan {
        int cv[4], sv[4], pv[4];
        long long ec, es, ep;
    };
    auto clear_hist = [&]() {
        for (int b = tid; b < SL_NB; b += SL_THREADS) {
            sm.hcp[b] = 0ull;
            sm.hsz[b] = 0u;
        }
        if (tid == 0) {
            sm.nb = sm.nb2 = 0;
            sm.first = sm.first2 = SL_NB;
        }
        __syncthreads();
    };
    auto add_hist = [&](int b, int sz) {
        atomicAdd(&sm.hcp[b], (1ull << 32) | (unsigned long long)(unsigned)pages_of(sz));
        atomicAdd(&sm.hsz[b], (unsigned)sz);
    };
    auto scan_hist = [&](long long C, long long Sz, long long Pg, Scan& sc) {
        unsigned long long cp4 = 0ull;
        unsigned int s4 = 0u;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int b = SL_NB - 1 - 4 * tid - q;
            const unsigned long long v = sm.hcp[b];
            const unsigned int w = sm.hsz[b];
            sc.cv[q] = (int)(v >> 32);
            sc.pv[q] = (int)(v & 0xffffffffull);
            sc.sv[q] = (int)w;
            cp4 += v;
            s4 += w;
        }
        unsigned long long icp = cp4;
        unsigned int is = s4;
        sl_scan_pair(icp, is, sm);
        const unsigned long long ecp = icp - cp4;
        sc.ec = C + (long long)(ecp >> 32);
        sc.ep = Pg + (long long)(ecp & 0xffffffffull);
        sc.es = Sz + (long long)(is - s4);
    };
    auto publish = [&](const Scan& sc, int fr, int& bucket, int& bcnt, long long* pre) {
        long long xc = sc.ec, xs = sc.es, xp = sc.ep;
        for (int q = 0; q < (fr & 3); ++q) {
            xc += sc.cv[q];
            xs += sc.sv[q];
            xp += sc.pv[q];
        }
        bucket = SL_NB - 1 - fr;
        bcnt = sc.cv[fr & 3];
        pre[0] = xc;
        pre[1] = xs;
        pre[2] = xp;
    };
    auto shift_of = [&](unsigned long long lo, unsigned long long hi) {
        const unsigned long long span = hi - lo;
        const int bits = span ? 64 - __clzll(span) : 0;
        return bits > SL_NB_BITS ? bits - SL_NB_BITS : 0;
    };

    // Refinement search for one boundary (the rare path: a boundary bucket with
    // more than 32 elements).  T: selected = key > T; flags = 1 when the rank or
    // token rule (not only the page rule) fires at the boundary element.
    auto search = [&](bool use_pages, unsigned long long& T_out, unsigned long long& flags_out) {
        unsigned long long lo = key_lo0, hi = key_hi0;
        long long C = 0, Sz = 0, Pg = 0;  // totals of candidates with key > hi
        while (true) {
            const int shift = shift_of(lo, hi);
            clear_hist();
            for (int c = tid; c < n; c += SL_THREADS) {
                const unsigned long long k = skey[c];
                if (k == 0ull || k < lo || k > hi) continue;
                add_hist((int)((k - lo) >> shift), ssz[c]);
            }
            __syncthreads();
            Scan sc;
            scan_hist(C, Sz, Pg, sc);
            {
                long long ec = sc.ec, es = sc.es, ep = sc.ep;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    if (sc.cv[q] > 0 && ((ec + sc.cv[q] > a.nprobe) || (es + sc.sv[q] >= a.max_tokens) ||
                                         (use_pages && ep + sc.pv[q] > a.buffer_pages))) {
                        atomicMin(&sm.first, 4 * tid + q);
                        break;
                    }
                    ec += sc.cv[q];
                    es += sc.sv[q];
                    ep += sc.pv[q];
                }
            }
            __syncthreads();
            const int fr = sm.first;
            if (fr == SL_NB) {
                T_out = lo > 0 ? lo - 1 : 0ull;  // no rule fires in [lo, hi]: all of it is selected
                flags_out = 0ull;
                __syncthreads();
                return;
            }
            if ((fr >> 2) == tid) publish(sc, fr, sm.bucket, sm.bcnt, sm.pre);
            __syncthreads();
            const int cnt = sm.bcnt;
            const long long qc = sm.pre[0], qsz = sm.pre[1], qp = sm.pre[2];
            const unsigned long long blo = lo + ((unsigned long long)sm.bucket << shift);
            const unsigned long long bend = blo + ((1ull << shift) - 1ull);
            const unsigned long long bhi = (bend < blo || bend > hi) ? hi : bend;
            if (cnt <= 32) {
                for (int c = tid; c < n; c += SL_THREADS) {
                    const unsigned long long k = skey[c];
                    if (k == 0ull || k < blo || k > bhi) continue;
                    const int at = atomicAdd(&sm.nb, 1);
                    if (at < 32) {
                        sm.bkeys[at] = k;
                        sm.bsz[at] = ssz[c];
                    }
                }
                __syncthreads();
                if (wid == 0) {
                    unsigned long long T, fl;
                    resolve(sm.bkeys, sm.bsz, min(sm.nb, 32), qc, qsz, qp, use_pages, blo, sm.rscr[0], T, fl);
                    if (lid == 0) {
                        sm.T = T;
                        sm.flags = fl;
                    }
                }
                __syncthreads();
                T_out = sm.T;
                flags_out = sm.flags;
                __syncthreads();
                return;
            }
            lo = blo;
            hi = bhi;
            C = qc;
            Sz = qsz;
            Pg = qp;
            __syncthreads();
        }
    };

    // First round for both boundaries at once (the common case resolves here):
    // A = all three rules, B = rank and token rules only (the kept list before
    // page truncation).  Returns false when a boundary bucket holds more than
    // 32 elements; the caller then refines each boundary on its own.
    auto search_both = [&](unsigned long long& TA, unsigned long long& TB) -> bool {
        // buckets linear in the score: b = floor((s - smin) * scale), monotone
        // in s; equal scores share a bucket and are ordered by the warp rank
        auto score_of = [](unsigned long long k) {
            const uint32_t o = (uint32_t)(k >> 32);
            return __uint_as_float((o & 0x80000000u) ? (o & 0x7fffffffu) : ~o);
        };
        const float smin = score_of(key_lo0), smax = score_of(key_hi0);
        const float scale = smax > smin ? (float)(SL_NB - 1) / (smax - smin) : 0.0f;
        auto bucket_of = [&](unsigned long long k) {
            const float v = (score_of(k) - smin) * scale;
            return min(SL_NB - 1, max(0, (int)v));
        };
        clear_hist();
        for (int c = tid; c < n; c += SL_THREADS) {
            const unsigned long long k = skey[c];
            if (k == 0ull) continue;
            add_hist(bucket_of(k), ssz[c]);
        }
        __syncthreads();
        Scan sc;
        scan_hist(0, 0, 0, sc);
        {
            long long ec = sc.ec, es = sc.es, ep = sc.ep;
            bool doneA = false, doneB = false;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                if (sc.cv[q] > 0) {
                    const bool rule = (ec + sc.cv[q] > a.nprobe) || (es + sc.sv[q] >= a.max_tokens);
                    if (!doneA && (rule || ep + sc.pv[q] > a.buffer_pages)) {
                        atomicMin(&sm.first, 4 * tid + q);
                        doneA = true;
                    }
                    if (!doneB && rule) {
                        atomicMin(&sm.first2, 4 * tid + q);
                        doneB = true;
                    }
                }
                ec += sc.cv[q];
                es += sc.sv[q];
                ep += sc.pv[q];
            }
        }
        __syncthreads();
        const int frA = sm.first, frB = sm.first2;
        if (frA < SL_NB && (frA >> 2) == tid) publish(sc, frA, sm.bucket, sm.bcnt, sm.pre);
        if (frB < SL_NB && (frB >> 2) == tid) publish(sc, frB, sm.bucket2, sm.bcnt2, sm.pre2);
        __syncthreads();
        const bool hasA = frA < SL_NB, hasB = frB < SL_NB;
        if ((hasA && sm.bcnt > 32) || (hasB && sm.bcnt2 > 32)) {
            __syncthreads();
            return false;
        }
        const int bA = hasA ? sm.bucket : -1, bB = hasB ? sm.bucket2 : -1;
        unsigned long long minA = ~0ull, minB = ~0ull;  // lowest key of each boundary bucket
        if (hasA || hasB) {
            for (int c = tid; c < n; c += SL_THREADS) {
                const unsigned long long k = skey[c];
                if (k == 0ull) continue;
                const int b = bucket_of(k);
                if (b == bA) {
                    const int at = atomicAdd(&sm.nb, 1);
                    if (at < 32) {
                        sm.bkeys[at] = k;
                        sm.bsz[at] = ssz[c];
                    }
                }
                if (b == bB) {
                    const int at = atomicAdd(&sm.nb2, 1);
                    if (at < 32) {
                        sm.bkeys2[at] = k;
                        sm.bsz2[at] = ssz[c];
                    }
                }
            }
        }
        __syncthreads();
        if (wid == 0) {
            unsigned long long T = ~0ull, fl = 0ull;
            if (hasA) {
                const int m = min(sm.nb, 32);
                for (int q = 0; q < m; ++q) minA = min(minA, sm.bkeys[q]);
                // "whole bucket kept" threshold = just below its lowest key
                resolve(sm.bkeys, sm.bsz, m, sm.pre[0], sm.pre[1], sm.pre[2], true, minA, sm.rscr[0], T, fl);
            } else {
                T = key_lo0 > 0 ? key_lo0 - 1 : 0ull;
            }
            if (lid == 0) sm.T = T;
        } else if (wid == 1) {
            unsigned long long T = ~0ull, fl = 0ull;
            if (hasB) {
                const int m = min(sm.nb2, 32);
                for (int q = 0; q < m; ++q) minB = min(minB, sm.bkeys2[q]);
                resolve(sm.bkeys2, sm.bsz2, m, sm.pre2[0], sm.pre2[1], sm.pre2[2], false, minB, sm.rscr[1], T, fl);
            } else {
                T = key_lo0 > 0 ? key_lo0 - 1 : 0ull;
            }
            if (lid == 0) sm.T2 = T;
        }
        __syncthreads();
        TA = sm.T;
        TB = sm.T2;
        __syncthreads();
        return true;
    };

    unsigned long long thrA = ~0ull, thrB = ~0ull;  // no candidates: nothing selected
    if (any_cand) {
        if (!search_both(thrA, thrB)) {
            unsigned long long fl;
            search(true, thrA, fl);
            if (fl) {
                thrB = thrA;
            } else {
                unsigned long long fl2;
                search(false, thrB, fl2);
            }
        }
    }
    stamp(3);

    // ---------------- leader: emission in slot order ----------------
    // warp w owns the contiguous slot range [w*R, (w+1)*R); lanes take
    // consecutive slots (conflict-free); ballots count and rank
    const int R = ((n + SL_WARPS - 1) / SL_WARPS + 31) & ~31;
    const int w0 = wid * R, w1 = min(n, w0 + R);
    {
        int wsel = 0, wkept = 0;
#pragma unroll 4
        for (int base = w0; base < w1; base += 32) {
            const int c = base + lid;
            const unsigned long long k = c < w1 ? skey[c] : 0ull;
            wsel += __popc(__ballot_sync(0xffffffffu, k != 0ull && k > thrA));
            wkept += __popc(__ballot_sync(0xffffffffu, k != 0ull && k > thrB));
        }
        if (lid == 0) {
            sm.wsel[wid] = wsel;
            sm.wkept[wid] = wkept;
        }
    }
    __syncthreads();
    int sel_base = 0, nsel = 0, nkept = 0;
#pragma unroll
    for (int q = 0; q < SL_WARPS; ++q) {
        if (q < wid) sel_base += sm.wsel[q];
        nsel += sm.wsel[q];
        nkept += sm.wkept[q];
    }
    {
        int si = sel_base;
        const unsigned lt = (1u << lid) - 1u;
#pragma unroll 4
        for (int base = w0; base < w1; base += 32) {
            const int c = base + lid;
            const unsigned long long k = c < w1 ? skey[c] : 0ull;
            const bool fin = k != 0ull && k > thrA;
            const unsigned fm = __ballot_sync(0xffffffffu, fin);
            if (fin) {
                const int my = si + __popc(fm & lt);
                if (my < a.nprobe) a.sel_cells[hs * a.nprobe + my] = c;
                if (my < SL_SEL_MAX) sel_slot[my] = c;
            }
            si += __popc(fm);
        }
    }
    __syncthreads();
    stamp(4);
    // row offsets of the selected cells (slot order) by one block scan;
    // thread t owns entries 4t .. 4t+3
    const int ns = min(nsel, SL_SEL_MAX);
    const int32_t* offs = a.cell_offsets + hs * (n + 1);
    const int static_len = a.static_len;
    int sel_rows = 0;
    {
        int szs[4], ofv[4], loc = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {  // the offset loads are in flight during the scan
            const int i = 4 * tid + q;
            const int slot = i < ns ? sel_slot[i] : 0;
            szs[q] = i < ns ? ssz[slot] : 0;
            ofv[q] = i < ns ? offs[slot] : 0;
            loc += szs[q];
        }
        int tot;
        int run = sl_scan(loc, sm.redi, &tot) - loc + static_len;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int i = 4 * tid + q;
            if (i < ns) {
                sel_start[i] = run;
                sel_off[i] = ofv[q];
            }
            run += szs[q];
        }
        sel_rows = tot;
    }
    __syncthreads();
    int32_t* rows = a.row_index + hs * (size_t)a.exec_capacity;
    for (int r = tid; r < static_len; r += SL_THREADS) rows[r] = (1 << 30) | r;
    for (int i = wid; i < ns; i += SL_WARPS) {
        const int s0 = sel_start[i], off = sel_off[i], sz = ssz[sel_slot[i]];
        for (int jj = lid; jj < sz; jj += 32)
            if (s0 + jj < a.exec_capacity) rows[s0 + jj] = off + jj;
    }
    int total = min(static_len + sel_rows, a.exec_capacity);
    if (a.delta_count) {
        const int dcount = min(a.delta_count[h], a.delta_capacity);
        const bool has_pad = nkept < a.nprobe;
        const int32_t* dids = a.delta_cell_ids + hs * a.delta_capacity;
        int appended = 0;
        for (int base = 0; base < dcount; base += SL_THREADS) {
            const int pidx = base + tid;
            int f = 0;
            if (pidx < dcount) {
                const int cid = dids[pidx];
                if (cid >= 0 && cid < n) {
                    const unsigned long long k = skey[cid];
                    f = (k != 0ull && k > thrB) ? 1 : 0;
                }
                if (cid == a.padding_id && has_pad) f = 1;
            }
            int tot;
            const int incl = sl_scan(f, sm.redi, &tot);
            if (f) {
                const int at = total + appended + incl - 1;
                if (at < a.exec_capacity) rows[at] = (2 << 30) | pidx;
            }
            appended += tot;
        }
        total = min(total + appended, a.exec_capacity);
    }
    __syncthreads();
    stamp(5);
    if (tid == 0) {
        a.sel_count[h] = min(nsel, a.nprobe);
        a.row_count[h] = total;
        if (a.kept_count) a.kept_count[h] = nkept;
    }
}

size_t select_smem_bytes(const SelectArgs& a) {
    const int S = a.parts == 0 ? 1 : a.parts;
    int table = 1;
    for (int s = 0; s < S - 1; ++s) table *= a.ks[s];
    const int sub = a.dim / S;
    size_t tables = 0;
    if (S > 1)
        for (int s = 0; s < S; ++s) tables += (size_t)sub * sl_ld(a.ks[s]) * sizeof(float);
    const size_t lists = 3 * (size_t)SL_SEL_MAX * sizeof(int);  // reused for the selected-cell lists
    const size_t region = tables > lists ? tables : lists;
    const size_t npad = ((size_t)a.n_slots + 1) & ~size_t(1);
    return ((sizeof(SelHdr) + 15) & ~size_t(15)) + 12 * npad + sizeof(float) * ((size_t)a.dim + table + 4) + region +
           16;
}

int select_max_slots() { return SL_MAX_SLOTS; }

cudaError_t launch_select(const SelectArgs& a, cudaStream_t st) {
    const size_t sm = select_smem_bytes(a);
    cudaError_t e = cudaFuncSetAttribute(imi_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) return e;
    imi_select_kernel<<<dim3(SL_CL, a.bg), SL_THREADS, sm, st>>>(a);
    return cudaGetLastError();
}

}  // namespace imi
