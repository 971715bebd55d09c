// select_core.cuh -- the selection machinery of the cluster select kernel and
// the sequence-sharded merge (select.cu), kept apart from them: the ranking key,
// the block-wide scans, the two-boundary histogram search over the candidates
// (all three rules: rank, tokens and pages; and rank and tokens only), the
// exact resolve of a boundary bucket, and the separable scorer's helpers.
// The rules are those of retrieval.py:295-303 (top-nprobe, token budget) and
// wave_buffer_cpu_hotcold.cpp:320-330 (page budget); see select.cu.
#pragma once
#include "common.cuh"
#include "imi_internal.h"

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
    unsigned long long rmin[SL_CL], rmax[SL_CL];  // per-rank candidate key range (DSMEM stores)
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
    unsigned long long T2, flags2;
    int wsel[SL_WARPS], wkept[SL_WARPS];
    // cluster-wide emission: the thresholds (leader -> every CTA), then each
    // CTA's selected / kept counts, selected rows and stop-marker candidate
    unsigned long long cthrA, cthrB;
    int pc_sel[SL_CL], pc_rows[SL_CL], pc_kept[SL_CL];
    unsigned long long pc_nx[SL_CL];
    unsigned long long rscr[2][48];  // resolve scratch per warp: 32 keys, then 32 sizes
};

// Leading dimension of a transposed [sub][k] centroid table: odd, so that a
// warp reading one row at scattered columns spreads over the banks.
__host__ __device__ inline int sl_ld(int k) { return (k & 1) ? k + 2 : k + 1; }

struct SelRules {
    int nprobe, max_tokens, buffer_pages, page_size, pg_shift, pg_pow2;
};

IMI_DEV int sl_pages(int sz, const SelRules& r) {
    if (sz <= 0) return 0;
    return r.pg_pow2 ? (sz + r.page_size - 1) >> r.pg_shift : (sz + r.page_size - 1) / r.page_size;
}

IMI_DEV float sl_key_score(unsigned long long k) {
    const uint32_t o = (uint32_t)(k >> 32);
    return __uint_as_float((o & 0x80000000u) ? (o & 0x7fffffffu) : ~o);
}

IMI_DEV void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                 "l"(src)
                 : "memory");
}

// Block-wide inclusive scan of one int (all NT threads call it).
template <int NT = SL_THREADS>
IMI_DEV int sl_scan(int v, int* red, int* total) {
    constexpr int NW = NT / 32;
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
        int y = l < NW ? red[l] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, y, o);
            if (l >= o) y += t;
        }
        if (l < NW) red[l] = y;
    }
    __syncthreads();
    const int base = (w > 0) ? red[w - 1] : 0;
    if (total) *total = red[NW - 1];
    __syncthreads();
    return x + base;
}

// Block-wide inclusive scan of a (64-bit, 32-bit) pair under one set of barriers.
template <int NT = SL_THREADS, class Hdr>
IMI_DEV void sl_scan_pair(unsigned long long& x, unsigned int& y, Hdr& sm) {
    constexpr int NW = NT / 32;
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
        unsigned long long xx = l < NW ? sm.red64[l] : 0ull;
        unsigned int yy = l < NW ? sm.red32[l] : 0u;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned long long tx = __shfl_up_sync(0xffffffffu, xx, o);
            const unsigned int ty = __shfl_up_sync(0xffffffffu, yy, o);
            if (l >= o) {
                xx += tx;
                yy += ty;
            }
        }
        if (l < NW) {
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

// ---------------------------------------------------------------------------
// histogram rounds (leader, all threads)
// ---------------------------------------------------------------------------
template <int NT = SL_THREADS>
IMI_DEV void hist_clear(SelHdr& sm) {
    for (int b = threadIdx.x; b < SL_NB; b += NT) {
        sm.hcp[b] = 0ull;
        sm.hsz[b] = 0u;
    }
    if (threadIdx.x == 0) {
        sm.nb = sm.nb2 = 0;
        sm.first = sm.first2 = SL_NB;
    }
    __syncthreads();
}

IMI_DEV void hist_add(SelHdr& sm, int b, int sz, const SelRules& r) {
    atomicAdd(&sm.hcp[b], (1ull << 32) | (unsigned long long)(unsigned)sl_pages(sz, r));
    atomicAdd(&sm.hsz[b], (unsigned)sz);
}

// Thread t's view of buckets SL_NB-1-4t .. SL_NB-4-4t (descending) with the
// exclusive (count, tokens, pages) prefixes of the candidates above them.
struct BucketView {  // BPT = SL_NB / threads buckets per thread (<= 8)
    int cv[8], sv[8], pv[8];
    long long ec, es, ep;
};

template <int NT = SL_THREADS>
IMI_DEV void hist_view(SelHdr& sm, long long C, long long Sz, long long Pg, BucketView& v) {
    constexpr int BPT = SL_NB / NT;
    unsigned long long cp4 = 0ull;
    unsigned int s4 = 0u;
#pragma unroll
    for (int q = 0; q < BPT; ++q) {
        const int b = SL_NB - 1 - BPT * (int)threadIdx.x - q;
        const unsigned long long x = sm.hcp[b];
        const unsigned int w = sm.hsz[b];
        v.cv[q] = (int)(x >> 32);
        v.pv[q] = (int)(x & 0xffffffffull);
        v.sv[q] = (int)w;
        cp4 += x;
        s4 += w;
    }
    unsigned long long icp = cp4;
    unsigned int is = s4;
    sl_scan_pair<NT>(icp, is, sm);
    const unsigned long long ecp = icp - cp4;
    v.ec = C + (long long)(ecp >> 32);
    v.ep = Pg + (long long)(ecp & 0xffffffffull);
    v.es = Sz + (long long)(is - s4);
}

// The owner of bucket index fr (descending order) records the bucket, its
// count and the exclusive prefixes at its start.
template <int NT = SL_THREADS>
IMI_DEV void view_publish(const BucketView& v, int fr, int* bucket, int* bcnt, long long* pre) {
    constexpr int BPT = SL_NB / NT;
    const int q0 = fr % BPT;
    long long xc = v.ec, xs = v.es, xp = v.ep;
    int cnt = 0;
#pragma unroll
    for (int q = 0; q < BPT; ++q) {
        if (q < q0) {
            xc += v.cv[q];
            xs += v.sv[q];
            xp += v.pv[q];
        }
        if (q == q0) cnt = v.cv[q];
    }
    *bucket = SL_NB - 1 - fr;
    *bcnt = cnt;
    pre[0] = xc;
    pre[1] = xs;
    pre[2] = xp;
}

// One warp resolves a boundary bucket exactly: rank its (<= 32) elements,
// place them in rank order (lane r holds the element of rank r), scan their
// tokens and pages, and let the first lane whose rule fires name the
// boundary.  T: selected = key > T; fl = 1 when the rank or token rule (not
// only the page rule) fires.  Lane 0 writes *T_out / *fl_out.
static __device__ __noinline__ void resolve_boundary(const unsigned long long* bk, const int* bs, int m, long long xc,
                                              long long xs, long long xp, int use_pages, unsigned long long blo,
                                              unsigned long long* scratch, SelRules r, unsigned long long* T_out,
                                              unsigned long long* fl_out) {
    const int lid = threadIdx.x & 31;
    const unsigned long long mk = lid < m ? bk[lid] : 0ull;
    const int msz = lid < m ? bs[lid] : 0;
    int rk = 0;
    for (int q = 0; q < m; ++q) rk += (__shfl_sync(0xffffffffu, mk, q) > mk) ? 1 : 0;
    int* ssz2 = reinterpret_cast<int*>(scratch + 32);
    if (lid < m) {
        scratch[rk] = mk;
        ssz2[rk] = msz;
    }
    __syncwarp();
    const unsigned long long k = lid < m ? scratch[lid] : 0ull;
    const int sz = lid < m ? ssz2[lid] : 0;
    const int pg = sl_pages(sz, r);
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
    const bool rc = (bc >= r.nprobe) || (bsum >= r.max_tokens);
    const bool rp = use_pages && (bpg + pg > r.buffer_pages);
    const unsigned fire = __ballot_sync(0xffffffffu, lid < m && (rc || rp));
    unsigned long long T, fl;
    if (fire) {
        const int f = __ffs(fire) - 1;
        T = __shfl_sync(0xffffffffu, k, f);
        fl = __shfl_sync(0xffffffffu, rc ? 1u : 0u, f) ? 1ull : 0ull;
    } else {
        T = blo > 0 ? blo - 1 : 0ull;
        fl = 1ull;  // nothing fires here: the token rule fires just below this bucket
    }
    if (lid == 0) {
        *T_out = T;
        *fl_out = fl;
    }
    __syncwarp();
}

// The candidates a boundary search walks: candidate c (0 <= c < ne) has key
// key(c) (0: not a candidate) and size size(c).  DenseKeys: arrays (shared
// memory).  RecordKeys: the shards' candidate records in global memory, as
// the sequence-sharded merge receives them (candidate s * cap + j is entry j
// of shard s's record; entries at or past the record's count are not
// candidates).
struct DenseKeys {
    static constexpr int kBatch = 1;  // shared memory: no latency to hide
    const unsigned long long* k;
    const int* s;
    IMI_DEV unsigned long long key(int c) const { return k[c]; }
    IMI_DEV int size(int c) const { return s[c]; }
};
struct RecordKeys {
    static constexpr int kBatch = 1;  // (eight in flight measured slower on the 1M merge)
    const unsigned long long* cand;  // shard s's record of this group at cand + s * shard_stride
    size_t shard_stride;
    int cap;
    const int* counts;  // [shards] record counts (shared memory)
    IMI_DEV unsigned long long key(int c) const {
        const int sh = c / cap, j = c - sh * cap;
        return j < counts[sh] ? __ldcg(cand + sh * shard_stride + j) : 0ull;
    }
    IMI_DEV int size(int c) const {
        const int sh = c / cap, j = c - sh * cap;
        return (int)__ldcg(cand + sh * shard_stride + cap + j);
    }
};

// Visit the candidates [0, ne) in batches of Keys::kBatch per thread: the
// keys and sizes of a batch are loaded before f runs on any of them, so
// passes over candidates in global memory keep that many loads in flight
// instead of waiting for each one behind the shared-memory atomics.
template <int NT = SL_THREADS, class Keys, class F>
IMI_DEV void for_candidates(const Keys& keys, int ne, F&& f) {
    constexpr int SL_BATCH = Keys::kBatch;
    for (int c0 = threadIdx.x; c0 < ne; c0 += SL_BATCH * NT) {
        unsigned long long k[SL_BATCH];
        int z[SL_BATCH];
#pragma unroll
        for (int u = 0; u < SL_BATCH; ++u) {
            const int c = c0 + u * NT;
            k[u] = c < ne ? keys.key(c) : 0ull;
        }
#pragma unroll
        for (int u = 0; u < SL_BATCH; ++u) {  // unconditional: one round of loads, not two
            const int c = c0 + u * NT;
            z[u] = c < ne ? keys.size(c) : 0;
        }
#pragma unroll
        for (int u = 0; u < SL_BATCH; ++u)
            if (k[u]) f(k[u], z[u]);
    }
}

// Refinement search for one boundary over power-of-two key ranges (the rare
// path: a first-round boundary bucket with more than 32 elements).  All
// threads call it; the result is left in sm.T / sm.flags.
template <int NT = SL_THREADS, class Keys>
__device__ __noinline__ void search_one(SelHdr& sm, const Keys& keys, int ne,
                                        unsigned long long lo, unsigned long long hi, int use_pages, SelRules r,
                                        long long C0 = 0, long long S0 = 0, long long P0 = 0) {
    constexpr int BPT = SL_NB / NT;
    const int tid = threadIdx.x;
    long long C = C0, Sz = S0, Pg = P0;  // totals of candidates with key > hi (some may lie outside `keys`)
    while (true) {
        const unsigned long long span = hi - lo;
        const int bits = span ? 64 - __clzll(span) : 0;
        const int shift = bits > SL_NB_BITS ? bits - SL_NB_BITS : 0;
        hist_clear<NT>(sm);
        for_candidates<NT>(keys, ne, [&](unsigned long long k, int z) {
            if (k >= lo && k <= hi) hist_add(sm, (int)((k - lo) >> shift), z, r);
        });
        __syncthreads();
        BucketView v;
        hist_view<NT>(sm, C, Sz, Pg, v);
        {
            long long ec = v.ec, es = v.es, ep = v.ep;
            bool done = false;
#pragma unroll
            for (int q = 0; q < BPT; ++q) {
                if (!done && v.cv[q] > 0 &&
                    ((ec + v.cv[q] > r.nprobe) || (es + v.sv[q] >= r.max_tokens) ||
                     (use_pages && ep + v.pv[q] > r.buffer_pages))) {
                    atomicMin(&sm.first, BPT * tid + q);
                    done = true;
                }
                ec += v.cv[q];
                es += v.sv[q];
                ep += v.pv[q];
            }
        }
        __syncthreads();
        const int fr = sm.first;
        if (fr == SL_NB) {
            if (tid == 0) {
                sm.T = lo > 0 ? lo - 1 : 0ull;  // no rule fires in [lo, hi]: all of it is selected
                sm.flags = 0ull;
            }
            __syncthreads();
            return;
        }
        if (fr / BPT == tid) view_publish<NT>(v, fr, &sm.bucket, &sm.bcnt, sm.pre);
        __syncthreads();
        const int cnt = sm.bcnt;
        const long long qc = sm.pre[0], qsz = sm.pre[1], qp = sm.pre[2];
        const unsigned long long blo = lo + ((unsigned long long)sm.bucket << shift);
        const unsigned long long bend = blo + ((1ull << shift) - 1ull);
        const unsigned long long bhi = (bend < blo || bend > hi) ? hi : bend;
        if (cnt <= 32) {
            for_candidates<NT>(keys, ne, [&](unsigned long long k, int z) {
                if (k < blo || k > bhi) return;
                const int at = atomicAdd(&sm.nb, 1);
                if (at < 32) {
                    sm.bkeys[at] = k;
                    sm.bsz[at] = z;
                }
            });
            __syncthreads();
            if ((tid >> 5) == 0)
                resolve_boundary(sm.bkeys, sm.bsz, min(sm.nb, 32), qc, qsz, qp, use_pages, blo, sm.rscr[0], r,
                                 &sm.T, &sm.flags);
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
}

// First round for both boundaries at once (the common case resolves here):
// A = all three rules, B = rank and token rules only (the kept list before page
// truncation), over buckets linear in the score (equal scores share a bucket
// and are ordered by the warp rank).  Returns false when a boundary bucket
// holds more than 32 elements.  Results in sm.T / sm.T2.
template <int NT = SL_THREADS, class Keys>
IMI_DEV bool search_both(SelHdr& sm, const Keys& keys, int ne,
                         unsigned long long key_lo0, unsigned long long key_hi0, const SelRules& r) {
    constexpr int BPT = SL_NB / NT;
    const int tid = threadIdx.x, wid = tid >> 5;
    const float smin = sl_key_score(key_lo0), smax = sl_key_score(key_hi0);
    const float scale = smax > smin ? (float)(SL_NB - 1) / (smax - smin) : 0.0f;
    hist_clear<NT>(sm);
    for_candidates<NT>(keys, ne, [&](unsigned long long k, int z) {
        hist_add(sm, min(SL_NB - 1, max(0, (int)((sl_key_score(k) - smin) * scale))), z, r);
    });
    __syncthreads();
    BucketView v;
    hist_view<NT>(sm, 0, 0, 0, v);
    {
        long long ec = v.ec, es = v.es, ep = v.ep;
        bool doneA = false, doneB = false;
#pragma unroll
        for (int q = 0; q < BPT; ++q) {
            if (v.cv[q] > 0) {
                const bool rule = (ec + v.cv[q] > r.nprobe) || (es + v.sv[q] >= r.max_tokens);
                if (!doneA && (rule || ep + v.pv[q] > r.buffer_pages)) {
                    atomicMin(&sm.first, BPT * tid + q);
                    doneA = true;
                }
                if (!doneB && rule) {
                    atomicMin(&sm.first2, BPT * tid + q);
                    doneB = true;
                }
            }
            ec += v.cv[q];
            es += v.sv[q];
            ep += v.pv[q];
        }
    }
    __syncthreads();
    const int frA = sm.first, frB = sm.first2;
    if (frA < SL_NB && frA / BPT == tid) view_publish<NT>(v, frA, &sm.bucket, &sm.bcnt, sm.pre);
    if (frB < SL_NB && frB / BPT == tid) view_publish<NT>(v, frB, &sm.bucket2, &sm.bcnt2, sm.pre2);
    __syncthreads();
    const bool hasA = frA < SL_NB, hasB = frB < SL_NB;
    if ((hasA && sm.bcnt > 32) || (hasB && sm.bcnt2 > 32)) {
        __syncthreads();
        return false;
    }
    const int bA = hasA ? sm.bucket : -1, bB = hasB ? sm.bucket2 : -1;
    if (hasA || hasB) {
        for_candidates<NT>(keys, ne, [&](unsigned long long k, int z) {
            const int b = min(SL_NB - 1, max(0, (int)((sl_key_score(k) - smin) * scale)));
            if (b == bA) {
                const int at = atomicAdd(&sm.nb, 1);
                if (at < 32) {
                    sm.bkeys[at] = k;
                    sm.bsz[at] = z;
                }
            }
            if (b == bB) {
                const int at = atomicAdd(&sm.nb2, 1);
                if (at < 32) {
                    sm.bkeys2[at] = k;
                    sm.bsz2[at] = z;
                }
            }
        });
    }
    __syncthreads();
    // warp 0 resolves A, warp 1 resolves B (one shared copy of the code); a
    // bucket that is kept whole has its threshold just below its lowest key
    if (wid < 2) {
        const bool isA = wid == 0;
        const bool has = isA ? hasA : hasB;
        if (has) {
            const unsigned long long* bk = isA ? sm.bkeys : sm.bkeys2;
            const int m = min(isA ? sm.nb : sm.nb2, 32);
            unsigned long long mn = (tid & 31) < m ? bk[tid & 31] : ~0ull;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mn = min(mn, (unsigned long long)__shfl_xor_sync(0xffffffffu, mn, o));
            const long long* pre = isA ? sm.pre : sm.pre2;
            resolve_boundary(bk, isA ? sm.bsz : sm.bsz2, m, pre[0], pre[1], pre[2], isA ? 1 : 0, mn, sm.rscr[wid], r,
                             isA ? &sm.T : &sm.T2, isA ? &sm.flags : &sm.flags2);
        } else if ((tid & 31) == 0) {
            *(isA ? &sm.T : &sm.T2) = key_lo0 > 0 ? key_lo0 - 1 : 0ull;
        }
    }
    __syncthreads();
    return true;
}

// ---------------------------------------------------------------------------
// scoring helpers (every CTA)
// ---------------------------------------------------------------------------
// Interleaved fma chains over the last subspace for J cells per thread (a
// cell that is not separable runs the chain on column 0 and keeps acc).
template <int J>
IMI_DEV void score_chains(float (&acc)[SL_CPT], const bool (&sep)[SL_CPT], const int (&il)[SL_CPT],
                          const float* q2, const float* cT, int ldT, int sub) {
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
}

IMI_DEV int prefix_table_offset(const SelectArgs& a, int s, int sub) {
    int off = 0;
    for (int t = 0; t < s; ++t) off += sub * sl_ld(a.ks[t]);
    return off;
}


}  // namespace imi
