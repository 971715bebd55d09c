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
// refinement over the 64-bit key range (key = score bits, then the complement
// of the slot, so keys are unique): a round histograms the candidates into
// 2048 power-of-two buckets of the key range weighted by (1, tokens, pages), a
// block-wide descending scan finds the first bucket where a rule can fire, and
// once that bucket holds at most 32 elements one warp ranks them and walks the
// rules exactly.  The boundary with all three rules (the selected cells) and
// the boundary without the page rule (the kept list that delta rows match
// against) come out of the same pass.  Attention does not depend on row order,
// so the selected cells are emitted in slot order without a sort.
//
// The kernel sits on the decode critical path (attention waits on it), so it
// is written for latency: a cluster of 8 CTAs per KV group scores the cells
// (subspace centroids staged transposed in shared memory, two interleaved fma
// chains per thread) and stores every key and size straight into the leader
// CTA's shared memory through DSMEM; the leader alone then runs the boundary
// search and emits the rows (warp-contiguous slot ranges, ballot ranks).  Two
// cluster barriers in all.
#include <cooperative_groups.h>

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

struct SelHdr {
    unsigned long long kmin, kmax;
    int hist[3][SL_NB];
    int red[64];
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
    int wsel[SL_WARPS], wrows[SL_WARPS], wkept[SL_WARPS];
};

__device__ __forceinline__ int sl_scan(int v, int* red, int* total) {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, x, o);
        if (l >= o) x += t;
    }
    __syncthreads();
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

__device__ __forceinline__ int warp_incl_scan(int x) {
    const int l = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, x, o);
        if (l >= o) x += t;
    }
    return x;
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
    const int k_last = a.ks[S - 1];
    int table = 1;
    for (int s = 0; s < S - 1; ++s) table *= a.ks[s];
    int kpre = 1;  // largest k among the first S-1 subspaces
    for (int s = 0; s < S - 1; ++s) kpre = max(kpre, a.ks[s]);
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
    float* cT = reinterpret_cast<float*>(p);  // last subspace, [sub][k_last + 1]
    p += sizeof(float) * (S > 1 ? (size_t)sub * (k_last + 1) : 0);
    float* cP = reinterpret_cast<float*>(p);  // one prefix subspace at a time, [sub][kpre + 1]
    int* sel_slot = reinterpret_cast<int*>(cP);  // leader, reused after scoring
    int* sel_start = sel_slot + 2048;

    const size_t hs = (size_t)h;
    auto stamp = [&](int k) {
        if (a.phase_ns && tid == 0 && rank == 0) {
            unsigned long long t;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
            a.phase_ns[hs * 8 + k] = t;
        }
    };
    stamp(0);
    const int32_t* sizes = a.cell_sizes + hs * n;
    const uint8_t* mask = a.cell_mask + hs * n;
    const int32_t* code = a.cell_code + hs * n;
    const uint8_t* dirty = a.cell_dirty ? a.cell_dirty + hs * n : nullptr;
    const float* merged = a.centroids + hs * n * (size_t)a.dim;
    const float* subc = a.sub_centroids + hs * (size_t)S * a.kmax * sub;

    // ---------------- every CTA: q_sum, last subspace, prefix sums ----------------
    // all staging loads are issued before the first barrier
    // q_sum: every load of a thread is issued before the adds
    if (tid < a.dim) {
        float qv[8];
#pragma unroll
        for (int g = 0; g < 8; ++g) qv[g] = g < a.G ? bf16_bits_to_f32(a.q[(hs * a.G + g) * a.dim + tid]) : 0.0f;
        float acc = 0.0f;
        for (int g = 0; g < a.G; ++g) acc = __fadd_rn(acc, qv[g]);
        qs[tid] = acc;
    }
    // centroid staging: batches of 16 loads in registers, then the stores
    auto stage_T = [&](const float* src, int k, float* dst, int ld) {
        const int total = k * sub;
        for (int base = 0; base < total; base += 16 * SL_THREADS) {
            float v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int e = base + j * SL_THREADS + tid;
                v[j] = e < total ? src[e] : 0.0f;
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int e = base + j * SL_THREADS + tid;
                if (e < total) {
                    const int i = e / sub, d = e - i * sub;
                    dst[d * ld + i] = v[j];
                }
            }
        }
    };
    if (S > 1) {
        stage_T(subc + (size_t)(S - 1) * a.kmax * sub, k_last, cT, k_last + 1);
        stage_T(subc, a.ks[0], cP, kpre + 1);
        if (tid == 0) tab[0] = 0.0f;
    }
    if (rank == 0 && tid == 0) {
        sm.kmin = ~0ull;
        sm.kmax = 0ull;
    }
    if (S > 1) {
        int width = 1;
        for (int s = 0; s < S - 1; ++s) {
            const int ks = a.ks[s];
            if (s > 0) {
                __syncthreads();
                stage_T(subc + (size_t)s * a.kmax * sub, ks, cP, kpre + 1);
            }
            __syncthreads();
            const int total = width * ks;
            float vals[16];
            int cnt = 0;
            for (int e = tid; e < total && cnt < 16; e += blockDim.x, ++cnt) {
                const int pi = e / ks, i = e - pi * ks;
                float acc = tab[pi];
                const float* qq = qs + s * sub;
#pragma unroll 8
                for (int d = 0; d < sub; ++d) acc = __fmaf_rn(qq[d], cP[d * (kpre + 1) + i], acc);
                vals[cnt] = acc;
            }
            __syncthreads();
            cnt = 0;
            for (int e = tid; e < total && cnt < 16; e += blockDim.x, ++cnt) tab[e] = vals[cnt];
            width = total;
        }
    }
    __syncthreads();
    stamp(1);
    cluster.sync();  // every CTA is running (DSMEM may be used) and the leader's header is set
    // ---------------- every CTA: score its slots, scatter into the leader ----------------
    {
        SelHdr* lead = cluster.map_shared_rank(&sm, 0);
        unsigned long long* lkey = cluster.map_shared_rank(skey, 0);
        int* lsz = cluster.map_shared_rank(ssz, 0);
        const int chunk = (n + SL_CL - 1) / SL_CL;
        const int c0 = rank * chunk;
        const int c1 = min(n, c0 + chunk);
        const float* q2 = qs + (S - 1) * sub;
        unsigned long long kmn = ~0ull, kmx = 0ull;
        for (int cb = c0 + tid; cb < c1; cb += 2 * SL_THREADS) {
            // two interleaved chains per thread
            float acc[2];
            int il[2], ccv[2], szv[2];
            bool sep[2], cand[2], mk[2], dk[2];
            const int cs[2] = {cb, cb + SL_THREADS};
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int c = cs[j];
                const bool in = c < c1;
                ccv[j] = in ? code[c] : -1;
                mk[j] = in ? mask[c] != 0 : true;
                szv[j] = in ? sizes[c] : 0;
                dk[j] = in && dirty ? dirty[c] != 0 : false;
            }
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int c = cs[j];
                acc[j] = 0.0f;
                il[j] = 0;
                sep[j] = cand[j] = false;
                if (c < c1) {
                    const int cc = ccv[j];
                    if (!mk[j] && cc >= 0) {
                        cand[j] = true;
                        if (S > 1 && !dk[j]) {
                            int pidx = 0;
                            for (int t = 0; t < S - 1; ++t) pidx = pidx * a.ks[t] + ((cc >> (8 * t)) & 0xff);
                            il[j] = (cc >> (8 * (S - 1))) & 0xff;
                            acc[j] = tab[pidx];
                            sep[j] = true;
                        }
                    }
                }
            }
            if (S > 1 && (sep[0] || sep[1])) {
#pragma unroll 8
                for (int d = 0; d < sub; ++d) {
                    const float qd = q2[d];
                    const float* row = cT + d * (k_last + 1);
                    if (sep[0]) acc[0] = __fmaf_rn(qd, row[il[0]], acc[0]);
                    if (sep[1]) acc[1] = __fmaf_rn(qd, row[il[1]], acc[1]);
                }
            }
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int c = cs[j];
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
    // walk them in order applying the rules from the bucket's prefix.
    auto resolve = [&](const unsigned long long* bk, const int* bs, int m, long long xc, long long xs, long long xp,
                       bool use_pages, unsigned long long blo, unsigned long long& T, unsigned long long& fl) {
        const unsigned long long mk = lid < m ? bk[lid] : 0ull;
        const int msz = lid < m ? bs[lid] : 0;
        int rk = 0;
        for (int q = 0; q < m; ++q) rk += (__shfl_sync(0xffffffffu, mk, q) > mk) ? 1 : 0;
        T = blo > 0 ? blo - 1 : 0ull;
        fl = 1ull;  // nothing fires here: the token rule fires just below this bucket
        bool found = false;
        for (int r = 0; r < m && !found; ++r) {
            const unsigned hm = __ballot_sync(0xffffffffu, lid < m && rk == r);
            const int src = __ffs(hm) - 1;
            const unsigned long long k = __shfl_sync(0xffffffffu, mk, src);
            const int sz = __shfl_sync(0xffffffffu, msz, src);
            const int pg = pages_of(sz);
            const bool rc = (xc >= a.nprobe) || (xs >= a.max_tokens);
            const bool rp = use_pages && (xp + pg > a.buffer_pages);
            if (rc || rp) {
                T = k;
                fl = rc ? 1ull : 0ull;
                found = true;
            } else {
                xc += 1;
                xs += sz;
                xp += pg;
            }
        }
    };

    // Histogram of the candidates with lo <= key <= hi into power-of-two
    // buckets, and the descending block scan; returns per-thread bucket
    // values (thread t owns buckets SL_NB-1-4t .. SL_NB-4-4t).
    struct Scan {
        int cv[4], sv[4], pv[4];
        long long ec, es, ep;  // exclusive prefixes before the thread's first bucket
    };
    auto histogram = [&](unsigned long long lo, unsigned long long hi, int shift, long long C, long long Sz,
                         long long Pg, Scan& sc) {
        for (int b = tid; b < SL_NB; b += blockDim.x) sm.hist[0][b] = sm.hist[1][b] = sm.hist[2][b] = 0;
        if (tid == 0) {
            sm.nb = sm.nb2 = 0;
            sm.first = sm.first2 = SL_NB;
        }
        __syncthreads();
        for (int c = tid; c < n; c += blockDim.x) {
            const unsigned long long k = skey[c];
            if (k == 0ull || k < lo || k > hi) continue;
            const int b = (int)((k - lo) >> shift);
            const int sz = ssz[c];
            atomicAdd(&sm.hist[0][b], 1);
            atomicAdd(&sm.hist[1][b], sz);
            atomicAdd(&sm.hist[2][b], pages_of(sz));
        }
        __syncthreads();
        int c4 = 0, s4 = 0, p4 = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int b = SL_NB - 1 - 4 * tid - q;
            sc.cv[q] = sm.hist[0][b];
            sc.sv[q] = sm.hist[1][b];
            sc.pv[q] = sm.hist[2][b];
            c4 += sc.cv[q];
            s4 += sc.sv[q];
            p4 += sc.pv[q];
        }
        const int ic = sl_scan(c4, sm.red, nullptr);
        const int is = sl_scan(s4, sm.red, nullptr);
        const int ip = sl_scan(p4, sm.red, nullptr);
        sc.ec = C + ic - c4;
        sc.es = Sz + is - s4;
        sc.ep = Pg + ip - p4;
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
            Scan sc;
            histogram(lo, hi, shift, C, Sz, Pg, sc);
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
                for (int c = tid; c < n; c += blockDim.x) {
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
                    resolve(sm.bkeys, sm.bsz, min(sm.nb, 32), qc, qsz, qp, use_pages, blo, T, fl);
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
        for (int b = tid; b < SL_NB; b += blockDim.x) sm.hist[0][b] = sm.hist[1][b] = sm.hist[2][b] = 0;
        if (tid == 0) {
            sm.nb = sm.nb2 = 0;
            sm.first = sm.first2 = SL_NB;
        }
        __syncthreads();
        for (int c = tid; c < n; c += blockDim.x) {
            const unsigned long long k = skey[c];
            if (k == 0ull) continue;
            const int b = bucket_of(k);
            const int sz = ssz[c];
            atomicAdd(&sm.hist[0][b], 1);
            atomicAdd(&sm.hist[1][b], sz);
            atomicAdd(&sm.hist[2][b], pages_of(sz));
        }
        __syncthreads();
        Scan sc;
        {
            int c4 = 0, s4 = 0, p4 = 0;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int b = SL_NB - 1 - 4 * tid - q;
                sc.cv[q] = sm.hist[0][b];
                sc.sv[q] = sm.hist[1][b];
                sc.pv[q] = sm.hist[2][b];
                c4 += sc.cv[q];
                s4 += sc.sv[q];
                p4 += sc.pv[q];
            }
            const int ic = sl_scan(c4, sm.red, nullptr);
            const int is = sl_scan(s4, sm.red, nullptr);
            const int ip = sl_scan(p4, sm.red, nullptr);
            sc.ec = ic - c4;
            sc.es = is - s4;
            sc.ep = ip - p4;
        }
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
            for (int c = tid; c < n; c += blockDim.x) {
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
                resolve(sm.bkeys, sm.bsz, m, sm.pre[0], sm.pre[1], sm.pre[2], true, minA, T, fl);
            } else {
                T = key_lo0 > 0 ? key_lo0 - 1 : 0ull;
            }
            if (lid == 0) sm.T = T;
        } else if (wid == 1) {
            unsigned long long T = ~0ull, fl = 0ull;
            if (hasB) {
                const int m = min(sm.nb2, 32);
                for (int q = 0; q < m; ++q) minB = min(minB, sm.bkeys2[q]);
                resolve(sm.bkeys2, sm.bsz2, m, sm.pre2[0], sm.pre2[1], sm.pre2[2], false, minB, T, fl);
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
    // consecutive slots (conflict-free), warp ballots give the in-order ranks
    const int R = ((n + SL_WARPS - 1) / SL_WARPS + 31) & ~31;
    const int w0 = wid * R, w1 = min(n, w0 + R);
    int wsel = 0, wrows = 0, wkept = 0;
    for (int base = w0; base < w1; base += 32) {
        const int c = base + lid;
        const unsigned long long k = c < w1 ? skey[c] : 0ull;
        const bool fin = k != 0ull && k > thrA;
        const bool kept = k != 0ull && k > thrB;
        wsel += __popc(__ballot_sync(0xffffffffu, fin));
        wkept += __popc(__ballot_sync(0xffffffffu, kept));
        wrows += warp_sum_i(fin ? ssz[c] : 0);
    }
    if (lid == 0) {
        sm.wsel[wid] = wsel;
        sm.wrows[wid] = wrows;
        sm.wkept[wid] = wkept;
    }
    __syncthreads();
    int sel_base = 0, row_base = 0, nsel = 0, sel_rows = 0, nkept = 0;
#pragma unroll
    for (int q = 0; q < SL_WARPS; ++q) {
        if (q < wid) {
            sel_base += sm.wsel[q];
            row_base += sm.wrows[q];
        }
        nsel += sm.wsel[q];
        sel_rows += sm.wrows[q];
        nkept += sm.wkept[q];
    }
    const int static_len = a.static_len;
    {
        int si = sel_base, ri = static_len + row_base;
        for (int base = w0; base < w1; base += 32) {
            const int c = base + lid;
            const unsigned long long k = c < w1 ? skey[c] : 0ull;
            const bool fin = k != 0ull && k > thrA;
            const unsigned fm = __ballot_sync(0xffffffffu, fin);
            const int sz = fin ? ssz[c] : 0;
            const int incl = warp_incl_scan(sz);
            if (fin) {
                const int my = si + __popc(fm & ((1u << lid) - 1u));
                if (my < a.nprobe) a.sel_cells[hs * a.nprobe + my] = c;
                if (my < 2048) {
                    sel_slot[my] = c;
                    sel_start[my] = ri + incl - sz;
                }
            }
            si += __popc(fm);
            ri += __shfl_sync(0xffffffffu, incl, 31);
        }
    }
    __syncthreads();
    stamp(4);
    int32_t* rows = a.row_index + hs * (size_t)a.exec_capacity;
    const int32_t* offs = a.cell_offsets + hs * (n + 1);
    for (int r = tid; r < static_len; r += blockDim.x) rows[r] = (1 << 30) | r;
    {
        // warp w takes cells [32w', 32w'+32) for w' = w, w + SL_WARPS, ...; the
        // lanes first load the 32 cells' list offsets together
        const int ns = min(nsel, 2048);
        for (int i0 = wid * 32; i0 < ns; i0 += SL_WARPS * 32) {
            const int mi = i0 + lid;
            const int mslot = mi < ns ? sel_slot[mi] : 0;
            const int moff = mi < ns ? offs[mslot] : 0;
            const int mst = mi < ns ? sel_start[mi] : 0;
            const int msz = mi < ns ? ssz[mslot] : 0;
            const int cnt = min(32, ns - i0);
            for (int q = 0; q < cnt; ++q) {
                const int off = __shfl_sync(0xffffffffu, moff, q);
                const int s0 = __shfl_sync(0xffffffffu, mst, q);
                const int sz = __shfl_sync(0xffffffffu, msz, q);
                for (int jj = lid; jj < sz; jj += 32)
                    if (s0 + jj < a.exec_capacity) rows[s0 + jj] = off + jj;
            }
        }
    }
    int total = min(static_len + sel_rows, a.exec_capacity);
    if (a.delta_count) {
        const int dcount = min(a.delta_count[h], a.delta_capacity);
        const bool has_pad = nkept < a.nprobe;
        const int32_t* dids = a.delta_cell_ids + hs * a.delta_capacity;
        int appended = 0;
        for (int base = 0; base < dcount; base += blockDim.x) {
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
            const int incl = sl_scan(f, sm.red, &tot);
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
    int table = 1, kpre = 1;
    for (int s = 0; s < S - 1; ++s) {
        table *= a.ks[s];
        kpre = a.ks[s] > kpre ? a.ks[s] : kpre;
    }
    const int sub = a.dim / S;
    const size_t ct = S > 1 ? (size_t)sub * (a.ks[S - 1] + 1) : 0;
    size_t cp = S > 1 ? (size_t)sub * (kpre + 1) * 4 : 0;
    if (cp < 2 * 2048 * 4) cp = 2 * 2048 * 4;  // reused for the selected-cell lists
    const size_t npad = ((size_t)a.n_slots + 1) & ~size_t(1);
    return ((sizeof(SelHdr) + 15) & ~size_t(15)) + 12 * npad + sizeof(float) * ((size_t)a.dim + table + 4 + ct) +
           cp + 16;
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
