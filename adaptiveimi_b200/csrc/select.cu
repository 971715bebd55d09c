// select.cu -- decode-time cell scoring and selection, one thread-block
// cluster (8 CTAs, distributed shared memory) per KV group (sm_100a).
//
// Semantics (the reference's decode path, all on the device):
//   * cell scores: compute_impl.cu:62-103 (q_sum over the group's query heads
//     in g order, then an fma chain over d = 0..D-1 with the merged centroid);
//     evaluated separably: the chain over the first S-1 subspaces is shared by
//     every cell with the same digit prefix, the last subspace finishes it per
//     cell -- the same operations in the same order, so the same bits;
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
// ends before the first element A violating any rule.  A is found by
// histogram refinement over the 64-bit key range (key = score bits, then the
// complement of the slot): every CTA histograms its own candidates, the
// cluster merges the histogram slice-wise through DSMEM, the bucket holding A
// is found from cluster-wide descending prefix sums, and once that bucket has
// at most 32 elements CTA 0 ranks them and walks the rules exactly.  Attention
// is independent of row order, so no sort of the selected cells is needed;
// they are emitted in slot order.
#include <cooperative_groups.h>

#include "common.cuh"
#include "imi_internal.h"

namespace cg = cooperative_groups;

namespace imi {

constexpr int SC_CL = 8;                 // CTAs per cluster (one cluster per KV group)
constexpr int SC_THREADS = 512;
constexpr int SC_NB = 2048;              // histogram buckets per refinement round
constexpr int SC_SLICE = SC_NB / SC_CL;  // buckets merged by each CTA
constexpr int SC_MAX_SLOTS = 16384;
constexpr int SC_CHUNK_MAX = SC_MAX_SLOTS / SC_CL;

// Fixed-size shared state (addresses identical in every CTA of the cluster,
// which is what map_shared_rank needs).
struct SelState {
    unsigned long long kmin, kmax;
    int ncand;
    int hist[3][SC_NB];          // local histograms: count, tokens, pages
    int mslice[3][SC_SLICE];     // this CTA's merged slice
    long long slice_tot[3];
    int hit;                     // first hit (descending rank within the slice), -1 if none
    int hit_bucket, hit_cnt;
    long long hit_pre[3];
    int nb;                      // boundary-bucket gather (used in CTA 0)
    int bsz[32];
    unsigned long long bkeys[32];
    unsigned long long T, flags;
    int e_sel, e_rows, e_kept;   // emission totals of this CTA
    int scratch[64];
    long long scratch64[32];
    unsigned long long red64[64];
    uint32_t kept_bits[SC_CHUNK_MAX / 32];
    unsigned long long skey[SC_CHUNK_MAX];  // 0 = not a candidate
    int ssz[SC_CHUNK_MAX];
    int sel_slot[SC_CHUNK_MAX];
    int sel_start[SC_CHUNK_MAX];
};

__device__ int sc_block_scan(int v, int* red, int* total) {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    int x = v;
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, x, o);
        if (l >= o) x += t;
    }
    __syncthreads();
    if (l == 31) red[w] = x;
    __syncthreads();
    if (w == 0) {
        const int nw = blockDim.x >> 5;
        int y = (l < nw) ? red[l] : 0;
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, y, o);
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

__device__ long long sc_block_sum_ll(long long v, long long* red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    long long r = 0;
    for (int q = 0; q < (int)(blockDim.x >> 5); ++q) r += red[q];
    __syncthreads();
    return r;
}

__global__ void __cluster_dims__(SC_CL, 1, 1) __launch_bounds__(SC_THREADS, 1)
    imi_select_cluster_kernel(SelectArgs a) {
    extern __shared__ __align__(16) unsigned char dyn[];
    // the fixed state sits at the start of dynamic shared memory: the same
    // offset in every CTA, as map_shared_rank requires
    SelState& st = *reinterpret_cast<SelState*>(dyn);
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
    const int chunk = (a.n_slots + SC_CL - 1) / SC_CL;
    const int c0 = rank * chunk;
    const int c1 = min(a.n_slots, c0 + chunk);
    const int nloc = max(0, c1 - c0);

    float* qs = reinterpret_cast<float*>(dyn + ((sizeof(SelState) + 15) & ~size_t(15)));  // [dim]
    float* tab = qs + a.dim;                                          // [table]
    float* cT = tab + table + 4;                                      // [sub][k_last+1] (S > 1)

    const size_t hs = (size_t)h;
    const int32_t* sizes = a.cell_sizes + hs * a.n_slots;
    const uint8_t* mask = a.cell_mask + hs * a.n_slots;
    const int32_t* code = a.cell_code + hs * a.n_slots;
    const uint8_t* dirty = a.cell_dirty ? a.cell_dirty + hs * a.n_slots : nullptr;
    const float* merged = a.centroids + hs * a.n_slots * (size_t)a.dim;
    const float* subc = a.sub_centroids + hs * (size_t)S * a.kmax * sub;

    // ---------------- scores of this CTA's slots ----------------
    for (int d = tid; d < a.dim; d += blockDim.x) {
        float acc = 0.0f;
        for (int g = 0; g < a.G; ++g) acc = __fadd_rn(acc, bf16_bits_to_f32(a.q[(hs * a.G + g) * a.dim + d]));
        qs[d] = acc;
    }
    if (S > 1) {
        const float* cl = subc + (size_t)(S - 1) * a.kmax * sub;
        for (int e = tid; e < k_last * sub; e += blockDim.x) {
            const int i = e / sub, d = e - i * sub;
            cT[d * (k_last + 1) + i] = cl[(size_t)i * sub + d];
        }
        if (tid == 0) tab[0] = 0.0f;
    }
    for (int w = tid; w < SC_CHUNK_MAX / 32; w += blockDim.x) st.kept_bits[w] = 0u;
    __syncthreads();
    if (S > 1) {
        int width = 1;
        for (int s = 0; s < S - 1; ++s) {
            const int ks = a.ks[s];
            const float* cs = subc + (size_t)s * a.kmax * sub;
            const int total = width * ks;
            float vals[16];
            int cnt = 0;
            for (int e = tid; e < total && cnt < 16; e += blockDim.x, ++cnt) {
                const int pi = e / ks, i = e - pi * ks;
                float acc = tab[pi];
                const float* cr = cs + (size_t)i * sub;
                for (int d = 0; d < sub; ++d) acc = __fmaf_rn(qs[s * sub + d], cr[d], acc);
                vals[cnt] = acc;
            }
            __syncthreads();
            cnt = 0;
            for (int e = tid; e < total && cnt < 16; e += blockDim.x, ++cnt) tab[e] = vals[cnt];
            __syncthreads();
            width = total;
        }
    }
    unsigned long long kmn = ~0ull, kmx = 0ull;
    int ncand = 0;
    for (int i = tid; i < nloc; i += blockDim.x) {
        const int c = c0 + i;
        const int cc = code[c];
        unsigned long long key = 0ull;
        float s = -INFINITY;
        if (!mask[c] && cc >= 0) {
            if (S == 1 || (dirty && dirty[c])) {
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
            key = ((unsigned long long)ord_f32(s) << 32) | (0xffffffffu - (uint32_t)c);
            kmn = min(kmn, key);
            kmx = max(kmx, key);
            ++ncand;
        }
        st.skey[i] = key;
        st.ssz[i] = key ? sizes[c] : 0;
        if (a.scores_out) a.scores_out[hs * a.n_slots + c] = s;
    }
    for (int o = 16; o > 0; o >>= 1) {
        kmn = min(kmn, (unsigned long long)__shfl_xor_sync(0xffffffffu, kmn, o));
        kmx = max(kmx, (unsigned long long)__shfl_xor_sync(0xffffffffu, kmx, o));
        ncand += __shfl_xor_sync(0xffffffffu, ncand, o);
    }
    if (lid == 0) {
        st.red64[wid] = kmn;
        st.red64[32 + wid] = kmx;
        st.scratch[wid] = ncand;
    }
    __syncthreads();
    if (tid == 0) {
        unsigned long long x = ~0ull, y = 0ull;
        int n = 0;
        for (int q = 0; q < (int)(blockDim.x >> 5); ++q) {
            x = min(x, st.red64[q]);
            y = max(y, st.red64[32 + q]);
            n += st.scratch[q];
        }
        st.kmin = x;
        st.kmax = y;
        st.ncand = n;
        st.nb = 0;
    }
    cluster.sync();
    unsigned long long key_lo0 = ~0ull, key_hi0 = 0ull;
    for (int q = 0; q < SC_CL; ++q) {
        const SelState* rs = cluster.map_shared_rank(&st, q);
        key_lo0 = min(key_lo0, rs->kmin);
        key_hi0 = max(key_hi0, rs->kmax);
    }
    const bool any_cand = key_hi0 != 0ull;

    // ---------------- boundary search ----------------
    // result: threshold T (selected = key > T), flags = 1 when the rank or the
    // token rule (not only the page rule) fires at the boundary element
    auto search = [&](bool use_pages, unsigned long long& T_out, unsigned long long& flags_out) {
        unsigned long long lo = key_lo0, hi = key_hi0;
        long long C = 0, Sz = 0, Pg = 0;  // totals of candidates with key > hi
        while (true) {
            const unsigned __int128 range = (unsigned __int128)(hi - lo) + 1;
            for (int b = tid; b < SC_NB; b += blockDim.x) st.hist[0][b] = st.hist[1][b] = st.hist[2][b] = 0;
            if (tid == 0 && rank == 0) st.nb = 0;
            __syncthreads();
            for (int i = tid; i < nloc; i += blockDim.x) {
                const unsigned long long k = st.skey[i];
                if (k == 0ull || k < lo || k > hi) continue;
                const int b = (int)(((unsigned __int128)(k - lo) * SC_NB) / range);
                const int sz = st.ssz[i];
                atomicAdd(&st.hist[0][b], 1);
                atomicAdd(&st.hist[1][b], sz);
                atomicAdd(&st.hist[2][b], sz > 0 ? (sz + a.page_size - 1) / a.page_size : 0);
            }
            cluster.sync();  // (1) every local histogram is complete
            // merge this CTA's slice of buckets over the cluster
            long long tot[3] = {0, 0, 0};
            for (int e = tid; e < 3 * SC_SLICE; e += blockDim.x) {
                const int which = e / SC_SLICE, j = e - which * SC_SLICE;
                const int b = rank * SC_SLICE + j;
                int v = 0;
                for (int q = 0; q < SC_CL; ++q) v += cluster.map_shared_rank(&st, q)->hist[which][b];
                st.mslice[which][j] = v;
                tot[which] += v;
            }
            for (int which = 0; which < 3; ++which) {
                const long long t = sc_block_sum_ll(tot[which], st.scratch64);
                if (tid == 0) st.slice_tot[which] = t;
            }
            cluster.sync();  // (2) merged slices and slice totals are published
            // prefix over the slices above this one (descending bucket order)
            long long pc = C, ps = Sz, pp = Pg;
            for (int q = rank + 1; q < SC_CL; ++q) {
                const SelState* rs = cluster.map_shared_rank(&st, q);
                pc += rs->slice_tot[0];
                ps += rs->slice_tot[1];
                pp += rs->slice_tot[2];
            }
            // descending scan of this slice: thread t < SC_SLICE owns bucket
            // index j = SC_SLICE - 1 - t
            const int j = SC_SLICE - 1 - tid;
            const int cb = tid < SC_SLICE ? st.mslice[0][j] : 0;
            const int sb = tid < SC_SLICE ? st.mslice[1][j] : 0;
            const int pb = tid < SC_SLICE ? st.mslice[2][j] : 0;
            int t0, t1, t2;
            const int ic = sc_block_scan(cb, st.scratch, &t0);
            const int is = sc_block_scan(sb, st.scratch, &t1);
            const int ip = sc_block_scan(pb, st.scratch, &t2);
            const long long ec = pc + ic - cb, es = ps + is - sb, ep = pp + ip - pb;
            const bool hit = tid < SC_SLICE && cb > 0 &&
                             ((ec + cb > a.nprobe) || (es + sb >= a.max_tokens) ||
                              (use_pages && ep + pb > a.buffer_pages));
            if (tid == 0) st.hit = SC_SLICE;
            __syncthreads();
            if (hit) atomicMin(&st.hit, tid);
            __syncthreads();
            if (st.hit == tid) {
                st.hit_bucket = rank * SC_SLICE + j;
                st.hit_cnt = cb;
                st.hit_pre[0] = ec;
                st.hit_pre[1] = es;
                st.hit_pre[2] = ep;
            }
            cluster.sync();  // (3) per-slice first hits are published
            int owner = -1;
            for (int q = SC_CL - 1; q >= 0; --q) {
                if (cluster.map_shared_rank(&st, q)->hit < SC_SLICE) {
                    owner = q;
                    break;
                }
            }
            if (owner < 0) {
                // no element of [lo, hi] triggers a rule: all of it is selected
                T_out = lo > 0 ? lo - 1 : 0ull;
                flags_out = 0ull;
                cluster.sync();
                return;
            }
            const SelState* os = cluster.map_shared_rank(&st, owner);
            const int bb = os->hit_bucket, cnt = os->hit_cnt;
            const long long qc = os->hit_pre[0], qs_ = os->hit_pre[1], qp = os->hit_pre[2];
            const unsigned long long blo =
                lo + (unsigned long long)(((unsigned __int128)bb * range + SC_NB - 1) / SC_NB);
            const unsigned long long bhi =
                lo + (unsigned long long)(((unsigned __int128)(bb + 1) * range + SC_NB - 1) / SC_NB) - 1ull;
            if (cnt <= 32) {
                // gather the bucket into CTA 0 and walk the rules in rank order
                SelState* s0 = cluster.map_shared_rank(&st, 0);
                for (int i = tid; i < nloc; i += blockDim.x) {
                    const unsigned long long k = st.skey[i];
                    if (k == 0ull || k < blo || k > bhi) continue;
                    const int at = atomicAdd(&s0->nb, 1);
                    if (at < 32) {
                        s0->bkeys[at] = k;
                        s0->bsz[at] = st.ssz[i];
                    }
                }
                cluster.sync();  // (4) the bucket is gathered
                if (rank == 0 && wid == 0) {
                    const int n = min(st.nb, 32);
                    const unsigned long long mk = lid < n ? st.bkeys[lid] : 0ull;
                    const int msz = lid < n ? st.bsz[lid] : 0;
                    int rk = 0;
                    for (int q = 0; q < n; ++q) rk += (__shfl_sync(0xffffffffu, mk, q) > mk) ? 1 : 0;
                    long long xc = qc, xs = qs_, xp = qp;
                    unsigned long long T = blo > 0 ? blo - 1 : 0ull;
                    unsigned long long fl = 1ull;  // if nothing fires here, the token rule fires just below
                    bool found = false;
                    for (int r = 0; r < n && !found; ++r) {
                        const unsigned hm = __ballot_sync(0xffffffffu, lid < n && rk == r);
                        const int src = __ffs(hm) - 1;
                        const unsigned long long k = __shfl_sync(0xffffffffu, mk, src);
                        const int sz = __shfl_sync(0xffffffffu, msz, src);
                        const int pg = sz > 0 ? (sz + a.page_size - 1) / a.page_size : 0;
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
                    if (lid == 0) {
                        st.T = T;
                        st.flags = fl;
                    }
                }
                cluster.sync();  // (5) CTA 0 published the boundary
                const SelState* z = cluster.map_shared_rank(&st, 0);
                T_out = z->T;
                flags_out = z->flags;
                cluster.sync();  // (6) everyone has read it before reuse
                return;
            }
            lo = blo;
            hi = bhi;
            C = qc;
            Sz = qs_;
            Pg = qp;
            cluster.sync();  // slices / hits may be rewritten in the next round
        }
    };

    unsigned long long thrA = ~0ull, thrB = ~0ull;  // no candidates: nothing selected
    if (any_cand) {
        unsigned long long fl;
        search(true, thrA, fl);
        if (fl) {
            thrB = thrA;
        } else {
            unsigned long long fl2;
            search(false, thrB, fl2);
        }
    }

    // ---------------- emission ----------------
    int lsel = 0, lrows = 0, lkept = 0;
    for (int i = tid; i < nloc; i += blockDim.x) {
        const unsigned long long k = st.skey[i];
        if (k == 0ull) continue;
        if (k > thrA) {
            ++lsel;
            lrows += st.ssz[i];
        }
        if (k > thrB) {
            ++lkept;
            atomicOr(&st.kept_bits[i >> 5], 1u << (i & 31));
        }
    }
    {
        int t;
        sc_block_scan(lsel, st.scratch, &t);
        if (tid == 0) st.e_sel = t;
        sc_block_scan(lrows, st.scratch, &t);
        if (tid == 0) st.e_rows = t;
        sc_block_scan(lkept, st.scratch, &t);
        if (tid == 0) st.e_kept = t;
    }
    cluster.sync();  // emission totals and kept bitmaps are published
    int sel_base = 0, row_base = 0, nsel = 0, sel_rows = 0, nkept = 0;
    for (int q = 0; q < SC_CL; ++q) {
        const SelState* rs = cluster.map_shared_rank(&st, q);
        if (q < rank) {
            sel_base += rs->e_sel;
            row_base += rs->e_rows;
        }
        nsel += rs->e_sel;
        sel_rows += rs->e_rows;
        nkept += rs->e_kept;
    }
    int32_t* rows = a.row_index + hs * (size_t)a.exec_capacity;
    const int32_t* offs = a.cell_offsets + hs * (a.n_slots + 1);
    const int static_len = a.static_len;
    int run_sel = 0, run_rows = 0;
    for (int base = 0; base < nloc; base += blockDim.x) {
        const int i = base + tid;
        bool fin = false;
        int sz = 0;
        if (i < nloc) {
            const unsigned long long k = st.skey[i];
            fin = k != 0ull && k > thrA;
            sz = fin ? st.ssz[i] : 0;
        }
        int tf, tr;
        const int rf = sc_block_scan(fin ? 1 : 0, st.scratch, &tf) + run_sel;
        const int rr = sc_block_scan(sz, st.scratch, &tr) + run_rows;
        if (fin) {
            const int gi = sel_base + rf - 1;
            if (gi < a.nprobe) a.sel_cells[hs * a.nprobe + gi] = c0 + i;
            st.sel_slot[rf - 1] = c0 + i;
            st.sel_start[rf - 1] = static_len + row_base + rr - sz;
        }
        run_sel += tf;
        run_rows += tr;
    }
    __syncthreads();
    for (int i = wid; i < run_sel; i += (SC_THREADS >> 5)) {
        const int slot = st.sel_slot[i];
        const int s0 = st.sel_start[i];
        const int off = offs[slot];
        const int sz = sizes[slot];
        for (int jj = lid; jj < sz; jj += 32)
            if (s0 + jj < a.exec_capacity) rows[s0 + jj] = off + jj;
    }
    if (rank == 0) {
        for (int r = tid; r < static_len; r += blockDim.x) rows[r] = (1 << 30) | r;
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
                    if (cid >= 0 && cid < a.n_slots) {
                        const int ow = cid / chunk, li = cid - ow * chunk;
                        f = (cluster.map_shared_rank(&st, ow)->kept_bits[li >> 5] >> (li & 31)) & 1;
                    }
                    if (cid == a.padding_id && has_pad) f = 1;
                }
                int tot;
                const int incl = sc_block_scan(f, st.scratch, &tot);
                if (f) {
                    const int at = total + appended + incl - 1;
                    if (at < a.exec_capacity) rows[at] = (2 << 30) | pidx;
                }
                appended += tot;
            }
            total = min(total + appended, a.exec_capacity);
        }
        if (tid == 0) {
            a.sel_count[h] = min(nsel, a.nprobe);
            a.row_count[h] = total;
            if (a.kept_count) a.kept_count[h] = nkept;
        }
    }
    cluster.sync();  // no CTA leaves while another may still read its shared memory
}

size_t select_smem_bytes(const SelectArgs& a) {
    const int S = a.parts == 0 ? 1 : a.parts;
    int table = 1;
    for (int s = 0; s < S - 1; ++s) table *= a.ks[s];
    const size_t ct = S > 1 ? (size_t)(a.dim / S) * (a.ks[S - 1] + 1) : 0;
    return ((sizeof(SelState) + 15) & ~size_t(15)) + sizeof(float) * ((size_t)a.dim + table + 4 + ct) + 16;
}

static size_t select_dynamic_smem(const SelectArgs& a) { return select_smem_bytes(a); }

int select_max_slots() { return SC_MAX_SLOTS; }

cudaError_t launch_select(const SelectArgs& a, cudaStream_t st) {
    const size_t dyn = select_dynamic_smem(a);
    cudaError_t e =
        cudaFuncSetAttribute(imi_select_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn);
    if (e != cudaSuccess) return e;
    imi_select_cluster_kernel<<<dim3(SC_CL, a.bg), SC_THREADS, dyn, st>>>(a);
    return cudaGetLastError();
}

}  // namespace imi
