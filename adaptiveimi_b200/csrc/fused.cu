// fused.cu -- one decode layer's retrieval and attention in a single launch
// (sm_100a): cell scoring, the two selection boundaries, the execution-row
// layout and the split-K gather attention with its split merge.
//
// Semantics: exactly those of the select kernel (select.cu; retrieval.py:295-303,
// wave_buffer_cpu_hotcold.cpp:303-371, async_update.py:46-76) followed by the
// attention kernel (attention.cu; weighted_flash_decoding as retrieval.py:439-447
// calls it).  Only the orchestration differs.
//
// Grid (splits, groups), one CTA per SM, a cooperative launch (every CTA is
// resident at once, so a CTA may wait for the others of its group).  Each CTA:
//  1. scores its slice of the group's occupied slots (the separable fma chains
//     of the select kernel, bit-identical to compute_impl.cu:62-103) and writes
//     the slice's ranking keys and sizes to the group's scratch, then arrives at
//     the group's counter (release);
//  2. waits for the group's other CTAs (acquire, bounded: a wait that runs out
//     sets bit 1 of the attention status and the CTA contributes nothing);
//  3. loads every key of the group into shared memory and finds both
//     boundaries itself (all CTAs of a group reach the same thresholds, so no
//     broadcast is needed);
//  4. lays out the execution rows as runs in shared memory -- the steady zone,
//     each selected cell's list rows (cells in slot order), each matching delta
//     row -- so a row's source is one binary search away;
//  5. streams its contiguous share of the group's 16-row tiles through the
//     attention loop of attention.cu and writes one (m, l, o) partial; the last
//     CTA of the group (a ticket) merges the partials into the output and
//     re-arms the group's counters.
// CTA 0 of a group writes the selection outputs (selected cells, counts); every
// CTA writes the row-list entries of its own tiles when a row list is given.
// Compared with the select kernel followed by the attention kernel this saves
// the hand-off between the two launches, the cluster barriers of the
// selection, and the row list's round trip through memory.
#include "attn_core.cuh"
#include "common.cuh"
#include "imi_internal.h"
#include "select_core.cuh"

namespace imi {

constexpr int FU_THREADS = AT_WARPS * 32;  // the streaming warps do the selection too
constexpr int FU_WARPS = AT_WARPS;
constexpr int FU_CPT = 4;                  // slots per thread when scoring a slice
constexpr unsigned FU_SPIN_LIMIT = 1u << 21;

struct FusedArgs {
    SelectArgs s;
    AttnArgs a;
    AppendArgs ap;                // ap.new_keys set: the step's steady-zone append, done before the barrier
    unsigned long long* keys;     // [bg, n_slots] scratch: ranking keys (0: not a candidate)
    int32_t* sizes;               // [bg, n_slots] scratch
    unsigned long long* range;    // [bg, splits, 2] scratch: each slice's lowest and highest key
    uint32_t* arrive;             // [bg] group counters: zero before the first call, re-armed by the kernel
    int runs_cap;                 // run-table entries (static + nprobe + delta capacity)
};

// Byte offsets of the shared-memory regions (identical in every CTA).
struct FusedLayout {
    size_t keys, sizes, qs, tab, tables, sel_end, runs, total;
};

__host__ __device__ inline size_t fu_align(size_t x) { return (x + 127) & ~size_t(127); }

__host__ __device__ inline FusedLayout fused_layout(const SelectArgs& a, int runs_cap) {
    const int S = a.parts == 0 ? 1 : a.parts;
    const int sub = a.dim / S;
    int table = 1;
    for (int s = 0; s < S - 1; ++s) table *= a.ks[s];
    const int ne = (a.slot_bound > 0 && a.slot_bound < a.n_slots) ? a.slot_bound : a.n_slots;
    FusedLayout L;
    size_t o = fu_align(sizeof(SelHdr));
    L.keys = o;
    o = fu_align(o + 8 * (size_t)ne);
    L.sizes = o;
    o = fu_align(o + 4 * (size_t)ne);
    L.qs = o;
    o = fu_align(o + 4 * (size_t)a.dim);
    L.tab = o;
    o = fu_align(o + 4 * ((size_t)table + 4));
    L.tables = o;
    size_t tables = 0;
    if (S > 1) {
        for (int s = 0; s < S; ++s) tables += (size_t)sub * sl_ld(a.ks[s]) * sizeof(float);
        if (S > 2) tables += (256 + (size_t)a.ks[0] * a.ks[1]) * sizeof(float);
    }
    o = fu_align(o + tables);
    L.sel_end = o;
    // the run table lives past both the selection area and the attention ring
    const size_t ring = (size_t)AT_RING_BYTES;
    L.runs = fu_align(o > ring ? o : ring);
    L.total = L.runs + 8 * ((size_t)runs_cap + 1);
    return L;
}

IMI_DEV void fu_stamp(const SelectArgs& a, int h, int k, bool on) {
    if (on) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        a.phase_ns[(size_t)h * 8 + k] = t;
    }
}

__global__ void __launch_bounds__(FU_THREADS, 1) imi_decode_fused_kernel(const __grid_constant__ FusedArgs f) {
    extern __shared__ __align__(128) unsigned char fsm[];
    const SelectArgs& a = f.s;
    const AttnArgs& at = f.a;
    const int h = blockIdx.y, split = blockIdx.x, J = gridDim.x;
    const int tid = threadIdx.x, wid = tid >> 5, lid = tid & 31;
    const size_t hs = (size_t)h;
    const int S = a.parts == 0 ? 1 : a.parts;
    const int sub = a.dim / S;
    const int sub_shift = __ffs(sub) - 1;
    const int k_last = a.ks[S - 1];
    const int n = a.n_slots;
    const int ne = (a.slot_bound > 0 && a.slot_bound < n) ? a.slot_bound : n;
    SelRules rules;
    rules.nprobe = a.nprobe;
    rules.max_tokens = a.max_tokens;
    rules.buffer_pages = a.buffer_pages;
    rules.page_size = a.page_size;
    rules.pg_shift = __ffs(a.page_size) - 1;
    rules.pg_pow2 = (a.page_size & (a.page_size - 1)) == 0;
    const FusedLayout Lo = fused_layout(a, f.runs_cap);
    SelHdr& sm = *reinterpret_cast<SelHdr*>(fsm);
    unsigned long long* skey = reinterpret_cast<unsigned long long*>(fsm + Lo.keys);
    int* ssz = reinterpret_cast<int*>(fsm + Lo.sizes);
    float* qs = reinterpret_cast<float*>(fsm + Lo.qs);
    float* tab = reinterpret_cast<float*>(fsm + Lo.tab);
    float* cT = reinterpret_cast<float*>(fsm + Lo.tables);
    const int ldT = sl_ld(k_last);
    float* cP = cT + (S > 1 ? sub * ldT : 0);
    float* bufA = cP + (S > 1 ? prefix_table_offset(a, S - 1, sub) : 0);
    float* bufB = bufA + 256;
    int* run_start = reinterpret_cast<int*>(fsm + Lo.runs);  // [runs + 1] first execution row of each run
    int* run_src = run_start + f.runs_cap + 1;               // [runs] row-list entry of the run's first row
    const bool stamping = a.phase_ns != nullptr && tid == 0 && split == 0;
    __shared__ int s_fail, s_nruns, s_total;

    fu_stamp(a, h, 0, stamping);
    // the next layer's kernel may be scheduled once every CTA here runs; it
    // waits for this grid's completion before touching memory
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    const int chunk = (ne + J - 1) / J;
    const int c0 = min(ne, split * chunk), c1 = min(ne, c0 + chunk);
    {  // warm L2 for this CTA's inputs while the previous kernel drains
        auto pf = [](const void* ptr) { asm volatile("prefetch.global.L2 [%0];" ::"l"(ptr)); };
        const size_t base = hs * n;
        for (int i = c0 + tid * 32; i < c1; i += FU_THREADS * 32) {
            pf(a.cell_code + base + i);
            pf(a.cell_sizes + base + i);
            if ((i & 127) == 0) pf(a.cell_mask + base + i);
        }
        if (S > 1) {
            const char* sc = reinterpret_cast<const char*>(a.sub_centroids + hs * S * a.kmax * sub);
            const size_t bytes = (size_t)S * a.kmax * sub * 4;
            for (size_t o = (size_t)tid * 128; o < bytes; o += (size_t)FU_THREADS * 128) pf(sc + o);
        }
    }
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    if (f.ap.new_keys && split == J - 1 && wid < 2) append_group(f.ap, h, wid, lid);

    // ---------------- 1. score this CTA's slice ----------------
    const int32_t* sizes = a.cell_sizes + hs * n;
    const uint8_t* mask = a.cell_mask + hs * n;
    const int32_t* code = a.cell_code + hs * n;
    const uint8_t* dirty = a.cell_dirty ? a.cell_dirty + hs * n : nullptr;
    const float* merged = a.centroids + hs * n * (size_t)a.dim;
    const float* subc = a.sub_centroids + hs * (size_t)S * a.kmax * sub;
    if (S > 1) {
        for (int s = 0; s < S; ++s) {
            const int k = a.ks[s];
            float* dst = s == S - 1 ? cT : cP + prefix_table_offset(a, s, sub);
            const int ld = sl_ld(k);
            const float* src = subc + (size_t)s * a.kmax * sub;
            for (int e = tid; e < k * sub; e += FU_THREADS) cp_async4(dst + (e & (sub - 1)) * ld + (e >> sub_shift), src + e);
        }
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
    int ccv[FU_CPT], szv[FU_CPT];
    bool mkv[FU_CPT], dkv[FU_CPT];
#pragma unroll
    for (int j = 0; j < FU_CPT; ++j) {
        const int c = c0 + tid + j * FU_THREADS;
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
    if (tid == 0) s_fail = 0;
    asm volatile("cp.async.wait_all;\n" ::: "memory");
    __syncthreads();
    if (S > 1) {  // prefix table over the first S-1 subspaces (level s chains subspace s onto level s-1)
        int width = 1;
        for (int s = 0; s < S - 1; ++s) {
            const int ks = a.ks[s], ld = sl_ld(ks);
            const int total = width * ks;
            const float* cs = cP + prefix_table_offset(a, s, sub);
            const float* src = s == 0 ? nullptr : (((s - 1) & 1) ? bufB : bufA);
            float* dst = s == S - 2 ? tab : ((s & 1) ? bufB : bufA);
            const float* qq = qs + s * sub;
            for (int e = tid; e < total; e += FU_THREADS) {
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
    {
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
            const float* q2 = qs + (S - 1) * sub;
            if (c1 - c0 <= 2 * FU_THREADS)
                score_chains<2>(acc, sep, il, q2, cT, ldT, sub);
            else
                score_chains<SL_CPT>(acc, sep, il, q2, cT, ldT, sub);
        }
        unsigned long long kmn = ~0ull, kmx = 0ull;
#pragma unroll
        for (int j = 0; j < FU_CPT; ++j) {
            const int c = c0 + tid + j * FU_THREADS;
            if (c >= c1) continue;
            unsigned long long key = 0ull;
            float s = -INFINITY;
            if (cand[j]) {
                if (sep[j]) {
                    s = acc[j];
                } else {  // an updated (or IVF) centroid: the chain over the live merged row
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
            f.keys[hs * n + c] = key;
            f.sizes[hs * n + c] = key ? szv[j] : 0;
            if (a.scores_out) a.scores_out[hs * n + c] = s;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            kmn = min(kmn, (unsigned long long)__shfl_xor_sync(0xffffffffu, kmn, o));
            kmx = max(kmx, (unsigned long long)__shfl_xor_sync(0xffffffffu, kmx, o));
        }
        if (lid == 0) {
            sm.rscr[0][wid] = kmn;
            sm.rscr[1][wid] = kmx;
        }
        __syncthreads();
        if (tid == 0) {
            for (int w = 1; w < FU_WARPS; ++w) {
                kmn = min(kmn, sm.rscr[0][w]);
                kmx = max(kmx, sm.rscr[1][w]);
            }
            f.range[(hs * J + split) * 2 + 0] = kmn;
            f.range[(hs * J + split) * 2 + 1] = kmx;
        }
    }
    if (a.scores_out)
        for (int c = ne + split * FU_THREADS + tid; c < n; c += J * FU_THREADS) a.scores_out[hs * n + c] = -INFINITY;
    fu_stamp(a, h, 1, stamping);

    // ---------------- 2. the group barrier ----------------
    __syncthreads();  // every thread's keys, sizes and range are stored
    if (tid == 0) {
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;\n" ::"l"(f.arrive + h) : "memory");
        unsigned seen = 0, spins = 0;
        while (true) {
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(seen) : "l"(f.arrive + h) : "memory");
            if (seen >= (unsigned)J) break;
            if (++spins > FU_SPIN_LIMIT) {
                s_fail = 1;
                if (at.status) atomicOr(at.status, 2);
                break;
            }
            __nanosleep(32);
        }
    }
    __syncthreads();
    fu_stamp(a, h, 2, stamping);

    // ---------------- 3. both boundaries, in every CTA ----------------
    unsigned long long thrA = ~0ull, thrB = ~0ull;  // no candidates: nothing selected
    int dcount = 0;
    if (!s_fail) {
        const unsigned long long* gk = f.keys + hs * n;
        const int* gz = f.sizes + hs * n;
        for (int c = tid; c < ne; c += FU_THREADS) {
            skey[c] = __ldcg(gk + c);
            ssz[c] = __ldcg(gz + c);
        }
        unsigned long long key_lo0 = ~0ull, key_hi0 = 0ull;
        for (int r = 0; r < J; ++r) {
            key_lo0 = min(key_lo0, __ldcg(f.range + (hs * J + r) * 2 + 0));
            key_hi0 = max(key_hi0, __ldcg(f.range + (hs * J + r) * 2 + 1));
        }
        dcount = a.delta_count ? min(a.delta_count[h], a.delta_capacity) : 0;
        __syncthreads();
        if (key_hi0 != 0ull) {
            const DenseKeys dk{skey, ssz};
            if (search_both<FU_THREADS>(sm, dk, ne, key_lo0, key_hi0, rules)) {
                thrA = sm.T;
                thrB = sm.T2;
            } else {
                search_one<FU_THREADS>(sm, dk, ne, key_lo0, key_hi0, 1, rules);
                thrA = sm.T;
                const bool token_or_rank = sm.flags != 0ull;
                __syncthreads();
                if (token_or_rank) {
                    thrB = thrA;
                } else {
                    search_one<FU_THREADS>(sm, dk, ne, key_lo0, key_hi0, 0, rules);
                    thrB = sm.T;
                }
            }
            __syncthreads();
        }
    }
    fu_stamp(a, h, 3, stamping);

    // ---------------- 4. the execution rows as runs ----------------
    // Slots in contiguous per-thread ranges (slot order = thread order): one
    // scan ranks the selected cells and places their rows.
    const int static_len = a.static_len;
    const int base_run = static_len > 0 ? 1 : 0;
    if (!s_fail) {
        const int per = (ne + FU_THREADS - 1) / FU_THREADS;
        const int e0 = min(ne, tid * per), e1 = min(ne, e0 + per);
        unsigned int nsel = 0, nkept = 0, rows = 0;
        for (int c = e0; c < e1; ++c) {
            const unsigned long long k = skey[c];
            if (k != 0ull && k > thrA) {
                ++nsel;
                rows += (unsigned)ssz[c];
            }
            if (k != 0ull && k > thrB) ++nkept;
        }
        unsigned long long x = ((unsigned long long)nkept << 32) | nsel;
        unsigned int y = rows;
        sl_scan_pair<FU_THREADS>(x, y, sm);  // inclusive
        const unsigned long long xt = sm.red64[FU_WARPS - 1];
        const int tot_sel = (int)(xt & 0xffffffffu), tot_kept = (int)(xt >> 32);
        const int sel_rows = (int)sm.red32[FU_WARPS - 1];
        int my = (int)((x & 0xffffffffu) - nsel);
        int row = static_len + (int)(y - rows);
        const int32_t* offs = a.cell_offsets + hs * (n + 1);
        for (int c = e0; c < e1; ++c) {
            const unsigned long long k = skey[c];
            if (k != 0ull && k > thrA) {
                run_start[base_run + my] = row;
                run_src[base_run + my] = __ldg(offs + c);
                if (split == 0 && my < a.nprobe) a.sel_cells[hs * a.nprobe + my] = c;
                ++my;
                row += ssz[c];
            }
        }
        if (tid == 0 && static_len > 0) {
            run_start[0] = 0;
            run_src[0] = 1 << 30;
        }
        // delta rows whose cell is in the kept list (or the padding id when
        // that list holds a dropped entry), in ring order, after the cells
        int appended = 0;
        const int r0 = base_run + tot_sel;
        if (dcount > 0) {
            const int32_t* dids = a.delta_cell_ids + hs * a.delta_capacity;
            const bool has_pad = tot_kept < a.nprobe;
            for (int base = 0; base < dcount; base += FU_THREADS) {
                const int pidx = base + tid;
                int fl = 0;
                if (pidx < dcount) {
                    const int cid = dids[pidx];
                    if (cid >= 0 && cid < ne) {
                        const unsigned long long k = skey[cid];
                        fl = (k != 0ull && k > thrB) ? 1 : 0;
                    }
                    if (cid == a.padding_id && has_pad) fl = 1;
                }
                int tot;
                const int incl = sl_scan<FU_THREADS>(fl, sm.redi, &tot);
                if (fl) {
                    const int at_ = appended + incl - 1;
                    run_start[r0 + at_] = static_len + sel_rows + at_;
                    run_src[r0 + at_] = (2 << 30) | pidx;
                }
                appended += tot;
            }
        }
        const int total = min(static_len + sel_rows + appended, a.exec_capacity);
        if (tid == 0) {
            s_nruns = r0 + appended;
            s_total = total;
            run_start[r0 + appended] = static_len + sel_rows + appended;
            if (split == 0) {
                a.sel_count[h] = min(tot_sel, a.nprobe);
                if (a.row_count) a.row_count[h] = total;
                if (a.kept_count) a.kept_count[h] = tot_kept;
            }
        }
    } else if (tid == 0) {
        s_nruns = 0;
        s_total = 0;
    }
    __syncthreads();  // the run table is complete; the selection area becomes the ring
    fu_stamp(a, h, 4, stamping);

    // ---------------- 5. attention over this CTA's tiles ----------------
    const int rows_total = s_total, nruns = s_nruns;
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
        const int r = t * AT_TILE + (lid & 15);
        if (t >= ct1 || r >= rows_total) return -1;
        int lo = 0, hi = nruns;  // the last run whose start is <= r
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (run_start[mid] <= r) lo = mid;
            else hi = mid;
        }
        const int e = run_src[lo] + (r - run_start[lo]);
        if (rlist && lid < 16) rlist[r] = e;
        return e;
    };
    attn_stream(at, h, wid, lid, smem_u32(fsm), ct0, ct1, rows_total, qa, entry, m_run, l_run, o);
    fu_stamp(a, h, 5, stamping);
    attn_write_partial(at, h, split, fsm, m_run, l_run, o);
    if (attn_ticket_merge(at, h, fsm)) {
        // every CTA of the group has passed the barrier (each took the ticket
        // after it): re-arm it for the next launch
        if (tid == 0) f.arrive[h] = 0;
        fu_stamp(a, h, 6, tid == 0 && a.phase_ns != nullptr);
    }
}

size_t fused_scratch_bytes(int bg, int n_slots, int splits) {
    auto r = [](size_t x) { return (x + 255) & ~size_t(255); };
    return r((size_t)bg * 4) + r((size_t)bg * n_slots * 8) + r((size_t)bg * n_slots * 4) + r((size_t)bg * splits * 16);
}

int fused_runs_cap(const SelectArgs& s) { return 1 + s.nprobe + (s.delta_count ? s.delta_capacity : 0); }

size_t fused_smem_bytes(const SelectArgs& s) { return fused_layout(s, fused_runs_cap(s)).total; }

// Whether this layer can run as one fused launch: the selection's shared
// memory and the run table fit next to the attention ring, every CTA scores
// at most FU_CPT slots per thread, and the grid is co-resident.
bool fused_eligible(const SelectArgs& s, const AttnArgs& a, size_t scratch_bytes, const char** why) {
    if (!s.fused_scratch) return (*why = "no fused scratch"), false;
    if (scratch_bytes < fused_scratch_bytes(s.bg, s.n_slots, a.splits)) return (*why = "fused scratch too small"), false;
    if (s.cand_out || s.key_base != 0 || a.o_part || a.ml_part || !a.counters)
        return (*why = "sequence-sharding outputs or no merge counters"), false;
    if (fused_smem_bytes(s) > 227 * 1024) return (*why = "selection too large for one CTA"), false;
    const int ne = (s.slot_bound > 0 && s.slot_bound < s.n_slots) ? s.slot_bound : s.n_slots;
    if ((ne + a.splits - 1) / a.splits > FU_CPT * FU_THREADS) return (*why = "too few splits for the slots"), false;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) !=
                                                  cudaSuccess)
        return (*why = "device query failed"), false;
    if ((long long)a.splits * a.bg > sms) return (*why = "more CTAs than SMs"), false;
    return true;
}

cudaError_t launch_decode_fused(const SelectArgs& s, const AttnArgs& a, cudaStream_t st, const AppendArgs* app) {
    FusedArgs f{};
    f.s = s;
    f.a = a;
    if (app) f.ap = *app;
    unsigned char* base = static_cast<unsigned char*>(s.fused_scratch);
    auto r = [](size_t x) { return (x + 255) & ~size_t(255); };
    f.arrive = reinterpret_cast<uint32_t*>(base);
    base += r((size_t)s.bg * 4);
    f.keys = reinterpret_cast<unsigned long long*>(base);
    base += r((size_t)s.bg * s.n_slots * 8);
    f.sizes = reinterpret_cast<int32_t*>(base);
    base += r((size_t)s.bg * s.n_slots * 4);
    f.range = reinterpret_cast<unsigned long long*>(base);
    f.runs_cap = fused_runs_cap(s);
    const size_t sm = fused_layout(s, f.runs_cap).total;
    static int smem_set[64] = {};
    cudaError_t e = ensure_smem(reinterpret_cast<const void*>(&imi_decode_fused_kernel), sm, smem_set, 64);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.splits, a.bg);
    cfg.blockDim = dim3(FU_THREADS);
    cfg.dynamicSmemBytes = sm;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    e = cudaLaunchKernelEx(&cfg, imi_decode_fused_kernel, f);
    if (e != cudaSuccess) {  // a cooperative launch that may not also be programmatic: launch it plainly ordered
        (void)cudaGetLastError();
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, imi_decode_fused_kernel, f);
    }
    return e;
}

}  // namespace imi
