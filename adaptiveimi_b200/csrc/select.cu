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
// through DSMEM, with its slice's key range in a per-rank slot (plain stores:
// no shared initial value that remote updates could race with).  The first
// cluster barrier is split (arrive at entry, wait just before the first DSMEM
// store) so it costs nothing.  The leader alone runs the boundary search and
// sends both thresholds to every CTA through DSMEM.  The emission is spread
// over the cluster: each CTA ranks its own slice's selected cells (one block
// scan of per-slot flags), places their rows (a second scan), publishes its
// counts to every CTA, and after one cluster barrier writes its cells and
// rows at the cluster-wide offsets; the leader adds the steady-zone rows, the
// delta rows, the stop marker and the counts.  Only slots below `slot_bound`
// (the occupied compact ids) are scored and scanned.
//
// Code shape matters here: the leader's code runs once per launch, so it is
// kept compact -- plain functions with explicit arguments, one shared copy of
// the boundary resolve, the rare fallback out of line, no local arrays.
#include <cooperative_groups.h>

#include "common.cuh"
#include "imi_internal.h"
#include "select_core.cuh"

namespace cg = cooperative_groups;

namespace imi {

__global__ void __cluster_dims__(SL_CL, 1, 1) __launch_bounds__(SL_THREADS, 1)
    imi_select_kernel(const __grid_constant__ SelectArgs a, const __grid_constant__ AppendArgs ap) {
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
    // slots at or above the bound are padding (masked by construction): they
    // are never candidates, so neither the scoring nor the leader visits them
    const int ne = (a.slot_bound > 0 && a.slot_bound < n) ? a.slot_bound : n;
    const int npad = (n + 1) & ~1;
    SelRules rules;
    rules.nprobe = a.nprobe;
    rules.max_tokens = a.max_tokens;
    rules.buffer_pages = a.buffer_pages;
    rules.page_size = a.page_size;
    rules.pg_shift = __ffs(a.page_size) - 1;
    rules.pg_pow2 = (a.page_size & (a.page_size - 1)) == 0;

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
    // the prefix subspaces back to back, then two scratch buffers for the
    // intermediate prefix levels (S = 4); the leader reuses the region for
    // the selected-cell lists once scoring is over
    float* cT = reinterpret_cast<float*>(p);
    const int ldT = sl_ld(k_last);
    float* cP = cT + (S > 1 ? sub * ldT : 0);
    float* bufA = cP + (S > 1 ? prefix_table_offset(a, S - 1, sub) : 0);
    float* bufB = bufA + 256;
    int* sel_slot = reinterpret_cast<int*>(p);
    int* sel_start = sel_slot + SL_SEL_MAX;
    int* sel_off = sel_start + SL_SEL_MAX;

    const size_t hs = (size_t)h;
    const bool stamping = a.phase_ns != nullptr && tid == 0 && rank == 0;
#define SL_STAMP(k)                                                \
    do {                                                           \
        if (stamping) {                                            \
            unsigned long long t_;                                 \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_)); \
            a.phase_ns[hs * 8 + (k)] = t_;                         \
        }                                                          \
    } while (0)
    SL_STAMP(0);
    // let the attention kernel that follows (a programmatic dependent launch)
    // start setting up on the SMs this kernel leaves free
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    // first half of the cluster barrier that guards the DSMEM stores: every
    // CTA is running
    asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory");
    // While the previous kernel drains, warm L2 (and the address translations)
    // for every input line this CTA will read.  A prefetch returns no data,
    // so it cannot observe anything the previous kernel writes; the loads
    // proper come after the wait below.
    {
        const int chunk0 = (((a.slot_bound > 0 && a.slot_bound < a.n_slots) ? a.slot_bound : a.n_slots) + SL_CL - 1) / SL_CL;
        const int p0 = rank * chunk0;
        const size_t base = (size_t)h * a.n_slots;
        auto pf = [](const void* ptr) { asm volatile("prefetch.global.L2 [%0];" ::"l"(ptr)); };
        // 32 slots per line of the 4-byte arrays, 128 of the byte arrays
        for (int i = tid * 32; i < chunk0; i += SL_THREADS * 32) {
            pf(a.cell_code + base + p0 + i);
            pf(a.cell_sizes + base + p0 + i);
            if (a.row_index) pf(a.cell_offsets + (size_t)h * (a.n_slots + 1) + p0 + i);
            if ((i & 127) == 0) {
                pf(a.cell_mask + base + p0 + i);
                if (a.cell_dirty) pf(a.cell_dirty + base + p0 + i);
            }
        }
        const int S0 = a.parts == 0 ? 1 : a.parts;
        if (S0 > 1) {  // the sub-centroid tables, one line per thread step
            const char* sc = reinterpret_cast<const char*>(a.sub_centroids + (size_t)h * S0 * a.kmax * (a.dim / S0));
            const size_t bytes = (size_t)S0 * a.kmax * (a.dim / S0) * 4;
            for (size_t o = (size_t)tid * 128; o < bytes; o += (size_t)SL_THREADS * 128) pf(sc + o);
        }
        if (tid < (a.G * a.dim * 2 + 127) / 128) pf(reinterpret_cast<const char*>(a.q + (size_t)h * a.G * a.dim) + tid * 128);
    }
    // launched as a programmatic dependent (of the append): everything above
    // overlapped the previous kernel; every global read comes after this
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    // the fused steady-zone append of this group (ap.new_keys set): two warps
    // of the last CTA, which has nothing else to do until the scores
    if (ap.new_keys && rank == SL_CL - 1 && wid < 2) append_group(ap, h, wid, lid);

    const int32_t* sizes = a.cell_sizes + hs * n;
    const uint8_t* mask = a.cell_mask + hs * n;
    const int32_t* code = a.cell_code + hs * n;
    const uint8_t* dirty = a.cell_dirty ? a.cell_dirty + hs * n : nullptr;
    const float* merged = a.centroids + hs * n * (size_t)a.dim;
    const float* subc = a.sub_centroids + hs * (size_t)S * a.kmax * sub;

    // ---------------- every CTA: all global loads at once ----------------
    if (S > 1) {
        for (int s = 0; s < S; ++s) {
            const int k = a.ks[s];
            float* dst = s == S - 1 ? cT : cP + prefix_table_offset(a, s, sub);
            const int ld = sl_ld(k);
            const float* src = subc + (size_t)s * a.kmax * sub;
            const int total = k * sub;
            for (int e = tid; e < total; e += SL_THREADS)
                cp_async4(dst + (e & (sub - 1)) * ld + (e >> sub_shift), src + e);
        }
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
    const int chunk = (ne + SL_CL - 1) / SL_CL;
    const int c0 = rank * chunk;
    const int c1 = min(ne, c0 + chunk);
    int ccv[SL_CPT], szv[SL_CPT], ofv[SL_CPT];
    bool mkv[SL_CPT], dkv[SL_CPT];
    const int32_t* offs = a.cell_offsets + hs * (n + 1);
#pragma unroll
    for (int j = 0; j < SL_CPT; ++j) {
        const int c = c0 + tid + j * SL_THREADS;
        const bool in = c < c1;
        ccv[j] = in ? code[c] : -1;
        mkv[j] = in ? mask[c] != 0 : true;
        szv[j] = in ? sizes[c] : 0;
        dkv[j] = in && dirty ? dirty[c] != 0 : false;
        ofv[j] = in && a.row_index ? offs[c] : 0;  // used by the emission, loaded with the rest
    }
    // the leader's delta-ring inputs, loaded with the rest as well
    const int32_t* dids = a.delta_count ? a.delta_cell_ids + hs * a.delta_capacity : nullptr;
    const int dcount0 = (rank == 0 && a.delta_count) ? a.delta_count[h] : 0;
    const int did0 = (rank == 0 && dids && tid < a.delta_capacity) ? dids[tid] : -1;
    if (tid < a.dim) {
        float acc = 0.0f;
        for (int g = 0; g < a.G; ++g) acc = __fadd_rn(acc, bf16_bits_to_f32(a.q[(hs * a.G + g) * a.dim + tid]));
        qs[tid] = acc;
    }
    asm volatile("cp.async.wait_all;\n" ::: "memory");
    __syncthreads();

    // ---------------- every CTA: prefix table over the first S-1 subspaces ----------------
    // level s chains subspace s from level s-1; the last level lands in tab
    if (S > 1) {
        int width = 1;
        for (int s = 0; s < S - 1; ++s) {
            const int ks = a.ks[s], ld = sl_ld(ks);
            const int total = width * ks;
            const float* cs = cP + prefix_table_offset(a, s, sub);
            const float* src = s == 0 ? nullptr : (((s - 1) & 1) ? bufB : bufA);
            float* dst = s == S - 2 ? tab : ((s & 1) ? bufB : bufA);
            const float* qq = qs + s * sub;
            for (int e = tid; e < total; e += SL_THREADS) {
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
    SL_STAMP(1);

    // ---------------- every CTA: score its slice ----------------
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
        // the number of live cells per thread is uniform over the CTA
        const float* q2 = qs + (S - 1) * sub;
        if (c1 - c0 <= 2 * SL_THREADS)
            score_chains<2>(acc, sep, il, q2, cT, ldT, sub);
        else
            score_chains<SL_CPT>(acc, sep, il, q2, cT, ldT, sub);
    }
    asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
    unsigned long long mykey[SL_CPT];  // this thread's slots' keys (0: not a candidate), kept for the emission
    {
        SelHdr* lead = cluster.map_shared_rank(&sm, 0);
        unsigned long long* lkey = cluster.map_shared_rank(skey, 0);
        int* lsz = cluster.map_shared_rank(ssz, 0);
        unsigned long long kmn = ~0ull, kmx = 0ull;
#pragma unroll
        for (int j = 0; j < SL_CPT; ++j) {
            const int c = c0 + tid + j * SL_THREADS;
            mykey[j] = 0ull;
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
                key = ((unsigned long long)ord_f32(s) << 32) | (0xffffffffu - (uint32_t)(a.key_base + c));
                kmn = min(kmn, key);
                kmx = max(kmx, key);
            }
            lkey[c] = key;
            lsz[c] = key ? szv[j] : 0;
            mykey[j] = key;
            if (a.scores_out) a.scores_out[hs * n + c] = s;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            kmn = min(kmn, (unsigned long long)__shfl_xor_sync(0xffffffffu, kmn, o));
            kmx = max(kmx, (unsigned long long)__shfl_xor_sync(0xffffffffu, kmx, o));
        }
        unsigned long long* wmn = sm.rscr[0];  // [SL_WARPS] minima, then maxima (free until the resolve)
        if (lid == 0) {
            wmn[wid] = kmn;
            wmn[SL_WARPS + wid] = kmx;
        }
        __syncthreads();
        if (tid < 32) {
            unsigned long long m0 = tid < SL_WARPS ? wmn[tid] : ~0ull, m1 = tid < SL_WARPS ? wmn[SL_WARPS + tid] : 0ull;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                m0 = min(m0, (unsigned long long)__shfl_xor_sync(0xffffffffu, m0, o));
                m1 = max(m1, (unsigned long long)__shfl_xor_sync(0xffffffffu, m1, o));
            }
            if (tid == 0) {
                lead->rmin[rank] = m0;
                lead->rmax[rank] = m1;
            }
        }
    }
    if (a.scores_out)
        for (int c = ne + rank * SL_THREADS + tid; c < n; c += SL_CL * SL_THREADS) a.scores_out[hs * n + c] = -INFINITY;
    cluster.sync();  // every score is in the leader
    unsigned long long thrA = ~0ull, thrB = ~0ull;  // no candidates: nothing selected
    if (rank == 0) {
        SL_STAMP(2);
        unsigned long long key_lo0 = ~0ull, key_hi0 = 0ull;
        for (int r = 0; r < SL_CL; ++r) {
            key_lo0 = min(key_lo0, sm.rmin[r]);
            key_hi0 = max(key_hi0, sm.rmax[r]);
        }

        // ---------------- leader: the two boundaries ----------------
        if (key_hi0 != 0ull) {
            const DenseKeys dk{skey, ssz};
            if (search_both(sm, dk, ne, key_lo0, key_hi0, rules)) {
                thrA = sm.T;
                thrB = sm.T2;
            } else {
                search_one(sm, dk, ne, key_lo0, key_hi0, 1, rules);
                thrA = sm.T;
                const bool token_or_rank = sm.flags != 0ull;
                __syncthreads();
                if (token_or_rank) {
                    thrB = thrA;
                } else {
                    search_one(sm, dk, ne, key_lo0, key_hi0, 0, rules);
                    thrB = sm.T;
                }
            }
            __syncthreads();
        }
        SL_STAMP(3);
        if (tid < SL_CL) {  // the thresholds into every CTA
            SelHdr* dst = cluster.map_shared_rank(&sm, tid);
            dst->cthrA = thrA;
            dst->cthrB = thrB;
        }
    }
    cluster.sync();  // the thresholds are everywhere
    thrA = sm.cthrA;
    thrB = sm.cthrB;

    // ---------------- every CTA: its slice's part of the emission ----------------
    // Slot order within the slice is (j, tid).  One block scan of the
    // per-j selected flags (16-bit fields of one word) ranks this thread's
    // slots among the slice's selected cells; the selected cells' sizes then
    // go into a compact list in that order and a second scan places their rows.
    int lsel[SL_CPT];  // slice-local rank of a selected slot (-1: not selected)
    int csel = 0, ckept = 0;
    unsigned long long nxl = 0ull;  // highest-ranked candidate left out in this slice
    {
        unsigned long long x = 0ull;
        unsigned int y = 0u;
#pragma unroll
        for (int j = 0; j < SL_CPT; ++j) {
            const unsigned long long k = mykey[j];
            if (k != 0ull && k > thrA) x |= 1ull << (16 * j);
            if (k != 0ull && k > thrB) ++y;
            if (k != 0ull && k <= thrA) nxl = max(nxl, k);
        }
        const unsigned long long mine = x;
        sl_scan_pair(x, y, sm);  // inclusive; the fields never carry (at most 512 per field)
        const unsigned long long tot = sm.red64[SL_WARPS - 1];
        ckept = (int)sm.red32[SL_WARPS - 1];
        int before = 0;  // selected slots of the earlier j
#pragma unroll
        for (int j = 0; j < SL_CPT; ++j) {
            const int fj = (int)((x >> (16 * j)) & 0xffff), mj = (int)((mine >> (16 * j)) & 1);
            lsel[j] = mj ? before + fj - 1 : -1;
            before += (int)((tot >> (16 * j)) & 0xffff);
        }
        csel = before;
    }
    int* l_start = sel_start;
    int* l_off = sel_off;
    int* l_sz = sel_slot;
#pragma unroll
    for (int j = 0; j < SL_CPT; ++j) {
        if (lsel[j] < 0) continue;
        l_sz[lsel[j]] = szv[j];
        l_off[lsel[j]] = ofv[j];
    }
    __syncthreads();
    int crow = 0;
    {  // row starts of the compact list (slice-local), thread t owns entries 4t .. 4t+3
        int szs[4], loc = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int i = 4 * tid + q;
            szs[q] = i < csel ? l_sz[i] : 0;
            loc += szs[q];
        }
        int run = sl_scan(loc, sm.redi, &crow) - loc;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int i = 4 * tid + q;
            if (i < csel) l_start[i] = run;
            run += szs[q];
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) nxl = max(nxl, (unsigned long long)__shfl_xor_sync(0xffffffffu, nxl, o));
    if (lid == 0) sm.rscr[0][wid] = nxl;
    __syncthreads();
    if (tid < SL_CL) {  // this slice's counts into every CTA
        unsigned long long nx = 0ull;
        for (int q = 0; q < SL_WARPS; ++q) nx = max(nx, sm.rscr[0][q]);
        SelHdr* dst = cluster.map_shared_rank(&sm, tid);
        dst->pc_sel[rank] = csel;
        dst->pc_rows[rank] = crow;
        dst->pc_kept[rank] = ckept;
        dst->pc_nx[rank] = nx;
    }
    cluster.sync();
    int sel_base = 0, row_base = a.static_len, nsel = 0, nkept = 0, sel_rows = 0;
    unsigned long long nx = 0ull;
    for (int r = 0; r < SL_CL; ++r) {
        if (r < rank) {
            sel_base += sm.pc_sel[r];
            row_base += sm.pc_rows[r];
        }
        nsel += sm.pc_sel[r];
        sel_rows += sm.pc_rows[r];
        nkept += sm.pc_kept[r];
        nx = max(nx, sm.pc_nx[r]);
    }
    SL_STAMP(4);
    unsigned long long* rec = a.cand_out ? a.cand_out + hs * (2 * (size_t)(a.nprobe + 1) + 1) : nullptr;
    int32_t* rows = a.row_index ? a.row_index + hs * (size_t)a.exec_capacity : nullptr;
#pragma unroll
    for (int j = 0; j < SL_CPT; ++j) {
        if (lsel[j] < 0) continue;
        const int my = sel_base + lsel[j];
        if (my < a.nprobe) {
            a.sel_cells[hs * a.nprobe + my] = c0 + tid + j * SL_THREADS;
            if (rec) {
                rec[my] = mykey[j];
                rec[a.nprobe + 1 + my] = (unsigned long long)szv[j];
            }
        }
    }
    if (rows) {
        for (int i = wid; i < csel; i += SL_WARPS) {
            const int s0 = row_base + l_start[i], off = l_off[i], sz = l_sz[i];
            for (int jj = lid; jj < sz; jj += 32)
                if (s0 + jj < a.exec_capacity) rows[s0 + jj] = off + jj;
        }
    }
    if (rank != 0) return;

    // ---------------- leader: stop marker, static and delta rows, counts ----------------
    if (tid == 0 && rec) {  // the stop marker after the selected cells, then the count
        const int ns = min(nsel, a.nprobe);
        if (nx) {
            const int slot = (int)(0xffffffffu - (uint32_t)nx) - a.key_base;
            rec[ns] = nx;
            rec[a.nprobe + 1 + ns] = (unsigned long long)ssz[slot];
        }
        rec[2 * (a.nprobe + 1)] = (unsigned long long)(ns + (nx ? 1 : 0));
    }
    if (!rows) {  // candidates only (the sharded merge writes the rows)
        if (tid == 0) {
            a.sel_count[h] = min(nsel, a.nprobe);
            if (a.kept_count) a.kept_count[h] = nkept;
        }
        return;
    }
    const int static_len = a.static_len;
    for (int r = tid; r < static_len; r += SL_THREADS) rows[r] = (1 << 30) | r;
    int total = min(static_len + sel_rows, a.exec_capacity);
    if (a.delta_count) {
        const int dcount = min(dcount0, a.delta_capacity);
        const bool has_pad = nkept < a.nprobe;
        int appended = 0;
        for (int base = 0; base < dcount; base += SL_THREADS) {
            const int pidx = base + tid;
            int f = 0;
            if (pidx < dcount) {
                const int cid = base == 0 ? did0 : dids[pidx];
                if (cid >= 0 && cid < ne) {
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
    SL_STAMP(5);
#undef SL_STAMP
    if (tid == 0) {
        a.sel_count[h] = min(nsel, a.nprobe);
        a.row_count[h] = total;
        if (a.kept_count) a.kept_count[h] = nkept;
    }
}

// ---------------------------------------------------------------------------
// Sequence sharding: the global selection over every shard's candidates.
// One CTA per group.  The candidates (keys carry global cell ids, so every
// shard orders them alike) are loaded into shared memory, the two boundaries
// are found exactly as in the per-shard selection, and this shard's cells
// above boundary A become its selected cells and its row list.  A shard's
// part of the global selection is a prefix of its own order, so its local
// selection under the global rules plus its stop marker cover it.
// ---------------------------------------------------------------------------
// Whether the merge copies every candidate into shared memory (otherwise it
// searches the records in global memory, where they arrived).
constexpr int MERGE_LIST = 8192;  // boundary-bucket candidates the non-dense merge refines in shared memory
__host__ __device__ inline bool merge_dense(const MergeArgs& a) {
    return (size_t)a.shards * a.cap <= 8192;
}

// list_k / list_s (list_cap entries, shared memory, or null): room for the
// boundary bucket's candidates when the first round cannot resolve it.
template <class Keys>
IMI_DEV void merge_select(const MergeArgs& a, SelHdr& sm, const Keys& keys, int ne, int* sel_start, int* sel_off,
                          const SelRules& rules, unsigned long long* list_k = nullptr, int* list_s = nullptr,
                          int list_cap = 0) {
    const int h = blockIdx.x;
    const int tid = threadIdx.x, wid = tid >> 5, lid = tid & 31;
    const size_t hs = h;
    unsigned long long kmn = ~0ull, kmx = 0ull;
    for_candidates(keys, ne, [&](unsigned long long k, int) {
        kmn = min(kmn, k);
        kmx = max(kmx, k);
    });
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
    unsigned long long key_lo0 = ~0ull, key_hi0 = 0ull;
    for (int q = 0; q < SL_WARPS; ++q) {
        key_lo0 = min(key_lo0, sm.rscr[0][q]);
        key_hi0 = max(key_hi0, sm.rscr[1][q]);
    }
    __syncthreads();
    unsigned long long thrA = ~0ull;
    if (key_hi0 != 0ull) {
        if (search_both(sm, keys, ne, key_lo0, key_hi0, rules)) {
            thrA = sm.T;
        } else if (list_k != nullptr && sm.first < SL_NB && sm.bcnt <= list_cap) {
            // Boundary A's first-round bucket is too full to resolve at once:
            // copy its candidates into shared memory and refine there, from
            // the first round's totals above that bucket, instead of passing
            // over every record again per round.
            const int bA = sm.bucket;
            const long long qc = sm.pre[0], qs = sm.pre[1], qp = sm.pre[2];
            __shared__ int s_nl;
            if (tid == 0) s_nl = 0;
            __syncthreads();
            const float smin = sl_key_score(key_lo0), smax = sl_key_score(key_hi0);
            const float scale = smax > smin ? (float)(SL_NB - 1) / (smax - smin) : 0.0f;
            unsigned long long lmn = ~0ull, lmx = 0ull;
            for_candidates(keys, ne, [&](unsigned long long k, int z) {
                if (min(SL_NB - 1, max(0, (int)((sl_key_score(k) - smin) * scale))) != bA) return;
                const int at = atomicAdd(&s_nl, 1);
                list_k[at] = k;
                list_s[at] = z;
                lmn = min(lmn, k);
                lmx = max(lmx, k);
            });
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                lmn = min(lmn, (unsigned long long)__shfl_xor_sync(0xffffffffu, lmn, o));
                lmx = max(lmx, (unsigned long long)__shfl_xor_sync(0xffffffffu, lmx, o));
            }
            if (lid == 0) {
                sm.rscr[0][wid] = lmn;
                sm.rscr[1][wid] = lmx;
            }
            __syncthreads();
            unsigned long long llo = ~0ull, lhi = 0ull;
            for (int q = 0; q < SL_WARPS; ++q) {
                llo = min(llo, sm.rscr[0][q]);
                lhi = max(lhi, sm.rscr[1][q]);
            }
            const int nl = s_nl;
            __syncthreads();
            search_one(sm, DenseKeys{list_k, list_s}, nl, llo, lhi, 1, rules, qc, qs, qp);
            thrA = sm.T;
        } else {
            search_one(sm, keys, ne, key_lo0, key_hi0, 1, rules);
            thrA = sm.T;
        }
        __syncthreads();
    }

    // this shard's candidates sit in slot order at [rank * cap, rank * cap + count)
    const size_t rec_len = 2 * (size_t)a.cap + 1;
    const int base = a.rank * a.cap;
    const int cnt = (int)a.cand[((size_t)a.rank * a.bg + hs) * rec_len + 2 * a.cap];
    const int per = (cnt + SL_THREADS - 1) / SL_THREADS;  // contiguous entries per thread
    const int e0 = min(cnt, tid * per), e1 = min(cnt, e0 + per);
    unsigned int nloc = 0, sloc = 0;
    for (int e = e0; e < e1; ++e) {
        const unsigned long long k = keys.key(base + e);
        if (k != 0ull && k > thrA) {
            ++nloc;
            sloc += (unsigned)keys.size(base + e);
        }
    }
    unsigned long long ix = nloc;
    unsigned int iy = sloc;
    sl_scan_pair(ix, iy, sm);
    if (tid == SL_THREADS - 1) {
        sm.wsel[0] = (int)ix;
        sm.wkept[0] = (int)iy;
    }
    const int32_t* offs = a.cell_offsets + hs * (a.n_slots + 1);
    {
        int my = (int)(ix - nloc);
        int run = a.static_len + (int)(iy - sloc);
        for (int e = e0; e < e1; ++e) {
            const unsigned long long k = keys.key(base + e);
            if (k != 0ull && k > thrA) {
                const int slot = (int)(0xffffffffu - (uint32_t)k) - a.key_base;
                if (my < a.nprobe) a.sel_cells[hs * a.nprobe + my] = slot;
                sel_start[my] = run;  // my < cnt <= cap: the lists hold cap entries
                sel_off[my] = offs[slot];
                ++my;
                run += keys.size(base + e);
            }
        }
    }
    __syncthreads();
    const int ntot = sm.wsel[0], rows_sel = sm.wkept[0];
    int32_t* rows = a.row_index + hs * (size_t)a.exec_capacity;
    for (int r = tid; r < a.static_len; r += SL_THREADS) rows[r] = (1 << 30) | r;
    for (int i = wid; i < ntot; i += SL_WARPS) {
        const int s0 = sel_start[i], off = sel_off[i];
        const int sz = (i + 1 < ntot ? sel_start[i + 1] : a.static_len + rows_sel) - s0;
        for (int jj = lid; jj < sz; jj += 32)
            if (s0 + jj < a.exec_capacity) rows[s0 + jj] = off + jj;
    }
    if (tid == 0) {
        a.sel_count[h] = min(ntot, a.nprobe);
        a.row_count[h] = min(a.static_len + rows_sel, a.exec_capacity);
    }
}

__global__ void __launch_bounds__(SL_THREADS, 1) imi_merge_kernel(const __grid_constant__ MergeArgs a) {
    extern __shared__ __align__(16) unsigned char dyn[];
    SelHdr& sm = *reinterpret_cast<SelHdr*>(dyn);
    const int h = blockIdx.x;
    const int tid = threadIdx.x;
    const size_t hs = h;
    const int ne = a.shards * a.cap;
    const bool dense = merge_dense(a);
    const int npad = dense ? (ne + 1) & ~1 : 0;
    unsigned char* p = dyn + ((sizeof(SelHdr) + 15) & ~size_t(15));
    unsigned long long* skey = reinterpret_cast<unsigned long long*>(p);
    p += sizeof(unsigned long long) * npad;
    int* ssz = reinterpret_cast<int*>(p);
    p += sizeof(int) * npad;
    int* counts = reinterpret_cast<int*>(p);  // [shards]
    p += sizeof(int) * ((a.shards + 3) & ~3);
    int* sel_start = reinterpret_cast<int*>(p);  // [cap]
    int* sel_off = sel_start + a.cap;            // [cap]
    p += 2 * sizeof(int) * (((size_t)a.cap + 1) & ~size_t(1));
    // non-dense: room for one first-round bucket's candidates
    unsigned long long* list_k = dense ? nullptr : reinterpret_cast<unsigned long long*>(p);  // [MERGE_LIST]
    int* list_s = dense ? nullptr : reinterpret_cast<int*>(list_k + MERGE_LIST);             // [MERGE_LIST]
    SelRules rules;
    rules.nprobe = a.nprobe;
    rules.max_tokens = a.max_tokens;
    rules.buffer_pages = a.buffer_pages;
    rules.page_size = a.page_size;
    rules.pg_shift = __ffs(a.page_size) - 1;
    rules.pg_pow2 = (a.page_size & (a.page_size - 1)) == 0;

    const size_t rec_len = 2 * (size_t)a.cap + 1;
    for (int sh = tid; sh < a.shards; sh += SL_THREADS)
        counts[sh] = min(a.cap, (int)a.cand[((size_t)sh * a.bg + hs) * rec_len + 2 * a.cap]);
    __syncthreads();
    const RecordKeys rk{a.cand + hs * rec_len, (size_t)a.bg * rec_len, a.cap, counts};
    if (dense) {
        for (int e = tid; e < ne; e += SL_THREADS) {
            const unsigned long long k = rk.key(e);
            skey[e] = k;
            ssz[e] = k ? rk.size(e) : 0;
        }
        __syncthreads();
        merge_select(a, sm, DenseKeys{skey, ssz}, ne, sel_start, sel_off, rules);
    } else {
        merge_select(a, sm, rk, ne, sel_start, sel_off, rules, list_k, list_s, MERGE_LIST);
    }
}

// ---------------------------------------------------------------------------
// Cluster merge (shards <= 8): CTA r of a group's cluster holds shard r's
// candidate record in its own shared memory.  Every CTA histograms its own
// candidates over the common score range; the leader sums the histograms
// through DSMEM and finds the bucket where a rule fires; the CTAs hand the
// leader that bucket's candidates through DSMEM; the leader resolves the
// boundary (refining in shared memory when the bucket is large) and the CTA
// holding this rank's shard writes its selected cells and row list.  Each CTA
// touches one shard's candidates, so the passes are 1/shards of a one-CTA
// merge's.
// ---------------------------------------------------------------------------
__host__ __device__ inline int cmerge_list_cap(int cap) {
    // what is left of 227 KB after the header, the shard's candidates and the emission lists
    const long long used = ((long long)sizeof(SelHdr) + 15) / 16 * 16 + 12LL * cap + 8LL * cap + 256;
    const long long room = (long long)(227 * 1024 - 1024) - used;
    return (int)(room > 12 * 32 ? room / 12 : 32);
}

size_t cmerge_smem_bytes(const MergeArgs& a) {
    return ((sizeof(SelHdr) + 15) & ~size_t(15)) + 12 * (size_t)a.cap + 8 * (size_t)a.cap + 256 +
           12 * (size_t)cmerge_list_cap(a.cap);
}

__global__ void __launch_bounds__(SL_THREADS, 1) imi_merge_cluster_kernel(const __grid_constant__ MergeArgs a) {
    extern __shared__ __align__(16) unsigned char dyn[];
    SelHdr& sm = *reinterpret_cast<SelHdr*>(dyn);
    cg::cluster_group cluster = cg::this_cluster();
    const int r = (int)cluster.block_rank();  // = the shard this CTA holds
    const int h = blockIdx.y;
    const int tid = threadIdx.x, wid = tid >> 5, lid = tid & 31;
    const size_t hs = h;
    const int cap = a.cap, list_cap = cmerge_list_cap(cap);
    unsigned char* p = dyn + ((sizeof(SelHdr) + 15) & ~size_t(15));
    unsigned long long* ck = reinterpret_cast<unsigned long long*>(p);  // [cap] this shard's keys
    p += 8 * (size_t)cap;
    int* cs = reinterpret_cast<int*>(p);  // [cap] sizes
    p += 4 * (size_t)cap;
    int* sel_start = reinterpret_cast<int*>(p);  // [cap]
    int* sel_off = sel_start + cap;              // [cap]
    p += 8 * (size_t)cap;
    p = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(p) + 255) & ~uintptr_t(255));
    unsigned long long* list_k = reinterpret_cast<unsigned long long*>(p);  // [list_cap] leader
    int* list_s = reinterpret_cast<int*>(list_k + list_cap);
    __shared__ unsigned long long c_lo[SL_CL], c_hi[SL_CL];  // leader: every CTA's key range
    __shared__ int c_bucket, c_nl, c_counts[SL_CL];
    __shared__ unsigned long long c_thr;
    SelRules rules;
    rules.nprobe = a.nprobe;
    rules.max_tokens = a.max_tokens;
    rules.buffer_pages = a.buffer_pages;
    rules.page_size = a.page_size;
    rules.pg_shift = __ffs(a.page_size) - 1;
    rules.pg_pow2 = (a.page_size & (a.page_size - 1)) == 0;

    // ---- this shard's candidates (entries in slot order) and their key range
    const size_t rec_len = 2 * (size_t)cap + 1;
    const unsigned long long* rec = a.cand + ((size_t)r * a.bg + hs) * rec_len;
    const int cnt = min(cap, (int)rec[2 * (size_t)cap]);
    unsigned long long kmn = ~0ull, kmx = 0ull;
    for (int j = tid; j < cnt; j += SL_THREADS) {
        const unsigned long long k = __ldcg(rec + j);
        ck[j] = k;
        cs[j] = (int)__ldcg(rec + cap + j);
        if (k) {
            kmn = min(kmn, k);
            kmx = max(kmx, k);
        }
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
    hist_clear(sm);  // (its barrier also publishes rscr)
    if (tid == 0) {
        unsigned long long lo = ~0ull, hi = 0ull;
        for (int q = 0; q < SL_WARPS; ++q) {
            lo = min(lo, sm.rscr[0][q]);
            hi = max(hi, sm.rscr[1][q]);
        }
        unsigned long long* llo = cluster.map_shared_rank(c_lo, 0);
        unsigned long long* lhi = cluster.map_shared_rank(c_hi, 0);
        llo[r] = lo;
        lhi[r] = hi;
        cluster.map_shared_rank(c_counts, 0)[r] = cnt;
        if (r == 0) c_nl = 0;
    }
    cluster.sync();  // #1: every range is in the leader
    unsigned long long key_lo0 = ~0ull, key_hi0 = 0ull;
    {
        const unsigned long long* llo = cluster.map_shared_rank(c_lo, 0);
        const unsigned long long* lhi = cluster.map_shared_rank(c_hi, 0);
        for (int q = 0; q < (int)cluster.num_blocks(); ++q) {
            key_lo0 = min(key_lo0, llo[q]);
            key_hi0 = max(key_hi0, lhi[q]);
        }
    }
    const float smin = sl_key_score(key_lo0), smax = sl_key_score(key_hi0);
    const float scale = smax > smin ? (float)(SL_NB - 1) / (smax - smin) : 0.0f;
    auto bin = [&](unsigned long long k) { return min(SL_NB - 1, max(0, (int)((sl_key_score(k) - smin) * scale))); };
    if (key_hi0 != 0ull) {
        for (int j = tid; j < cnt; j += SL_THREADS)
            if (ck[j]) hist_add(sm, bin(ck[j]), cs[j], rules);
    }
    cluster.sync();  // #2: every local histogram is complete
    if (key_hi0 != 0ull) {
        // the cluster's histogram, each CTA summing a share of the buckets
        // over every CTA into the leader's list area (free until #3)
        const int nb = (int)cluster.num_blocks();
        const int per = (SL_NB + nb - 1) / nb;
        unsigned long long* lsum = cluster.map_shared_rank(list_k, 0);                      // [SL_NB]
        unsigned int* lsz = reinterpret_cast<unsigned int*>(cluster.map_shared_rank(list_k, 0) + SL_NB);
        for (int b = r * per + tid; b < min(SL_NB, (r + 1) * per); b += SL_THREADS) {
            unsigned long long x = 0ull;
            unsigned int w = 0u;
            for (int q = 0; q < nb; ++q) {
                const SelHdr* o = cluster.map_shared_rank(&sm, q);
                x += o->hcp[b];
                w += o->hsz[b];
            }
            lsum[b] = x;
            lsz[b] = w;
        }
    }
    cluster.sync();  // #2b: the summed histogram is in the leader
    if (r == 0 && key_hi0 != 0ull) {
        const unsigned int* lsz = reinterpret_cast<const unsigned int*>(list_k + SL_NB);
        for (int b = tid; b < SL_NB; b += SL_THREADS) {
            sm.hcp[b] = list_k[b];
            sm.hsz[b] = lsz[b];
        }
        __syncthreads();
        BucketView v;
        hist_view(sm, 0, 0, 0, v);
        {
            long long ec = v.ec, es = v.es, ep = v.ep;
            bool done = false;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                if (!done && v.cv[q] > 0 &&
                    ((ec + v.cv[q] > rules.nprobe) || (es + v.sv[q] >= rules.max_tokens) ||
                     (ep + v.pv[q] > rules.buffer_pages))) {
                    atomicMin(&sm.first, 4 * tid + q);
                    done = true;
                }
                ec += v.cv[q];
                es += v.sv[q];
                ep += v.pv[q];
            }
        }
        __syncthreads();
        const int fr = sm.first;
        if (fr < SL_NB && (fr >> 2) == tid) view_publish(v, fr, &sm.bucket, &sm.bcnt, sm.pre);
        __syncthreads();
        if (tid < (int)cluster.num_blocks())
            *cluster.map_shared_rank(&c_bucket, tid) = fr < SL_NB ? sm.bucket : -1;
    }
    if (r == 0 && key_hi0 == 0ull && tid < (int)cluster.num_blocks()) *cluster.map_shared_rank(&c_bucket, tid) = -1;
    cluster.sync();  // #3: the boundary bucket is known everywhere
    const int bA = c_bucket;
    if (bA >= 0) {  // that bucket's candidates into the leader's list
        int* lnl = cluster.map_shared_rank(&c_nl, 0);
        unsigned long long* lk = cluster.map_shared_rank(list_k, 0);
        int* ls = cluster.map_shared_rank(list_s, 0);
        for (int j = tid; j < cnt; j += SL_THREADS) {
            const unsigned long long k = ck[j];
            if (k == 0ull || bin(k) != bA) continue;
            const int at = atomicAdd(lnl, 1);
            if (at < list_cap) {
                lk[at] = k;
                ls[at] = cs[j];
            }
        }
    }
    cluster.sync();  // #4: the list is complete
    if (r == 0) {
        unsigned long long thr = ~0ull;  // no candidates: nothing selected
        if (key_hi0 != 0ull) {
            if (bA < 0) {
                thr = key_lo0 > 0 ? key_lo0 - 1 : 0ull;  // no rule fires: every candidate is selected
            } else if (c_nl <= list_cap) {
                const int nl = c_nl;
                unsigned long long lmn = ~0ull, lmx = 0ull;
                for (int i = tid; i < nl; i += SL_THREADS) {
                    lmn = min(lmn, list_k[i]);
                    lmx = max(lmx, list_k[i]);
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    lmn = min(lmn, (unsigned long long)__shfl_xor_sync(0xffffffffu, lmn, o));
                    lmx = max(lmx, (unsigned long long)__shfl_xor_sync(0xffffffffu, lmx, o));
                }
                if (lid == 0) {
                    sm.rscr[0][wid] = lmn;
                    sm.rscr[1][wid] = lmx;
                }
                __syncthreads();
                unsigned long long llo = ~0ull, lhi = 0ull;
                for (int q = 0; q < SL_WARPS; ++q) {
                    llo = min(llo, sm.rscr[0][q]);
                    lhi = max(lhi, sm.rscr[1][q]);
                }
                const long long qc = sm.pre[0], qs = sm.pre[1], qp = sm.pre[2];
                __syncthreads();
                if (nl <= 32) {
                    if (wid == 0)
                        resolve_boundary(list_k, list_s, nl, qc, qs, qp, 1, llo, sm.rscr[0], rules, &sm.T, &sm.flags);
                } else {
                    search_one(sm, DenseKeys{list_k, list_s}, nl, llo, lhi, 1, rules, qc, qs, qp);
                }
                __syncthreads();
                thr = sm.T;
            } else {  // a bucket larger than the list: search every record in global memory
                const RecordKeys rk{a.cand + hs * rec_len, (size_t)a.bg * rec_len, cap, c_counts};
                search_one(sm, rk, (int)cluster.num_blocks() * cap, key_lo0, key_hi0, 1, rules);
                __syncthreads();
                thr = sm.T;
            }
        }
        if (tid == 0) *cluster.map_shared_rank(&c_thr, a.rank) = thr;
    }
    cluster.sync();  // #5: the threshold is with this rank's shard
    if (r != a.rank) return;
    const unsigned long long thrA = c_thr;

    // ---- this rank's shard: its selected cells (slot order) and row list
    const int per = (cnt + SL_THREADS - 1) / SL_THREADS;  // contiguous entries per thread
    const int e0 = min(cnt, tid * per), e1 = min(cnt, e0 + per);
    unsigned int nloc = 0, sloc = 0;
    for (int e = e0; e < e1; ++e) {
        const unsigned long long k = ck[e];
        if (k != 0ull && k > thrA) {
            ++nloc;
            sloc += (unsigned)cs[e];
        }
    }
    unsigned long long ix = nloc;
    unsigned int iy = sloc;
    sl_scan_pair(ix, iy, sm);
    if (tid == SL_THREADS - 1) {
        sm.wsel[0] = (int)ix;
        sm.wkept[0] = (int)iy;
    }
    const int32_t* offs = a.cell_offsets + hs * (a.n_slots + 1);
    {
        int my = (int)(ix - nloc);
        int run = a.static_len + (int)(iy - sloc);
        for (int e = e0; e < e1; ++e) {
            const unsigned long long k = ck[e];
            if (k != 0ull && k > thrA) {
                const int slot = (int)(0xffffffffu - (uint32_t)k) - a.key_base;
                if (my < a.nprobe) a.sel_cells[hs * a.nprobe + my] = slot;
                sel_start[my] = run;
                sel_off[my] = offs[slot];
                ++my;
                run += cs[e];
            }
        }
    }
    __syncthreads();
    const int ntot = sm.wsel[0], rows_sel = sm.wkept[0];
    int32_t* rows = a.row_index + hs * (size_t)a.exec_capacity;
    for (int q = tid; q < a.static_len; q += SL_THREADS) rows[q] = (1 << 30) | q;
    for (int i = wid; i < ntot; i += SL_WARPS) {
        const int s0 = sel_start[i], off = sel_off[i];
        const int sz = (i + 1 < ntot ? sel_start[i + 1] : a.static_len + rows_sel) - s0;
        for (int jj = lid; jj < sz; jj += 32)
            if (s0 + jj < a.exec_capacity) rows[s0 + jj] = off + jj;
    }
    if (tid == 0) {
        a.sel_count[h] = min(ntot, a.nprobe);
        a.row_count[h] = min(a.static_len + rows_sel, a.exec_capacity);
    }
}

size_t merge_smem_bytes(const MergeArgs& a) {
    const size_t ne = (size_t)a.shards * a.cap;
    const size_t npad = merge_dense(a) ? (ne + 1) & ~size_t(1) : 0;
    return ((sizeof(SelHdr) + 15) & ~size_t(15)) + 12 * npad + 4 * (((size_t)a.shards + 3) & ~size_t(3)) +
           2 * sizeof(int) * (((size_t)a.cap + 1) & ~size_t(1)) + (merge_dense(a) ? 0 : 12 * (size_t)MERGE_LIST) + 16;
}

cudaError_t launch_merge(const MergeArgs& a, cudaStream_t st) {
    // the cluster merge (its list area also carries the summed histogram: at least SL_NB entries)
    if (a.shards <= SL_CL && cmerge_list_cap(a.cap) >= SL_NB && cmerge_smem_bytes(a) <= 227 * 1024) {
        const size_t smc = cmerge_smem_bytes(a);
        static int cset[64] = {};
        cudaError_t e = ensure_smem(reinterpret_cast<const void*>(&imi_merge_cluster_kernel), smc, cset, 64);
        if (e != cudaSuccess) return e;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(a.shards, a.bg);
        cfg.blockDim = dim3(SL_THREADS);
        cfg.dynamicSmemBytes = smc;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = a.shards;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, imi_merge_cluster_kernel, a);
    }
    const size_t sm = merge_smem_bytes(a);
    static int smem_set[64] = {};
    cudaError_t e = ensure_smem(reinterpret_cast<const void*>(&imi_merge_kernel), sm, smem_set, 64);
    if (e != cudaSuccess) return e;
    imi_merge_kernel<<<a.bg, SL_THREADS, sm, st>>>(a);
    return cudaGetLastError();
}

size_t select_smem_bytes(const SelectArgs& a) {
    const int S = a.parts == 0 ? 1 : a.parts;
    int table = 1;
    for (int s = 0; s < S - 1; ++s) table *= a.ks[s];
    const int sub = a.dim / S;
    size_t tables = 0;
    if (S > 1) {
        for (int s = 0; s < S; ++s) tables += (size_t)sub * sl_ld(a.ks[s]) * sizeof(float);
        // intermediate prefix levels (S = 4): level 0 (<= 255) and level 1
        if (S > 2) tables += (256 + (size_t)a.ks[0] * a.ks[1]) * sizeof(float);
    }
    const size_t lists = 3 * (size_t)SL_SEL_MAX * sizeof(int);  // reused for the selected-cell lists
    const size_t region = tables > lists ? tables : lists;
    const size_t npad = ((size_t)a.n_slots + 1) & ~size_t(1);
    return ((sizeof(SelHdr) + 15) & ~size_t(15)) + 12 * npad + sizeof(float) * ((size_t)a.dim + table + 4) + region +
           16;
}

int select_max_slots() { return SL_MAX_SLOTS; }

cudaError_t launch_select(const SelectArgs& a, cudaStream_t st, const AppendArgs* app) {
    const size_t sm = select_smem_bytes(a);
    static int smem_set[64] = {};
    cudaError_t e = ensure_smem(reinterpret_cast<const void*>(&imi_select_kernel), sm, smem_set, 64);
    if (e != cudaSuccess) return e;
    AppendArgs none{};
    return launch_pdl(imi_select_kernel, dim3(SL_CL, a.bg), dim3(SL_THREADS), sm, st, a, app ? *app : none);
}

}  // namespace imi
