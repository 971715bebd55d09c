// decode.cu -- decode-time kernels of the IMI KV-cache path (sm_100a).
//
//   imi_similarity_kernel   reference-compatible cell scorer over merged fp32
//                           centroids (compute_impl.cu:62-103)
//   (cell selection: select.cu; gather attention: attention.cu)
//   imi_append_kernel       steady-zone append (runtime.py:378-392)
//   imi_async_score_kernel  batched decode-time cell assignment (argmax) and
//   imi_async_finish_kernel running-mean update (async_update.py:77-162)
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
// Steady-zone append: zone[h, pos, :] = new[h, :] for keys and values, and
// (optionally) the async-update batch slot (runtime.py:378-392,
// async_update.py:115-117).  One warp per (group, tensor).
// ----------------------------------------------------------------------------
__global__ void imi_append_kernel(const __grid_constant__ AppendArgs a) {
    // programmatic dependent of the previous kernel: wait for it, then let the
    // next one (the selection) start its launch
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
    const int t = threadIdx.x >> 5;  // 0 = keys, 1 = values
    if (t > 1) return;
    append_group(a, blockIdx.x, t, threadIdx.x & 31);
}

// ----------------------------------------------------------------------------
// Batched decode-time cell assignment and running-mean update
// (async_update.py:122-161).  Inner products follow the d-ordered fma chain
// (separable for unchanged cells, full row for updated ones); ties go to the
// lowest slot (torch.argmax).  Delta sums are added in token order.
//   imi_async_score_kernel  grid (chunks, groups): per-chunk argmax per key
//   imi_async_finish_kernel grid (groups): reduce, delta sums, running mean,
//                           delta ring
// ----------------------------------------------------------------------------
constexpr int ASYNC_CHUNK = 512;
constexpr int ASYNC_BMAX = 64;  // batch limit (checked by the C ABI)

// Leading dimension of a transposed [sub][k] centroid table (odd: a warp
// reading one row at scattered columns spreads over the banks).
__host__ __device__ inline int as_ld(int k) { return (k & 1) ? k + 2 : k + 1; }
__host__ __device__ inline int as_bpad(int B) { return (B + 3) & ~3; }

// Shared-memory plan of the score kernel, in floats: keys transposed
// [dim][bpad], prefix values [B][table], the transposed subspace tables, then
// the per-warp winners (8-byte aligned).
struct AsyncPlan {
    int S, sub, table, bpad;
    size_t kf, tab, tables, total_floats;
    __host__ __device__ AsyncPlan(const AsyncArgs& a) {
        S = a.parts == 0 ? 1 : a.parts;
        sub = a.dim / S;
        table = 1;
        for (int s = 0; s < S - 1; ++s) table *= a.ks[s];
        bpad = as_bpad(a.batch);
        kf = (size_t)a.dim * bpad;
        tab = (size_t)a.batch * table;
        tables = 0;
        if (S > 1)
            for (int s = 0; s < S; ++s) tables += (size_t)sub * as_ld(a.ks[s]);
        total_floats = kf + tab + tables;
    }
};

IMI_DEV void as_cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                 "l"(src)
                 : "memory");
}

__global__ void __launch_bounds__(ASYNC_CHUNK) imi_async_score_kernel(const __grid_constant__ AsyncArgs a) {
    extern __shared__ __align__(16) unsigned char as_smem[];
    const int h = blockIdx.y;
    const int tid = threadIdx.x;
    const AsyncPlan pl(a);
    const int S = pl.S, sub = pl.sub, table = pl.table, bp = pl.bpad;
    const int B = a.batch;
    const size_t hs = h;
    const int k_last = a.ks[S - 1];
    float* kfT = reinterpret_cast<float*>(as_smem);  // [dim][bp]
    float* tab = kfT + pl.kf;                         // [B][table]
    float* cT = tab + pl.tab;                         // last subspace [sub][ld(k_last)]
    const int ldT = as_ld(k_last);
    float* cP = cT + (S > 1 ? (size_t)sub * ldT : 0);  // prefix subspaces back to back
    unsigned long long* wbest = reinterpret_cast<unsigned long long*>(
        (reinterpret_cast<uintptr_t>(kfT + pl.total_floats) + 15) & ~uintptr_t(15));

    // every load up front: the subspace tables by cp.async (transposed), the
    // batch keys and this thread's slot metadata into registers
    const float* subc = a.sub_centroids + hs * (size_t)S * a.kmax * sub;
    int poff[4] = {0, 0, 0, 0};
    if (S > 1) {
        int off = 0;
        for (int s = 0; s < S - 1; ++s) {
            poff[s] = off;
            off += sub * as_ld(a.ks[s]);
        }
        for (int s = 0; s < S; ++s) {
            const int k = a.ks[s], ld = as_ld(k);
            float* dst = s == S - 1 ? cT : cP + poff[s];
            const float* src = subc + (size_t)s * a.kmax * sub;
            for (int e = tid; e < k * sub; e += ASYNC_CHUNK) {
                const int i = e / sub, d = e - i * sub;
                as_cp_async4(dst + d * ld + i, src + e);
            }
        }
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
    const int c = blockIdx.x * ASYNC_CHUNK + tid;
    int cc = -1;
    bool dirty = false;
    if (c < a.n_slots) {
        cc = a.cell_code[hs * a.n_slots + c];
        dirty = a.shadow_dirty && a.shadow_dirty[hs * a.n_slots + c];
    }
    for (int e = tid; e < B * a.dim; e += ASYNC_CHUNK) {
        const int b = e / a.dim, d = e - b * a.dim;
        kfT[d * bp + b] = bf16_bits_to_f32(a.batch_keys[(hs * a.batch_cap + b) * a.dim + d]);
    }
    asm volatile("cp.async.wait_all;\n" ::: "memory");
    __syncthreads();

    // prefix values over the first S-1 subspaces, per key (level by level)
    if (S > 1) {
        int width = 1;
        for (int s = 0; s < S - 1; ++s) {
            const int ks = a.ks[s], ld = as_ld(ks);
            const int total = width * ks;
            const float* cs = cP + poff[s];
            float vals[32];
            int cnt = 0;
            for (int e = tid; e < B * total && cnt < 32; e += ASYNC_CHUNK, ++cnt) {
                const int b = e / total, r = e - b * total;
                const int pi = r / ks, i = r - pi * ks;
                float acc = s == 0 ? 0.0f : tab[(size_t)b * table + pi];
                for (int d = 0; d < sub; ++d) acc = __fmaf_rn(kfT[(s * sub + d) * bp + b], cs[d * ld + i], acc);
                vals[cnt] = acc;
            }
            if (s > 0) __syncthreads();
            cnt = 0;
            for (int e = tid; e < B * total && cnt < 32; e += ASYNC_CHUNK, ++cnt) {
                const int b = e / total, r = e - b * total;
                tab[(size_t)b * table + r] = vals[cnt];
            }
            __syncthreads();
            width = total;
        }
    }

    // One slot per thread, every key of the batch, 16 keys at a time (each
    // centroid column is loaded once for all of them).  A padding slot whose
    // shadow row was never updated holds zeros, and its d-ordered fma chain
    // from +0 stays exactly +0: it scores 0 without a load.  Updated slots (and
    // every slot of a flat index) run the full chain over their shadow row.
    const int lane = tid & 31, w = tid >> 5;
    const bool valid = c < a.n_slots;
    const bool pad = valid && cc < 0 && !dirty;
    const bool full = valid && !pad && (S == 1 || dirty);
    int pidx = 0, il = 0;
    if (valid && !pad && !full) {
        for (int t = 0; t < S - 1; ++t) pidx = pidx * a.ks[t] + ((cc >> (8 * t)) & 0xff);
        il = (cc >> (8 * (S - 1))) & 0xff;
    }
    const float* row = a.shadow + (hs * a.n_slots + (valid ? c : 0)) * (size_t)a.dim;
    for (int b0 = 0; b0 < B; b0 += 16) {
        float acc[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[j] = 0.0f;
        if (full) {
            for (int d = 0; d < a.dim; ++d) {
                const float r = row[d];
                const float4* kv = reinterpret_cast<const float4*>(kfT + d * bp + b0);
#pragma unroll
                for (int j4 = 0; j4 < 4; ++j4) {
                    const float4 k4 = kv[j4];
                    acc[4 * j4 + 0] = __fmaf_rn(k4.x, r, acc[4 * j4 + 0]);
                    acc[4 * j4 + 1] = __fmaf_rn(k4.y, r, acc[4 * j4 + 1]);
                    acc[4 * j4 + 2] = __fmaf_rn(k4.z, r, acc[4 * j4 + 2]);
                    acc[4 * j4 + 3] = __fmaf_rn(k4.w, r, acc[4 * j4 + 3]);
                }
            }
        } else if (valid && !pad) {
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[j] = b0 + j < B ? tab[(size_t)(b0 + j) * table + pidx] : 0.0f;
            const int dk = (S - 1) * sub;
            for (int d = 0; d < sub; ++d) {
                const float r = cT[d * ldT + il];
                const float4* kv = reinterpret_cast<const float4*>(kfT + (dk + d) * bp + b0);
#pragma unroll
                for (int j4 = 0; j4 < 4; ++j4) {
                    const float4 k4 = kv[j4];
                    acc[4 * j4 + 0] = __fmaf_rn(k4.x, r, acc[4 * j4 + 0]);
                    acc[4 * j4 + 1] = __fmaf_rn(k4.y, r, acc[4 * j4 + 1]);
                    acc[4 * j4 + 2] = __fmaf_rn(k4.z, r, acc[4 * j4 + 2]);
                    acc[4 * j4 + 3] = __fmaf_rn(k4.w, r, acc[4 * j4 + 3]);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            if (b0 + j >= B) break;  // uniform over the block
            unsigned long long key =
                valid ? ((unsigned long long)ord_f32(acc[j]) << 32) | (0xffffffffu - (uint32_t)c) : 0ull;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
                key = other > key ? other : key;
            }
            if (lane == 0) wbest[w * B + b0 + j] = key;
        }
    }
    __syncthreads();
    for (int b = tid; b < B; b += blockDim.x) {
        unsigned long long best = 0ull;
        for (int q = 0; q < (int)(blockDim.x >> 5); ++q) best = max(best, wbest[q * B + b]);
        a.part_best[(hs * a.part_chunks + blockIdx.x) * B + b] = best;
    }
}

// One CTA per group.  The batch keys' winning cells; then, per distinct cell
// (first occurrence in token order), its delta sum gains the cell's keys in
// token order and, once its delta count reaches the threshold, the running
// mean replaces its shadow row -- one thread per (cell, d), no sequential walk
// over the batch; then the delta ring.
__global__ void __launch_bounds__(256) imi_async_finish_kernel(AsyncArgs a) {
    const int h = blockIdx.x;
    const int tid = threadIdx.x;
    const int B = a.batch;
    const size_t hs = h;
    __shared__ int ids[ASYNC_BMAX];
    __shared__ int first[ASYNC_BMAX], ucnt[ASYNC_BMAX], dcold[ASYNC_BMAX], cold[ASYNC_BMAX];
    __shared__ float kf[ASYNC_BMAX * 128];
    for (int e = tid; e < B * a.dim; e += blockDim.x) {
        const int b = e / a.dim, d = e - b * a.dim;
        kf[e] = bf16_bits_to_f32(a.batch_keys[(hs * a.batch_cap + b) * a.dim + d]);
    }
    if (tid < B) {
        unsigned long long best = 0ull;
        for (int q = 0; q < a.part_chunks; ++q) best = max(best, a.part_best[(hs * a.part_chunks + q) * B + tid]);
        ids[tid] = (int)(0xffffffffu - (uint32_t)(best & 0xffffffffull));
    }
    __syncthreads();
    if (tid < B) {
        const int cid = ids[tid];
        bool f = true;
        for (int e = 0; e < tid; ++e)
            if (ids[e] == cid) f = false;
        int cnt = 0;
        for (int e = tid; e < B; ++e) cnt += ids[e] == cid;
        first[tid] = f;
        ucnt[tid] = cnt;
        if (f) {
            const size_t cs = hs * a.n_slots + cid;
            dcold[tid] = a.delta_counts[cs];
            cold[tid] = a.counts[cs];
        }
    }
    __syncthreads();
    for (int e = tid; e < B * a.dim; e += blockDim.x) {
        const int b = e / a.dim, d = e - b * a.dim;
        if (!first[b]) continue;
        const int cid = ids[b];
        const size_t cs = hs * a.n_slots + cid;
        float* dsp = a.delta_sums + cs * a.dim + d;
        float ds = *dsp;
        for (int bb = b; bb < B; ++bb)
            if (ids[bb] == cid) ds = __fadd_rn(ds, kf[bb * a.dim + d]);
        const int dc = dcold[b] + ucnt[b];
        if (dc >= a.threshold) {
            const int nc = cold[b] + dc;
            const float denom = (float)max(nc, 1);
            float* rp = a.shadow + cs * a.dim + d;
            *rp = __fdiv_rn(__fadd_rn(__fmul_rn(*rp, (float)cold[b]), ds), denom);
            ds = 0.0f;
        }
        *dsp = ds;
    }
    if (tid < B && first[tid]) {
        const size_t cs = hs * a.n_slots + ids[tid];
        const int dc = dcold[tid] + ucnt[tid];
        if (dc >= a.threshold) {
            a.counts[cs] = cold[tid] + dc;
            a.delta_counts[cs] = 0;
            if (a.shadow_dirty) a.shadow_dirty[cs] = 1;
            if (a.pending) a.pending[cs] = 1;
        } else {
            a.delta_counts[cs] = dc;
        }
    }
    // delta ring (async_update.py:146-161); without ring_store only the write
    // position and count advance, as in the reference (its indexed copy_ lands
    // in a temporary)
    const int wp = a.ring_write_pos[h];
    for (int e = tid; a.ring_store && e < B * (a.dim / 8); e += blockDim.x) {
        const int b = e / (a.dim / 8), q8 = e - b * (a.dim / 8);
        const int pos = (wp + b) % a.ring_cap;
        const uint4* sk = reinterpret_cast<const uint4*>(a.batch_keys + (hs * a.batch_cap + b) * a.dim) + q8;
        const uint4* sv = reinterpret_cast<const uint4*>(a.batch_values + (hs * a.batch_cap + b) * a.dim) + q8;
        reinterpret_cast<uint4*>(a.ring_keys + (hs * a.ring_cap + pos) * a.dim)[q8] = *sk;
        reinterpret_cast<uint4*>(a.ring_values + (hs * a.ring_cap + pos) * a.dim)[q8] = *sv;
    }
    if (a.ring_store && tid < B) a.ring_cell_ids[hs * a.ring_cap + (wp + tid) % a.ring_cap] = ids[tid];
    __syncthreads();
    if (tid == 0) {
        a.ring_write_pos[h] = (wp + B) % a.ring_cap;
        a.ring_count[h] = min(a.ring_count[h] + B, a.ring_cap);
    }
    if (a.ids_out && tid < B) a.ids_out[hs * B + tid] = ids[tid];
}

// Publish the updated cells: live[c] = shadow[c] for slots flagged pending
// (async_update.py:7-19 copies the whole shadow; only changed rows differ).
// Each warp checks 32 slots with one ballot and copies the flagged rows.
__global__ void imi_apply_kernel(ApplyArgs a) {
    const int h = blockIdx.y;
    const size_t hs = h;
    const int lane = threadIdx.x & 31;
    const int c0 = (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 32;
    if (c0 >= a.n_slots) return;
    const int c = c0 + lane;
    const bool pend = c < a.n_slots && a.pending[hs * a.n_slots + c];
    unsigned m = __ballot_sync(0xffffffffu, pend);
    while (m) {
        const int q = __ffs(m) - 1;
        m &= m - 1;
        const size_t cs = hs * a.n_slots + c0 + q;
        for (int d = lane; d < a.dim; d += 32) a.live[cs * a.dim + d] = a.shadow[cs * a.dim + d];
    }
    if (pend) {
        a.pending[hs * a.n_slots + c] = 0;
        a.live_dirty[hs * a.n_slots + c] = 1;
    }
}

// ----------------------------------------------------------------------------
// host launchers
// ----------------------------------------------------------------------------
cudaError_t launch_similarity(const uint16_t* q, const float* cent, float* out, int bg, int G, int n_cells, int dim,
                              long long out_stride, cudaStream_t st) {
    dim3 grid((n_cells + 255) / 256, bg);
    imi_similarity_kernel<<<grid, 256, dim * sizeof(float), st>>>(q, cent, out, G, n_cells, dim, out_stride);
    return cudaGetLastError();
}

cudaError_t launch_append(const AppendArgs& a, cudaStream_t st) {
    return launch_pdl(imi_append_kernel, dim3(a.bg), dim3(64), 0, st, a);
}

size_t async_smem_bytes(const AsyncArgs& a) {
    const AsyncPlan pl(a);
    return sizeof(float) * pl.total_floats + 16 + 8 * (size_t)(ASYNC_CHUNK / 32) * a.batch;
}

int async_chunks(int n_slots) { return (n_slots + ASYNC_CHUNK - 1) / ASYNC_CHUNK; }

cudaError_t launch_async_assign(const AsyncArgs& a, cudaStream_t st) {
    const size_t sm = async_smem_bytes(a);
    static int smem_set[64] = {};
    cudaError_t e = ensure_smem(reinterpret_cast<const void*>(&imi_async_score_kernel), sm, smem_set, 64);
    if (e != cudaSuccess) return e;
    imi_async_score_kernel<<<dim3(a.part_chunks, a.bg), ASYNC_CHUNK, sm, st>>>(a);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    imi_async_finish_kernel<<<a.bg, 256, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_apply(const ApplyArgs& a, cudaStream_t st) {
    const int warps = (a.n_slots + 31) / 32;  // 4 warps (128 slots) per CTA
    imi_apply_kernel<<<dim3((warps + 3) / 4, a.bg), 128, 0, st>>>(a);
    return cudaGetLastError();
}

}  // namespace imi
