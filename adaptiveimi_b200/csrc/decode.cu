// decode.cu -- decode-time kernels of the IMI KV-cache path (sm_100a).
//
//   imi_similarity_kernel   reference-compatible cell scorer over merged fp32
//                           centroids (compute_impl.cu:62-103)
//   (cell selection: select.cu; gather attention: attention.cu)
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
// Batched decode-time cell assignment and running-mean update
// (async_update.py:122-161).  Inner products follow the d-ordered fma chain
// (separable for unchanged cells, full row for updated ones); ties go to the
// lowest slot (torch.argmax).  Delta sums are added in token order.
//   imi_async_score_kernel  grid (chunks, groups): per-chunk argmax per key
//   imi_async_finish_kernel grid (groups): reduce, delta sums, running mean,
//                           delta ring
// ----------------------------------------------------------------------------
constexpr int ASYNC_CHUNK = 512;

__global__ void __launch_bounds__(ASYNC_CHUNK) imi_async_score_kernel(AsyncArgs a) {
    extern __shared__ __align__(16) unsigned char as_smem[];
    const int h = blockIdx.y;
    const int tid = threadIdx.x;
    const int S = a.parts == 0 ? 1 : a.parts;
    const int sub = a.dim / S;
    const int B = a.batch;
    const size_t hs = h;
    int table = 1;
    for (int s = 0; s < S - 1; ++s) table *= a.ks[s];
    const int k_last = a.ks[S - 1];
    float* kf = reinterpret_cast<float*>(as_smem);                  // [B][dim]
    float* tab = kf + (size_t)B * a.dim;                            // [B][table]
    float* cT = tab + (size_t)B * table;                            // [sub][k_last+1] (S > 1)
    unsigned long long* wbest = reinterpret_cast<unsigned long long*>(
        (reinterpret_cast<uintptr_t>(cT + (S > 1 ? (size_t)sub * (k_last + 1) : 0)) + 15) & ~uintptr_t(15));
    for (int e = tid; e < B * a.dim; e += blockDim.x) {
        const int b = e / a.dim, d = e - b * a.dim;
        kf[e] = bf16_bits_to_f32(a.batch_keys[(hs * a.batch_cap + b) * a.dim + d]);
    }
    const float* subc = a.sub_centroids + hs * (size_t)S * a.kmax * sub;
    if (S > 1) {
        const float* cl = subc + (size_t)(S - 1) * a.kmax * sub;
        for (int e = tid; e < k_last * sub; e += blockDim.x) {
            const int i = e / sub, d = e - i * sub;
            cT[d * (k_last + 1) + i] = cl[(size_t)i * sub + d];
        }
        for (int b = tid; b < B; b += blockDim.x) tab[(size_t)b * table] = 0.0f;
    }
    __syncthreads();
    if (S > 1) {
        int width = 1;
        for (int s = 0; s < S - 1; ++s) {
            const int ks = a.ks[s];
            const int total = width * ks;
            const float* cs = subc + (size_t)s * a.kmax * sub;
            float vals[32];
            int cnt = 0;
            for (int e = tid; e < B * total && cnt < 32; e += blockDim.x, ++cnt) {
                const int b = e / total, r = e - b * total;
                const int pi = r / ks, i = r - pi * ks;
                float acc = tab[(size_t)b * table + pi];
                for (int d = 0; d < sub; ++d) acc = __fmaf_rn(kf[b * a.dim + s * sub + d], cs[(size_t)i * sub + d], acc);
                vals[cnt] = acc;
            }
            __syncthreads();
            cnt = 0;
            for (int e = tid; e < B * total && cnt < 32; e += blockDim.x, ++cnt) {
                const int b = e / total, r = e - b * total;
                tab[(size_t)b * table + r] = vals[cnt];
            }
            __syncthreads();
            width = total;
        }
    }
    // one slot per thread, every key of the batch
    const int c = blockIdx.x * ASYNC_CHUNK + tid;
    const int lane = tid & 31, w = tid >> 5;
    const float* shadow = a.shadow + hs * a.n_slots * (size_t)a.dim;
    int cc = -1, pidx = 0, il = 0;
    bool full = true;
    if (c < a.n_slots) {
        cc = a.cell_code[hs * a.n_slots + c];
        full = (S == 1 || cc < 0 || (a.shadow_dirty && a.shadow_dirty[hs * a.n_slots + c]));
        if (!full) {
            for (int t = 0; t < S - 1; ++t) pidx = pidx * a.ks[t] + ((cc >> (8 * t)) & 0xff);
            il = (cc >> (8 * (S - 1))) & 0xff;
        }
    }
    for (int b = 0; b < B; ++b) {
        unsigned long long key = 0ull;
        if (c < a.n_slots) {
            float s;
            if (full) {
                const float* row = shadow + (size_t)c * a.dim;
                s = 0.0f;
                for (int d = 0; d < a.dim; ++d) s = __fmaf_rn(kf[b * a.dim + d], row[d], s);
            } else {
                s = tab[(size_t)b * table + pidx];
                const float* kq = kf + b * a.dim + (S - 1) * sub;
#pragma unroll 8
                for (int d = 0; d < sub; ++d) s = __fmaf_rn(kq[d], cT[d * (k_last + 1) + il], s);
            }
            key = ((unsigned long long)ord_f32(s) << 32) | (0xffffffffu - (uint32_t)c);
        }
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
            key = other > key ? other : key;
        }
        if (lane == 0) wbest[w * B + b] = key;
    }
    __syncthreads();
    for (int b = tid; b < B; b += blockDim.x) {
        unsigned long long best = 0ull;
        for (int q = 0; q < (int)(blockDim.x >> 5); ++q) best = max(best, wbest[q * B + b]);
        a.part_best[(hs * a.part_chunks + blockIdx.x) * B + b] = best;
    }
}

__global__ void __launch_bounds__(256) imi_async_finish_kernel(AsyncArgs a) {
    const int h = blockIdx.x;
    const int tid = threadIdx.x;
    const int B = a.batch;
    const size_t hs = h;
    __shared__ int ids[64];
    __shared__ float kf[64 * 128];
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
    // running mean for cells that reached the threshold; each touched cell once
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
cudaError_t launch_similarity(const uint16_t* q, const float* cent, float* out, int bg, int G, int n_cells, int dim,
                              long long out_stride, cudaStream_t st) {
    dim3 grid((n_cells + 255) / 256, bg);
    imi_similarity_kernel<<<grid, 256, dim * sizeof(float), st>>>(q, cent, out, G, n_cells, dim, out_stride);
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
    const size_t ct = S > 1 ? (size_t)(a.dim / S) * (a.ks[S - 1] + 1) : 0;
    return sizeof(float) * ((size_t)a.batch * a.dim + (size_t)a.batch * table + ct) + 16 +
           8 * (size_t)(ASYNC_CHUNK / 32) * a.batch + 64;
}

int async_chunks(int n_slots) { return (n_slots + ASYNC_CHUNK - 1) / ASYNC_CHUNK; }

cudaError_t launch_async_assign(const AsyncArgs& a, cudaStream_t st) {
    const size_t sm = async_smem_bytes(a);
    cudaError_t e = cudaFuncSetAttribute(imi_async_score_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) return e;
    imi_async_score_kernel<<<dim3(a.part_chunks, a.bg), ASYNC_CHUNK, sm, st>>>(a);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    imi_async_finish_kernel<<<a.bg, 256, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_apply(const ApplyArgs& a, cudaStream_t st) {
    imi_apply_kernel<<<dim3(min(a.n_slots, 256), a.bg), 128, 0, st>>>(a);
    return cudaGetLastError();
}

}  // namespace imi
