// attention.cu -- split-K gather attention over the execution row list
// (sm_100a).  The semantics are those of weighted_flash_decoding as the
// reference calls it (retrieval.py:439-447): per KV group, softmax(scale *
// q.K^T) V over the group's rows for its G query heads; the data movement is
// that of Copy.gather_copy_and_concat (gather_copy.cu:100-213) fused in, so the
// selected rows are read once, straight from the HBM-resident lists.
//
// Grid (splits, groups); 8 warps per CTA, one CTA per SM.  A CTA owns a
// contiguous range of the group's rows.  It first resolves every row's source
// address into shared memory, then each warp streams 16-row tiles through a
// 3-deep cp.async ring (16-byte chunks XOR-swizzled by row so ldmatrix is
// conflict-free), computes S = Q K^T and O += P V with mma.sync m16n8k16
// (query heads on M: G <= 8 of the 16 rows are live), and keeps an online
// softmax in exp2 space.  The warps merge through shared memory; the CTA
// writes one (m, l, o) partial; the last CTA of a group (an atomic counter
// that it re-zeroes) merges the partials into the bf16 output, or a separate
// merge kernel does when no counter buffer is given.
//
// Why mma.sync and not tcgen05: with G = 4..8 query heads per KV group the
// product has M <= 8 against tcgen05's minimum M of 64, and the kernel moves
// 512 bytes per row for 4 * 128 * 2 multiply-adds -- it is bound by HBM, and
// the tensor instruction only has to keep the instruction count per byte low.
#include <mutex>
#include <string>

#include "common.cuh"
#include "imi_internal.h"

namespace imi {

constexpr int AT_WARPS = 8;
constexpr int AT_STAGES = 3;
constexpr int AT_TILE = 16;                            // rows per tile
constexpr int AT_ROWB = 256;                           // bytes per row (dim 128, bf16)
constexpr int AT_STAGE_BYTES = 2 * AT_TILE * AT_ROWB;  // K + V
constexpr int AT_RING_BYTES = AT_WARPS * AT_STAGES * AT_STAGE_BYTES;

IMI_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

IMI_DEV void cp_async16(uint32_t dst, const void* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes));
}
IMI_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
IMI_DEV void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}
IMI_DEV void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
IMI_DEV void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
IMI_DEV void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
IMI_DEV uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

// Source of a row-list entry: the key row's address with the source (0 list,
// 1 steady zone, 2 delta ring) in the low two bits (rows are 16-byte aligned);
// 0 when the entry has no backing buffer.
IMI_DEV unsigned long long row_key_addr(const AttnArgs& a, int h, int idx) {
    const unsigned src = (unsigned)idx >> 30;
    const long long row = idx & 0x3fffffff;
    const unsigned char* b;
    long long stride;
    if (src == 0) {
        b = reinterpret_cast<const unsigned char*>(a.list_keys);
        stride = a.list_rows;
    } else if (src == 1) {
        b = reinterpret_cast<const unsigned char*>(a.static_keys);
        stride = a.static_rows;
    } else {
        b = reinterpret_cast<const unsigned char*>(a.delta_keys);
        stride = a.delta_rows;
    }
    if (!b) return 0ull;
    return reinterpret_cast<unsigned long long>(b + ((long long)h * stride + row) * AT_ROWB) | src;
}

__global__ void __launch_bounds__(AT_WARPS * 32, 1) imi_attn_kernel(AttnArgs a) {
    extern __shared__ __align__(128) unsigned char att_smem[];
    const int h = blockIdx.y;
    const int split = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;
    const int rows_total = a.row_count[h];
    int chunk = (rows_total + a.splits - 1) / a.splits;
    chunk = (chunk + AT_TILE - 1) & ~(AT_TILE - 1);
    const int r0 = split * chunk;
    const int r1 = min(rows_total, r0 + chunk);
    const int nrows = max(0, r1 - r0);
    const int ntiles = (nrows + AT_TILE - 1) / AT_TILE;

    // row sources for the whole range, resolved once
    unsigned long long* rptr = reinterpret_cast<unsigned long long*>(att_smem + AT_RING_BYTES);
    {
        const int32_t* ridx = a.row_index + (size_t)h * a.exec_capacity + r0;
        for (int r = threadIdx.x; r < ntiles * AT_TILE; r += blockDim.x)
            rptr[r] = r < nrows ? row_key_addr(a, h, ridx[r]) : 0ull;
    }
    const long long vdiff0 = reinterpret_cast<const unsigned char*>(a.list_values) -
                             reinterpret_cast<const unsigned char*>(a.list_keys);
    const long long vdiff1 = reinterpret_cast<const unsigned char*>(a.static_values) -
                             reinterpret_cast<const unsigned char*>(a.static_keys);
    const long long vdiff2 = a.delta_keys ? reinterpret_cast<const unsigned char*>(a.delta_values) -
                                                reinterpret_cast<const unsigned char*>(a.delta_keys)
                                          : 0ll;
    __syncthreads();

    const uint32_t wbuf = smem_u32(att_smem) + warp * AT_STAGES * AT_STAGE_BYTES;
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
    const int my_tiles = ntiles > warp ? (ntiles - warp + AT_WARPS - 1) / AT_WARPS : 0;
    const int ch = lane & 15;
    const int half = lane >> 4;

    // copy tile `it` of this warp: lane copies chunk `ch` of rows 2j+half (K and V)
    auto issue = [&](int it) {
        const int t = warp + it * AT_WARPS;
        const uint32_t sb = wbuf + (it % AT_STAGES) * AT_STAGE_BYTES;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = 2 * j + half;
            const unsigned long long e = rptr[t * AT_TILE + i];
            const unsigned src = (unsigned)(e & 3ull);
            const unsigned char* kp = reinterpret_cast<const unsigned char*>(e & ~3ull);
            const long long vd = src == 0 ? vdiff0 : (src == 1 ? vdiff1 : vdiff2);
            const int nb = e ? 16 : 0;
            const unsigned char* ks = e ? kp + ch * 16 : reinterpret_cast<const unsigned char*>(a.q);
            const unsigned char* vs = e ? kp + vd + ch * 16 : reinterpret_cast<const unsigned char*>(a.q);
            const uint32_t dst = sb + i * AT_ROWB + ((ch ^ (i & 7)) << 4);
            cp_async16(dst, ks, nb);
            cp_async16(dst + AT_TILE * AT_ROWB, vs, nb);
        }
    };

#pragma unroll
    for (int it = 0; it < AT_STAGES - 1; ++it) {
        if (it < my_tiles) issue(it);
        cp_async_commit();
    }
    for (int it = 0; it < my_tiles; ++it) {
        if (it + AT_STAGES - 1 < my_tiles) issue(it + AT_STAGES - 1);
        cp_async_commit();
        cp_async_wait<AT_STAGES - 1>();
        __syncwarp();
        const int t = warp + it * AT_WARPS;
        const uint32_t kb = wbuf + (it % AT_STAGES) * AT_STAGE_BYTES;
        const uint32_t vb = kb + AT_TILE * AT_ROWB;
        float s0[4] = {0, 0, 0, 0}, s1[4] = {0, 0, 0, 0};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int row = (lane & 7) + ((lane >> 4) << 3);
            const int cc = 2 * j + ((lane >> 3) & 1);
            uint32_t b0, b1, b2, b3;
            ldsm_x4(kb + row * AT_ROWB + ((cc ^ (row & 7)) << 4), b0, b1, b2, b3);
            mma_bf16(s0, qa[j][0], 0u, qa[j][1], 0u, b0, b1);
            mma_bf16(s1, qa[j][0], 0u, qa[j][1], 0u, b2, b3);
        }
        const int rb = t * AT_TILE;  // relative to r0
        float x[4];
        x[0] = (rb + 2 * c < nrows) ? s0[0] * sl2 : -INFINITY;
        x[1] = (rb + 2 * c + 1 < nrows) ? s0[1] * sl2 : -INFINITY;
        x[2] = (rb + 8 + 2 * c < nrows) ? s1[0] * sl2 : -INFINITY;
        x[3] = (rb + 9 + 2 * c < nrows) ? s1[1] * sl2 : -INFINITY;
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
            if (alpha != 1.0f) {
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                    o[u][0] *= alpha;
                    o[u][1] *= alpha;
                }
            }
            m_run = m_new;
        }
        const uint32_t pa0 = pack_bf16(pr[0], pr[1]);
        const uint32_t pa2 = pack_bf16(pr[2], pr[3]);
#pragma unroll
        for (int u = 0; u < 16; u += 2) {
            const int row = (lane & 7) + (((lane >> 3) & 1) << 3);
            const int cc = u + (lane >> 4);
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(vb + row * AT_ROWB + ((cc ^ (row & 7)) << 4), b0, b1, b2, b3);
            mma_bf16(o[u], pa0, 0u, pa2, 0u, b0, b1);
            mma_bf16(o[u + 1], pa0, 0u, pa2, 0u, b2, b3);
        }
        __syncwarp();
    }
    cp_async_wait<0>();
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
    __syncthreads();
    // merge the warps through shared memory
    float* sm_m = reinterpret_cast<float*>(att_smem);  // [warps][8]
    float* sm_l = sm_m + AT_WARPS * 8;                  // [warps][8]
    float* sm_o = sm_l + AT_WARPS * 8;                  // [warps][8][128]
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
        for (int w = 0; w < AT_WARPS; ++w) M = fmaxf(M, sm_m[w * 8 + gg]);
        float acc = 0.0f, L = 0.0f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < AT_WARPS; ++w) {
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
    if (!a.counters) return;  // a separate merge launch follows
    // the last CTA of this group merges the split partials (the counter self-resets)
    __shared__ int s_last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = (atomicAdd(&a.counters[h], 1) == a.splits - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const size_t hb = (size_t)h * a.splits * a.G;
    for (int e = threadIdx.x; e < a.G * 128; e += blockDim.x) {
        const int gg = e >> 7, d = e & 127;
        float M = -INFINITY;
        for (int q = 0; q < a.splits; ++q) M = fmaxf(M, __ldcg(&a.part_ml[(hb + (size_t)q * a.G + gg) * 2]));
        float acc = 0.0f, L = 0.0f;
        if (M != -INFINITY) {
            for (int q = 0; q < a.splits; ++q) {
                const size_t pb = hb + (size_t)q * a.G + gg;
                const float f = exp2f(__ldcg(&a.part_ml[pb * 2]) - M);
                acc += __ldcg(&a.part_o[pb * 128 + d]) * f;
                L += __ldcg(&a.part_ml[pb * 2 + 1]) * f;
            }
        }
        const float r = L > 0.0f ? acc / L : 0.0f;
        reinterpret_cast<__nv_bfloat16*>(a.out)[((size_t)h * a.G + gg) * 128 + d] = __float2bfloat16_rn(r);
    }
    if (threadIdx.x == 0) a.counters[h] = 0;
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

size_t attn_smem_bytes(const AttnArgs& a) {
    int chunk = (a.exec_capacity + a.splits - 1) / a.splits;
    chunk = (chunk + AT_TILE - 1) & ~(AT_TILE - 1);
    return (size_t)AT_RING_BYTES + (size_t)chunk * 8;
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t st) {
    const size_t sm = attn_smem_bytes(a);
    cudaError_t e = cudaFuncSetAttribute(imi_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) return e;
    imi_attn_kernel<<<dim3(a.splits, a.bg), AT_WARPS * 32, sm, st>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess || a.counters) return e;
    imi_combine_kernel<<<a.bg, 512, 0, st>>>(a);
    return cudaGetLastError();
}

}  // namespace imi

// ---------------------------------------------------------------------------
// imi_sparse_attention_noalloc: the same attention, with its scratch (split
// partials and merge counters) in a fixed array that the library owns.
//
// For callers that cannot call cudaMalloc at all -- for example code running
// under an allocator that must not be re-entered, inside a host callback, or
// in a runtime that forbids device allocation once set up -- and so cannot
// provide part_o / part_ml / counters.  The array below is created when the
// library is loaded on a device and lives until the process exits (every GPU
// that loads the library holds IMI_NOALLOC_SCRATCH_BYTES of it).
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_attn_scratch[IMI_NOALLOC_SCRATCH_BYTES];

namespace {

std::mutex g_scratch_mu;
void* g_scratch_ptr[128] = {};

// Device address of g_attn_scratch for the current device.  The name is only
// a host-side stand-in, so the address is asked of the runtime, once per
// device, with that device current.
cudaError_t scratch_address(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_attn_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return cudaSuccess;
}

size_t round256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace

extern "C" IMI_API int imi_sparse_attention_noalloc(const imi_attn_desc* desc, void* stream) {
    if (!desc) {
        imi::set_last_error("imi_sparse_attention_noalloc: null descriptor");
        return IMI_ERR_INVALID;
    }
    if (desc->bg <= 0 || desc->G <= 0 || desc->splits <= 0) {
        imi::set_last_error("imi_sparse_attention_noalloc: bg, G and splits must be positive");
        return IMI_ERR_INVALID;
    }
    const size_t groups = (size_t)desc->bg * desc->splits * desc->G;
    const size_t need = round256((size_t)desc->bg * 4) + round256(groups * 2 * 4) + groups * 128 * 4;
    if (need > IMI_NOALLOC_SCRATCH_BYTES) {
        imi::set_last_error("imi_sparse_attention_noalloc: bg * splits * G needs " + std::to_string(need) +
                            " bytes of scratch; the fixed array holds " +
                            std::to_string((size_t)IMI_NOALLOC_SCRATCH_BYTES) +
                            " (lower splits or use imi_sparse_attention)");
        return IMI_ERR_INVALID;
    }
    void* base = nullptr;
    cudaError_t e = scratch_address(&base);
    if (e != cudaSuccess) {
        imi::set_last_error(std::string("imi_sparse_attention_noalloc: cudaGetSymbolAddress: ") +
                            cudaGetErrorString(e));
        return IMI_ERR_CUDA;
    }
    unsigned char* p = static_cast<unsigned char*>(base);
    imi_attn_desc d = *desc;
    d.counters = reinterpret_cast<int32_t*>(p);
    d.part_ml = reinterpret_cast<float*>(p + round256((size_t)desc->bg * 4));
    d.part_o = reinterpret_cast<float*>(p + round256((size_t)desc->bg * 4) + round256(groups * 2 * 4));
    // the merge counters must start at zero; the array keeps the last call's contents
    e = cudaMemsetAsync(d.counters, 0, (size_t)desc->bg * 4, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) {
        imi::set_last_error(std::string("imi_sparse_attention_noalloc: ") + cudaGetErrorString(e));
        return IMI_ERR_CUDA;
    }
    return imi_sparse_attention(&d, stream);
}
