// attention.cu -- split-K gather attention over the execution row list
// (sm_100a).  The semantics are those of weighted_flash_decoding as the
// reference calls it (retrieval.py:439-447): per KV group, softmax(scale *
// q.K^T) V over the group's rows for its G query heads; the data movement is
// that of Copy.gather_copy_and_concat (gather_copy.cu:100-213) fused in, so the
// selected rows are read once, straight from the HBM-resident lists.
//
// Grid (splits, groups); 8 warps per CTA, one CTA per SM.  A CTA owns a
// contiguous share of the group's 16-row tiles; its warps read the tiles'
// row-list entries two tiles ahead.  Each warp streams 16-row tiles (K and V, 8 KB) through a
// 3-deep ring of 16-byte cp.async pieces, half a warp per 256-byte row, so
// the copies ride the ordinary load path (per-row bulk copies were bound by
// the copy engine's request rate at about 33 GB/s per SM).  Rows sit at a
// 272-byte pitch so the eight rows of an ldmatrix fall on distinct banks.  The warp computes S = Q K^T and
// O += P V with mma.sync m16n8k16 (query heads on M: G <= 8 of the 16 rows are
// live) and keeps an online softmax in exp2 space.  The warps merge through
// shared memory; the CTA writes one (m, l, o) partial; the last CTA of a group
// (an atomic counter that it re-zeroes) merges the partials into the bf16
// output, or a separate merge kernel does when no counter buffer is given.
// The kernel has no spin-waits (cp.async groups complete in hardware).
//
// The kernel is launched as a programmatic dependent (PDL) of the kernel
// before it in the stream: its CTAs set up their barriers while that kernel
// (normally the selection) drains, and wait for it before reading memory.
//
// Why mma.sync and not tcgen05: with G = 4..8 query heads per KV group the
// product has M <= 8 against tcgen05's minimum M of 64, and the kernel moves
// 512 bytes per row for 4 * 128 * 2 multiply-adds -- it is bound by HBM, and
// the tensor instruction only has to keep the instruction count per byte low.
#include <mutex>
#include <string>

#include "attn_core.cuh"
#include "common.cuh"
#include "imi_internal.h"

namespace imi {

#ifdef ATT_STAMPS  // profiling aid: globaltimer per CTA phase past the partials (part_o is sized twice)
#define ATT_STAMP(k)                                                                                    \
    do {                                                                                                \
        if (threadIdx.x == 0) {                                                                         \
            unsigned long long t_;                                                                      \
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                      \
            reinterpret_cast<unsigned long long*>(a.part_o + (size_t)a.bg * a.splits * a.G * 128)      \
                [((size_t)blockIdx.y * a.splits + blockIdx.x) * 8 + (k)] = t_;                          \
        }                                                                                               \
    } while (0)
#else
#define ATT_STAMP(k) \
    do {             \
    } while (0)
#endif

__global__ void __launch_bounds__(AT_WARPS * 32, 1) imi_attn_kernel(AttnArgs a) {
    extern __shared__ __align__(128) unsigned char att_smem[];
    const int h = blockIdx.y;
    const int split = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t ring = smem_u32(att_smem);
    // Launched as a programmatic dependent of the select kernel: everything
    // above overlaps its tail; every global read comes after this wait.
    ATT_STAMP(0);
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    ATT_STAMP(1);
    // the next layer's append (a programmatic dependent) may start launching
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");

    const int rows_total = a.row_count[h];
    const int gtiles = (rows_total + AT_TILE - 1) / AT_TILE;  // the group's 16-row tiles
    // CTA `split` owns a contiguous share of the group's tiles; its warps take
    // every AT_WARPS-th tile of it.  (Taking tiles from a per-group atomic
    // counter instead balanced the CTAs but cost more in contention than it
    // saved.)
    int ct0, ct1;
    {
        const int per = (gtiles + a.splits - 1) / a.splits;
        ct0 = min(gtiles, split * per);
        ct1 = min(gtiles, ct0 + per);
    }
    const int32_t* rlist = a.row_index + (size_t)h * a.exec_capacity;
    uint32_t qa[8][2];
    attn_load_q(a, h, lane, qa);
    float m_run = -INFINITY, l_run = 0.0f;
    float o[16][4];
#pragma unroll
    for (int u = 0; u < 16; ++u) o[u][0] = o[u][1] = o[u][2] = o[u][3] = 0.0f;
    // the row-list entry of this lane's row of tile t (-1: no row)
    auto entry = [&](int t) -> int {
        const int r = t * AT_TILE + (lane & 15);
        return (t < ct1 && r < rows_total) ? rlist[r] : -1;
    };
    ATT_STAMP(2);
    attn_stream(a, h, warp, lane, ring, ct0, ct1, rows_total, qa, entry, m_run, l_run, o);
    ATT_STAMP(3);
    attn_write_partial(a, h, split, att_smem, m_run, l_run, o);
    ATT_STAMP(4);
    if (!a.counters) return;  // a separate merge launch follows
    if (attn_ticket_merge(a, h, att_smem)) ATT_STAMP(6);
    else ATT_STAMP(5);
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

// Sequence sharding: log-sum-exp combine of the shards' partials, one CTA per
// group, one thread per float4 column of the [G][128] output.
__global__ void imi_combine_shards_kernel(const __grid_constant__ CombineArgs a) {
    const int h = blockIdx.x;
    const int col = threadIdx.x;
    if (col >= a.G * 32) return;
    const int gg = col >> 5, d4 = col & 31;
    float M = -INFINITY;
    const size_t ps = a.part_stride ? (size_t)a.part_stride : (size_t)a.bg * a.G * 128;
    const size_t ms = a.part_stride ? (size_t)a.part_stride : (size_t)a.bg * a.G * 2;
    for (int s = 0; s < a.shards; ++s) M = fmaxf(M, a.ml_parts[s * ms + ((size_t)h * a.G + gg) * 2]);
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    float L = 0.0f;
    if (M != -INFINITY) {
        for (int s = 0; s < a.shards; ++s) {
            const size_t pg = (size_t)h * a.G + gg;
            const float f = exp2f(a.ml_parts[s * ms + pg * 2] - M);
            const float4 v = reinterpret_cast<const float4*>(a.o_parts + s * ps + pg * 128)[d4];
            acc.x += v.x * f;
            acc.y += v.y * f;
            acc.z += v.z * f;
            acc.w += v.w * f;
            L += a.ml_parts[s * ms + pg * 2 + 1] * f;
        }
    }
    const float inv = L > 0.0f ? 1.0f / L : 0.0f;
    uint2 packed;
    packed.x = pack_bf16(acc.x * inv, acc.y * inv);
    packed.y = pack_bf16(acc.z * inv, acc.w * inv);
    *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(a.out) + ((size_t)h * a.G + gg) * 128 + 4 * d4) = packed;
}

cudaError_t launch_combine_shards(const CombineArgs& a, cudaStream_t st) {
    imi_combine_shards_kernel<<<a.bg, a.G * 32, 0, st>>>(a);
    return cudaGetLastError();
}

size_t attn_smem_bytes(const AttnArgs&) { return (size_t)AT_RING_BYTES; }

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t st) {
    const size_t sm = attn_smem_bytes(a);
    static int smem_set[64] = {};
    cudaError_t e = ensure_smem(reinterpret_cast<const void*>(&imi_attn_kernel), sm, smem_set, 64);
    if (e != cudaSuccess) return e;
    // programmatic dependent launch: the CTAs may start (barrier set-up) while
    // the kernel before them in the stream finishes; they wait for it with
    // griddepcontrol.wait before their first global read
    e = launch_pdl(imi_attn_kernel, dim3(a.splits, a.bg), dim3(AT_WARPS * 32), sm, st, a);
    if (e != cudaSuccess) return e;
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
// per device: the context the address was looked up in, and the address
void* g_scratch_ctx[128] = {};
void* g_scratch_ptr[128] = {};

typedef int (*CtxGetCurrentFn)(void**);

// The current driver context (the primary context under the runtime API), or
// null when the entry point is unavailable.
void* current_context() {
    static CtxGetCurrentFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<CtxGetCurrentFn>(p);
        else
            (void)cudaGetLastError();
    }
    void* ctx = nullptr;
    if (fn && fn(&ctx) != 0) ctx = nullptr;
    return ctx;
}

// Device address of g_attn_scratch for the current device.  The name is only
// a host-side stand-in, so the address is asked of the runtime with that
// device current: once per device, and again whenever the device's context
// has changed since (after cudaDeviceReset the module, and with it the array,
// is loaded anew at another address).
cudaError_t scratch_address(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 128) return cudaErrorInvalidDevice;
    // null before the runtime has made a context current: the lookup below
    // does that, and the next call caches against the context
    void* ctx = current_context();
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_ptr[dev] || ctx == nullptr || ctx != g_scratch_ctx[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_attn_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_ptr[dev] = p;
        g_scratch_ctx[dev] = ctx;
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
