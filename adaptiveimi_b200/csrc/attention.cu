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

#include "common.cuh"
#include "imi_internal.h"

namespace imi {

constexpr int AT_WARPS = 8;
constexpr int AT_STAGES = 3;
constexpr int AT_TILE = 16;                              // rows per tile
constexpr int AT_ROWB = 256;                             // bytes per row in HBM (dim 128, bf16)
constexpr int AT_PITCH = 272;                            // bytes per row in shared memory: the 16-byte pad
                                                         // puts the 8 rows of an ldmatrix on distinct banks
constexpr int AT_STAGE_BYTES = 2 * AT_TILE * AT_PITCH;   // K tile + V tile
constexpr int AT_RING_BYTES = AT_WARPS * AT_STAGES * AT_STAGE_BYTES;

IMI_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

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

// Address of a row-list entry's key (kv = 0) or value (kv = 1) row; the top
// two bits of the entry name the source (0 list, 1 steady zone, 2 delta ring).
// NULL when that source has no buffer.
IMI_DEV const unsigned char* row_src(const AttnArgs& a, int h, int idx, int kv) {
    const unsigned src = (unsigned)idx >> 30;
    const long long row = idx & 0x3fffffff;
    const void* b;
    long long stride;
    if (src == 0) {
        b = kv ? a.list_values : a.list_keys;
        stride = a.list_rows;
    } else if (src == 1) {
        b = kv ? a.static_values : a.static_keys;
        stride = a.static_rows;
    } else if (src == 2) {
        b = kv ? a.delta_values : a.delta_keys;
        stride = a.delta_rows;
    } else {
        return nullptr;
    }
    if (!b) return nullptr;
    return reinterpret_cast<const unsigned char*>(b) + ((long long)h * stride + row) * AT_ROWB;
}

__global__ void __launch_bounds__(AT_WARPS * 32, 1) imi_attn_kernel(AttnArgs a) {
    extern __shared__ __align__(128) unsigned char att_smem[];
    const int h = blockIdx.y;
    const int split = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;
    const uint32_t ring = smem_u32(att_smem);
    // Launched as a programmatic dependent of the select kernel: everything
    // above overlaps its tail; every global read comes after this wait.
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
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
    const uint32_t wring = ring + warp * AT_STAGES * AT_STAGE_BYTES;
    const int tlimit = ct1;  // tiles at or past this are not this CTA's
    // the row-list entry of this lane's row of tile t (-1: no row)
    auto entry = [&](int t) -> int {
        const int r = t * AT_TILE + (lane & 15);
        return (t < tlimit && r < rows_total) ? rlist[r] : -1;
    };

    // Issue tile t into stage st.  Lane l holds the row-list entry of row
    // (l & 15) of the tile; lanes 0-15 resolve the K rows, 16-31 the V rows.
    // The rows are copied in 16-byte cp.async pieces, half a warp per row
    // (256 contiguous bytes), two rows per warp instruction.  Rows past the
    // range or without a source buffer are zero-filled (a past-the-range row
    // is also masked out of the softmax; a sourceless one counts as a zero row).
    auto issue = [&](int ent, int st) {
        const unsigned char* src = row_src(a, h, ent, lane >> 4);  // -1 (source bits 3): no row
        const unsigned long long sp = reinterpret_cast<unsigned long long>(src);
        const uint32_t base = wring + st * AT_STAGE_BYTES;
        const int piece = lane & 15;
#pragma unroll
        for (int q = 0; q < 16; ++q) {
            const int R = 2 * q + (lane >> 4);  // tile row (K: 0-15, V: 16-31) = the lane holding its source
            const unsigned long long rp = __shfl_sync(0xffffffffu, sp, R);
            const unsigned char* gp = rp ? reinterpret_cast<const unsigned char*>(rp) + 16 * piece
                                         : reinterpret_cast<const unsigned char*>(a.q);
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(base + R * AT_PITCH + 16 * piece),
                         "l"(gp), "r"(rp ? 16 : 0)
                         : "memory");
        }
        asm volatile("cp.async.commit_group;\n" ::: "memory");
    };

    // Software pipeline, per warp: tile q0 is computed while q1 is in flight
    // and the row-list entries of tB are loaded (tB is issued next).
    int q0 = ct0 + warp, q1 = q0 + AT_WARPS, tB = q0 + 2 * AT_WARPS;
    int eB = entry(tB);
    issue(entry(q0), 0);
    issue(entry(q1), 1);
    for (int it = 0; q0 < tlimit; ++it) {
        issue(eB, (it + 2) % AT_STAGES);  // tile tB into the stage freed by the tile before q0
        const int tN = tB;
        tB += AT_WARPS;
        eB = entry(tB);
        asm volatile("cp.async.wait_group %0;\n" ::"n"(AT_STAGES - 1) : "memory");
        __syncwarp();  // every lane's pieces of tile q0 have landed
        const int st = it % AT_STAGES;
        const uint32_t kb = wring + st * AT_STAGE_BYTES;
        const uint32_t vb = kb + AT_TILE * AT_PITCH;
        float s0[4] = {0, 0, 0, 0}, s1[4] = {0, 0, 0, 0};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int row = (lane & 7) + ((lane >> 4) << 3);
            const int cc = 2 * j + ((lane >> 3) & 1);
            uint32_t b0, b1, b2, b3;
            ldsm_x4(kb + row * AT_PITCH + (cc << 4), b0, b1, b2, b3);
            mma_bf16(s0, qa[j][0], 0u, qa[j][1], 0u, b0, b1);
            mma_bf16(s1, qa[j][0], 0u, qa[j][1], 0u, b2, b3);
        }
        const int rb = q0 * AT_TILE;
        float x[4];
        x[0] = (rb + 2 * c < rows_total) ? s0[0] * sl2 : -INFINITY;
        x[1] = (rb + 2 * c + 1 < rows_total) ? s0[1] * sl2 : -INFINITY;
        x[2] = (rb + 8 + 2 * c < rows_total) ? s1[0] * sl2 : -INFINITY;
        x[3] = (rb + 9 + 2 * c < rows_total) ? s1[1] * sl2 : -INFINITY;
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
            ldsm_x4_t(vb + row * AT_PITCH + (cc << 4), b0, b1, b2, b3);
            mma_bf16(o[u], pa0, 0u, pa2, 0u, b0, b1);
            mma_bf16(o[u + 1], pa0, 0u, pa2, 0u, b2, b3);
        }
        __syncwarp();  // the stage is refilled two tiles on
        q0 = q1;
        q1 = tN;
    }
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
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
    // the last CTA of this group merges the split partials (the counter
    // self-resets): the block barrier orders every thread's partial stores
    // before thread 0's release, and thread 0's acquire plus the barrier
    // order the merging CTA's loads after all of them
    __shared__ int s_last;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned old;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;\n"
                     : "=r"(old)
                     : "l"(a.counters + h)
                     : "memory");
        s_last = old == (unsigned)(a.splits - 1);
    }
    __syncthreads();
    if (!s_last) return;
    // Parallel merge in one round trip: every thread first puts its loads of
    // the partial outputs (a float4 column of the [G][128] output, for its
    // share of the splits) in flight, next to the (m, l) loads of all splits;
    // after one barrier warp g turns head g's (m, l) into M, L and one weight
    // 2^(m_q - M) per split, and after a second the loaded columns are summed
    // with those weights.  The ring is free by now: red[], the (m, l) copy and
    // the weights reuse it.
    const size_t hb = (size_t)h * a.splits * a.G;
    const int cols = a.G * 32;  // float4 columns of the [G][128] output
    const int P = (AT_WARPS * 32) / cols;
    constexpr int MB = 20;  // splits per thread per batch of loads
    float4* red = reinterpret_cast<float4*>(att_smem);                      // [P][G*32]
    float* sL = reinterpret_cast<float*>(att_smem + 256 * sizeof(float4));  // [8]
    float2* sml = reinterpret_cast<float2*>(sL + 8);                        // [splits][G]
    float* wsm = reinterpret_cast<float*>(sml + a.splits * a.G);            // [splits][G]
    const bool active = (int)threadIdx.x < P * cols;
    const int col = threadIdx.x % cols, ph = threadIdx.x / cols;
    const int gg = col >> 5, d4 = col & 31;
    const float4* po = reinterpret_cast<const float4*>(a.part_o);
    float4 v[MB];
#pragma unroll
    for (int k = 0; k < MB; ++k) {
        const int q = ph + k * P;
        v[k] = (active && q < a.splits) ? __ldcg(po + (hb + (size_t)q * a.G + gg) * 32 + d4)
                                        : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    const float2* pml = reinterpret_cast<const float2*>(a.part_ml);
    for (int t2 = threadIdx.x; t2 < a.splits * a.G; t2 += blockDim.x) sml[t2] = __ldcg(pml + hb + t2);
    __syncthreads();
    if (warp < a.G) {
        float M = -INFINITY;
        for (int q = lane; q < a.splits; q += 32) M = fmaxf(M, sml[q * a.G + warp].x);
#pragma unroll
        for (int o2 = 16; o2 > 0; o2 >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o2));
        float L = 0.0f;
        for (int q = lane; q < a.splits; q += 32) {
            const float2 ml = sml[q * a.G + warp];
            const float f = M == -INFINITY ? 0.0f : exp2f(ml.x - M);
            wsm[q * a.G + warp] = f;
            L += ml.y * f;
        }
#pragma unroll
        for (int o2 = 16; o2 > 0; o2 >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o2);
        if (lane == 0) {
            sL[warp] = L;
            if (a.ml_part) {  // sequence sharding: the group's (max, sum) for the cross-shard combine
                a.ml_part[((size_t)h * a.G + warp) * 2 + 0] = M;
                a.ml_part[((size_t)h * a.G + warp) * 2 + 1] = L;
            }
        }
    }
    __syncthreads();
    if (active) {
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        auto add = [&](int q, const float4& x) {
            const float f = wsm[q * a.G + gg];
            acc.x += x.x * f;
            acc.y += x.y * f;
            acc.z += x.z * f;
            acc.w += x.w * f;
        };
#pragma unroll
        for (int k = 0; k < MB; ++k)
            if (ph + k * P < a.splits) add(ph + k * P, v[k]);
        for (int q0 = ph + MB * P; q0 < a.splits; q0 += MB * P) {  // more splits than one batch
#pragma unroll
            for (int k = 0; k < MB; ++k) {
                const int q = q0 + k * P;
                v[k] = q < a.splits ? __ldcg(po + (hb + (size_t)q * a.G + gg) * 32 + d4)
                                    : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
#pragma unroll
            for (int k = 0; k < MB; ++k)
                if (q0 + k * P < a.splits) add(q0 + k * P, v[k]);
        }
        red[ph * cols + col] = acc;
    }
    __syncthreads();
    if ((int)threadIdx.x < cols) {
        float4 acc = red[col];
        for (int p2 = 1; p2 < P; ++p2) {
            const float4 w = red[p2 * cols + col];
            acc.x += w.x;
            acc.y += w.y;
            acc.z += w.z;
            acc.w += w.w;
        }
        if (a.o_part)  // sequence sharding: unnormalised, combined across shards later
            *reinterpret_cast<float4*>(a.o_part + ((size_t)h * a.G + gg) * 128 + 4 * d4) = acc;
        if (a.out) {
            const float L = sL[gg];
            const float inv = L > 0.0f ? 1.0f / L : 0.0f;
            uint2 packed;
            packed.x = pack_bf16(acc.x * inv, acc.y * inv);
            packed.y = pack_bf16(acc.z * inv, acc.w * inv);
            *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(a.out) + ((size_t)h * a.G + gg) * 128 +
                                      4 * d4) = packed;
        }
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
