// attn_core.cuh -- the gather-attention building blocks of the split-K
// attention kernel (attention.cu), as device functions any kernel can compose:
// the per-warp streaming loop over 16-row tiles (16-byte cp.async pieces into
// a 3-deep ring, mma.sync m16n8k16, online softmax in exp2 space), the CTA's
// warp merge into one (m, l, o) partial, and the split merge by the last CTA
// of a group.  The semantics are those of weighted_flash_decoding as the
// reference calls it (retrieval.py:439-447); see attention.cu.
#pragma once
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


// The group's query heads as mma A fragments (rows g < G live, the rest zero).
IMI_DEV void attn_load_q(const AttnArgs& a, int h, int lane, uint32_t (&qa)[8][2]) {
    const int g = lane >> 2, c = lane & 3;
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

// One warp's share of a CTA's tiles [ct0, ct1): tiles ct0 + warp, + AT_WARPS,
// ...  entry(t) gives this lane's row-list entry for row (lane & 15) of tile
// t (-1: no row).  Rows arrive as 16-byte cp.async pieces, half a warp per
// 256-byte row, two rows per warp instruction; rows past the range or without
// a source buffer are zero-filled (a past-the-range row is also masked out of
// the softmax; a sourceless one counts as a zero row).  Software pipeline:
// tile q0 is computed while q1 is in flight and the entries of tB are read
// (tB is issued next).  The running (m, l, o) stay in the caller's registers.
template <class EntryFn>
IMI_DEV void attn_stream(const AttnArgs& a, int h, int warp, int lane, uint32_t ring, int ct0, int ct1,
                         int rows_total, const uint32_t (&qa)[8][2], EntryFn&& entry, float& m_run, float& l_run,
                         float (&o)[16][4]) {
    const int c = lane & 3;
    const float sl2 = a.scale * 1.4426950408889634f;
    const uint32_t wring = ring + warp * AT_STAGES * AT_STAGE_BYTES;
    const int tlimit = ct1;
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
}

// Merge the AT_WARPS streaming warps through shared memory (smem: the ring,
// free once every warp is done) into this CTA's partial [G][128] + (m, l) at
// split `split` of group h.  Every thread of the block calls it; threads of
// warps >= AT_WARPS carry no state.
IMI_DEV void attn_write_partial(const AttnArgs& a, int h, int split, unsigned char* smem, float m_run, float l_run,
                                const float (&o)[16][4]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, c = lane & 3;
    __syncthreads();
    float* sm_m = reinterpret_cast<float*>(smem);  // [warps][8]
    float* sm_l = sm_m + AT_WARPS * 8;             // [warps][8]
    float* sm_o = sm_l + AT_WARPS * 8;             // [warps][8][128]
    if (warp < AT_WARPS) {
        if (c == 0) {
            sm_m[warp * 8 + g] = m_run;
            sm_l[warp * 8 + g] = l_run;
        }
#pragma unroll
        for (int u = 0; u < 16; ++u) {
            sm_o[(warp * 8 + g) * 128 + 8 * u + 2 * c] = o[u][0];
            sm_o[(warp * 8 + g) * 128 + 8 * u + 2 * c + 1] = o[u][1];
        }
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
}

// Take this group's ticket (a.counters[h], self-resetting); the last CTA to
// arrive merges every split's partial into the output and returns true.  The
// block barrier orders every thread's partial stores before thread 0's
// release, and thread 0's acquire plus the barrier order the merging CTA's
// loads after all of them.
IMI_DEV bool attn_ticket_merge(const AttnArgs& a, int h, unsigned char* smem) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
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
    if (!s_last) return false;
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
    float4* red = reinterpret_cast<float4*>(smem);                      // [P][G*32]
    float* sL = reinterpret_cast<float*>(smem + 256 * sizeof(float4));  // [8]
    float2* sml = reinterpret_cast<float2*>(sL + 8);                    // [splits][G]
    float* wsm = reinterpret_cast<float*>(sml + a.splits * a.G);        // [splits][G]
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
    return true;
}

}  // namespace imi
