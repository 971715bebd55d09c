// build.cu -- on-device IMI index build (sm_100a).
//
// Reproduces, bit for bit, the reference's CPU index build with one worker
// thread:
//   k-means++ seeding         kmeans_core.cpp:138-186
//   Lloyd iterations          kmeans_core.cpp:190-314
//   per-subspace executors    kmeans_core.cpp:384-772
//   compact + CSR reorganize  reorganize_core.cpp:18-311
//
// Exactness strategy:
//   * distances use the reference's 8-lane fma order (common.cuh);
//   * the k-means++ cumulative weight, a sequential double sum in the
//     reference, is computed as an exact 128-bit fixed-point sum; the kernel
//     proves that the reference's double cumsum never rounds (every prefix is
//     representable) and otherwise falls back to the sequential double loop;
//   * M-step sums run in sample order per cell over a stable counting-sort
//     member list; the early-stop inertia is a sequential fp32 sum, evaluated
//     only at iterations where the stop test can fire;
//   * random draws (mt19937_64 seeds 42.., mt19937(iter + 12345)) are taken on
//     the host with the same standard library and uploaded.
#include "common.cuh"
#include "imi_internal.h"

#include <cuda.h>
#include <float.h>
#include <limits.h>

#include <algorithm>
#include <random>
#include <vector>

namespace imi {

constexpr int BT = 256;     // threads per block for the streaming kernels
constexpr int SPB = 1024;   // samples per block (4 per thread)

struct Dev {
    int heads, n, dim, S, sub, T, kmax, NB;
    int kst;               // stride of the per-cell work arrays (max k)
    int ks[4];
    const uint16_t* keys;
    long long hstride, tstride;
    float* cent;           // [T][kmax][sub]
    int32_t* labels;       // [T][n]
    float* md;             // [T][n]
    int32_t* perm_a;       // [T][n]
    int32_t* perm_b;       // [T][n]
    unsigned long long* part_lo;  // [T][NB]
    unsigned long long* part_hi;
    int32_t* part_minl;    // [T][NB]
    int32_t* part_bad;     // [T][NB]
    int32_t* hist;         // [T][NB][256]
    int32_t* dig_off;      // [T][256]
    int32_t* dig_tot;      // [T][256]
    int32_t* counts;       // [T][kmax]
    int32_t* offs;         // [T][kmax+1]
    int32_t* erank;        // [T][kmax]
    int32_t* order;        // [T][kmax] cells by member count, largest first (the M-step's launch order)
    const double* draws_u; // [S][kmax]
    const int32_t* first;  // [S]
    const int32_t* reseed; // [iters][kmax]
    int32_t* done;         // [T]
    float* prev_inertia;   // [T]
    int32_t* iters_run;    // [T]
    uint8_t* used;         // [heads][G]
    int32_t* g2c;          // [heads][G]
    int G;
    // tensor-core E-step: centroids split into bf16 hi + lo halves in the
    // K-major core-matrix layout, their squared norms, and the padded count
    uint16_t* chi;         // [T][npad][sub]
    uint16_t* clo;         // [T][npad][sub]
    float* cn;             // [T][npad]
    float* xn;             // [T][nx] squared norms of the samples (the error band's scale)
    int nx;                // n rounded up to a whole tile of 128
    int npad;              // centroids rounded up to 16 (0 when the tensor-core E-step is not used)
    int32_t* status;       // [1] or null
    uint32_t* kpp_ticket;  // [T] k-means++ step tickets (zero between steps)
};

IMI_DEV int task_h(const Dev& b, int t) { return t / b.S; }
IMI_DEV int task_s(const Dev& b, int t) { return t % b.S; }

IMI_DEV const uint16_t* sample_ptr(const Dev& b, int t, int i) {
    return b.keys + (size_t)task_h(b, t) * b.hstride + (size_t)i * b.tstride + (size_t)task_s(b, t) * b.sub;
}

template <int SUB>
IMI_DEV void load_sample(const Dev& b, int t, int i, float (&x)[SUB]) {
    const uint4* p = reinterpret_cast<const uint4*>(sample_ptr(b, t, i));
#pragma unroll
    for (int q = 0; q < SUB / 8; ++q) {
        const uint4 v = __ldg(p + q);
        x[8 * q + 0] = bf16lo(v.x);
        x[8 * q + 1] = bf16hi(v.x);
        x[8 * q + 2] = bf16lo(v.y);
        x[8 * q + 3] = bf16hi(v.y);
        x[8 * q + 4] = bf16lo(v.z);
        x[8 * q + 5] = bf16hi(v.z);
        x[8 * q + 6] = bf16lo(v.w);
        x[8 * q + 7] = bf16hi(v.w);
    }
}

// float (>= 0) -> Q64.64 fixed point.  bad = not exactly representable within
// the bounds that keep a sum of up to 2^24 values below 2^128.
IMI_DEV u128 to_units(float v, int& lsb, int& bad) {
    u128 r{0ull, 0ull};
    lsb = INT_MAX;
    if (v == 0.0f) return r;
    const uint32_t bits = __float_as_uint(v);
    const int E = (bits >> 23) & 0xff;
    if (E == 0 || E == 255 || (bits >> 31)) {
        bad = 1;
        return r;
    }
    const uint32_t mant = (bits & 0x7fffffu) | 0x800000u;
    const int e2 = E - 127 - 23;
    lsb = e2 + __ffs(mant) - 1;
    const int sh = e2 + 64;
    if (sh > 80) {
        bad = 1;
        return r;
    }
    if (sh >= 64) {
        r.hi = (unsigned long long)mant << (sh - 64);
    } else if (sh >= 0) {
        r.lo = (unsigned long long)mant << sh;
        r.hi = sh > 40 ? ((unsigned long long)mant >> (64 - sh)) : 0ull;
    } else {
        const int rs = -sh;
        if (rs >= 32 || (mant & ((1u << rs) - 1u))) {
            bad = 1;
            return r;
        }
        r.lo = mant >> rs;
    }
    return r;
}

IMI_DEV int u128_bitlen(u128 v) { return v.hi ? 128 - __clzll(v.hi) : (v.lo ? 64 - __clzll(v.lo) : 0); }

IMI_DEV double u128_to_double_units(u128 v) {
    // exact when v has <= 53 significant bits (checked by the caller)
    return ((double)v.hi * 18446744073709551616.0 + (double)v.lo) * 5.421010862427522170037264e-20;  // * 2^-64
}

// ceil(target * 2^64) as u128 (target >= 0, finite)
IMI_DEV u128 ceil_units(double target) {
    u128 r{0ull, 0ull};
    if (!(target > 0.0)) return r;
    const unsigned long long bits = __double_as_longlong(target);
    const int E = (int)((bits >> 52) & 0x7ff);
    unsigned long long m = bits & 0xfffffffffffffull;
    int e2;
    if (E == 0) {
        e2 = -1074;
    } else {
        m |= 1ull << 52;
        e2 = E - 1075;
    }
    const int sh = e2 + 64;
    if (sh >= 0) {
        if (sh >= 64) {
            r.hi = m << (sh - 64);
        } else {
            r.lo = m << sh;
            r.hi = sh ? (m >> (64 - sh)) : 0ull;
        }
    } else {
        const int rs = -sh;
        if (rs >= 64) {
            r.lo = 1ull;  // 0 < target*2^64 < 1
        } else {
            r.lo = m >> rs;
            if (m & ((1ull << rs) - 1ull)) r.lo += 1ull;
        }
    }
    return r;
}

// ---------------------------------------------------------------------------
// k-means++
// ---------------------------------------------------------------------------
__global__ void kpp_first_kernel(Dev b) {
    const int t = blockIdx.x;
    const int s = task_s(b, t);
    const int i = b.first[s];
    const uint16_t* x = sample_ptr(b, t, i);
    for (int d = threadIdx.x; d < b.sub; d += blockDim.x)
        b.cent[(size_t)t * b.kmax * b.sub + d] = bf16_bits_to_f32(x[d]);
}

// Block-wide inclusive scan of one u128 per thread (NT threads); ws: [32] lo
// and [32] hi scratch.  Returns the inclusive prefix; *total = the block sum.
template <int NT>
IMI_DEV u128 kpp_scan_u128(u128 v, unsigned long long* wlo, unsigned long long* whi, u128* total) {
    constexpr int NW = NT / 32;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    u128 x = v;
    for (int o = 1; o < 32; o <<= 1) {
        u128 y = u128_shfl_up(x, o);
        if (lane >= o) x = u128_add(x, y);
    }
    if (lane == 31) {
        wlo[w] = x.lo;
        whi[w] = x.hi;
    }
    __syncthreads();
    if (w == 0) {
        u128 y = lane < NW ? u128{wlo[lane], whi[lane]} : u128{0ull, 0ull};
        for (int o = 1; o < 32; o <<= 1) {
            u128 z = u128_shfl_up(y, o);
            if (lane >= o) y = u128_add(y, z);
        }
        if (lane < NW) {
            wlo[lane] = y.lo;
            whi[lane] = y.hi;
        }
    }
    __syncthreads();
    if (w > 0) x = u128_add(x, u128{wlo[w - 1], whi[w - 1]});
    *total = u128{wlo[NW - 1], whi[NW - 1]};
    __syncthreads();
    return x;
}

// The k-means++ draw of centroid c of task t (kmeans_core.cpp:160-182): the
// exact Q64.64 total of the min-distances (the blocks' partials), the target
// u * total, the first sample whose inclusive cumulative weight reaches it;
// that sample becomes centroid c.  When the reference's sequential double
// cumsum could round (an unrepresentable value, or more than 53 significant
// bits) the reference's own loop runs instead.  All NT threads of the block
// call it; smem holds 16 * NB bytes.
template <int NT>
IMI_DEV void kpp_pick_block(const Dev& b, int t, int c, unsigned char* smem) {
    constexpr int NW = NT / 32;
    constexpr int PER = SPB / NT;  // samples per thread in the crossing block
    const int s = task_s(b, t);
    unsigned long long* plo = reinterpret_cast<unsigned long long*>(smem);  // inclusive prefix per block
    unsigned long long* phi = plo + b.NB;
    __shared__ int s_minl, s_bad, s_sel, s_blk;
    __shared__ unsigned long long wlo[32], whi[32];
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    u128 carry{0ull, 0ull};
    int ml = INT_MAX, bb = 0;
    for (int q0 = 0; q0 < b.NB; q0 += NT) {  // inclusive prefix of the block partials
        const int q = q0 + tid;
        u128 v{0ull, 0ull};
        if (q < b.NB) {
            const size_t o = (size_t)t * b.NB + q;
            v = u128{__ldcg(b.part_lo + o), __ldcg(b.part_hi + o)};
            ml = min(ml, __ldcg(b.part_minl + o));
            bb |= __ldcg(b.part_bad + o);
        }
        u128 tot;
        u128 x = u128_add(kpp_scan_u128<NT>(v, wlo, whi, &tot), carry);
        if (q < b.NB) {
            plo[q] = x.lo;
            phi[q] = x.hi;
        }
        carry = u128_add(carry, tot);
    }
    for (int o = 16; o > 0; o >>= 1) {
        ml = min(ml, __shfl_xor_sync(0xffffffffu, ml, o));
        bb |= __shfl_xor_sync(0xffffffffu, bb, o);
    }
    if (lane == 0) {
        wlo[w] = (unsigned long long)(unsigned)ml;
        whi[w] = (unsigned long long)bb;
    }
    __syncthreads();
    if (tid == 0) {
        int m2 = INT_MAX, b2 = 0;
        for (int q = 0; q < NW; ++q) {
            m2 = min(m2, (int)(unsigned)wlo[q]);
            b2 |= (int)whi[q];
        }
        s_minl = m2;
        s_bad = b2;
        s_sel = -1;
        s_blk = b.NB - 1;
    }
    __syncthreads();
    const u128 total = carry;
    const float* md = b.md + (size_t)t * b.n;
    const double u = b.draws_u[s * b.kst + c];
    bool exact = !s_bad;
    if (exact && (total.lo | total.hi)) exact = (u128_bitlen(total) - (s_minl + 64)) <= 53;
    if (!exact) {
        if (tid == 0) {  // the reference's own sequential double loop (kmeans_core.cpp:164-182)
            double tot = 0.0;
            for (int i = 0; i < b.n; ++i) tot += (double)__ldcg(md + i);
            const double target = u * tot + 0.0;
            double run = 0.0;
            int sel = 0;
            for (int i = 0; i < b.n; ++i) {
                run += (double)__ldcg(md + i);
                if (run >= target) {
                    sel = i;
                    break;
                }
            }
            s_sel = sel;
        }
    } else {
        const double totd = u128_to_double_units(total);
        const double target = u * totd + 0.0;
        const u128 tgt = ceil_units(target);
        for (int q = tid; q < b.NB; q += NT)
            if (u128_ge(u128{plo[q], phi[q]}, tgt)) atomicMin(&s_blk, q);  // the first block reaching the target
        __syncthreads();
        const int blk = s_blk;
        const u128 base = blk > 0 ? u128{plo[blk - 1], phi[blk - 1]} : u128{0ull, 0ull};
        // the crossing block's samples in order: PER consecutive ones per thread
        const int i0 = blk * SPB + tid * PER;
        u128 loc[PER];
        u128 sum{0ull, 0ull};
#pragma unroll
        for (int r = 0; r < PER; ++r) {
            int l, bad = 0;
            const int i = i0 + r;
            const u128 v = i < b.n ? to_units(__ldcg(md + i), l, bad) : u128{0ull, 0ull};
            sum = u128_add(sum, v);
            loc[r] = sum;
        }
        u128 btot;
        const u128 incl = kpp_scan_u128<NT>(sum, wlo, whi, &btot);
        // exclusive prefix of this thread = incl - sum (two's-complement 128-bit)
        u128 ex;
        ex.lo = incl.lo - sum.lo;
        ex.hi = incl.hi - sum.hi - (incl.lo < sum.lo ? 1ull : 0ull);
        ex = u128_add(ex, base);
#pragma unroll
        for (int r = 0; r < PER; ++r) {
            const int i = i0 + r;
            if (i < b.n && u128_ge(u128_add(ex, loc[r]), tgt)) {
                atomicMin(reinterpret_cast<unsigned int*>(&s_sel), (unsigned int)i);  // -1 -> 0xffffffff
                break;
            }
        }
    }
    __syncthreads();
    int sel = s_sel;
    if (sel < 0 || sel >= b.n) sel = 0;
    const uint16_t* xs = sample_ptr(b, t, sel);
    for (int d = tid; d < b.sub; d += NT) b.cent[((size_t)t * b.kmax + c) * b.sub + d] = bf16_bits_to_f32(xs[d]);
}

// Distances of every sample to the newest centroid; min with the running
// min-distance; the block's exact Q64.64 sum.  The sample rows are staged in
// shared memory 256 at a time by coalesced 16-byte cp.async (8-16 threads per
// row), double-buffered, so the pass streams at DRAM speed; each thread then
// reads its own row (a 16-byte pad per row keeps those reads conflict-free).
// One k-means++ step of tasks [t0, t0 + gridDim.y) in one launch: every block updates
// its samples' min-distances and writes its exact partial sum; the last block
// of each task (an atomic ticket) then draws the task's next centroid.
template <int SUB>
__global__ void __launch_bounds__(BT) kpp_step_kernel(Dev b, int c, int t0) {
    constexpr int CPR = SUB / 8;    // 16-byte chunks per row
    constexpr int PITCH = SUB + 8;  // bf16 per staged row
    const int t = t0 + blockIdx.y;
    // a programmatic dependent of the previous step: nothing is read before
    // the previous step (its min-distances and its centroid) has completed
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (t >= b.T || c >= b.ks[task_s(b, t)]) return;
    extern __shared__ __align__(16) uint16_t kst[];  // [2][BT][PITCH]
    __shared__ __align__(16) float cp[SUB];
    __shared__ unsigned long long rlo[BT / 32], rhi[BT / 32];
    __shared__ int rl[BT / 32], rb[BT / 32];
    const int base = blockIdx.x * SPB;
    auto stage = [&](int j, int buf) {
#pragma unroll
        for (int q = 0; q < CPR; ++q) {
            const int e = threadIdx.x + BT * q;
            const int r = e / CPR, ch = e - r * CPR;
            const int i = base + j * BT + r;
            const uint16_t* src = sample_ptr(b, t, i < b.n ? i : 0) + 8 * ch;
            const uint32_t dst =
                static_cast<uint32_t>(__cvta_generic_to_shared(kst + ((size_t)buf * BT + r) * PITCH + 8 * ch));
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(i < b.n ? 16 : 0)
                         : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    stage(0, 0);
    const float* cprev = b.cent + ((size_t)t * b.kmax + (c - 1)) * SUB;
    for (int d = threadIdx.x; d < SUB; d += BT) cp[d] = cprev[d];
    u128 acc{0ull, 0ull};
    int minl = INT_MAX, bad = 0;
    float* md = b.md + (size_t)t * b.n;
    constexpr int NIT = SPB / BT;
    for (int j = 0; j < NIT; ++j) {
        if (j + 1 < NIT && base + (j + 1) * BT < b.n) {
            stage(j + 1, (j + 1) & 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        const int i = base + j * BT + threadIdx.x;
        if (i < b.n) {
            float x[SUB];
            const uint4* row = reinterpret_cast<const uint4*>(kst + ((size_t)(j & 1) * BT + threadIdx.x) * PITCH);
#pragma unroll
            for (int q = 0; q < CPR; ++q) {
                const uint4 v = row[q];
                x[8 * q + 0] = bf16lo(v.x);
                x[8 * q + 1] = bf16hi(v.x);
                x[8 * q + 2] = bf16lo(v.y);
                x[8 * q + 3] = bf16hi(v.y);
                x[8 * q + 4] = bf16lo(v.z);
                x[8 * q + 5] = bf16hi(v.z);
                x[8 * q + 6] = bf16lo(v.w);
                x[8 * q + 7] = bf16hi(v.w);
            }
            const float d = dist_lanes8<SUB>(x, cp);
            const float prev = (c == 1) ? FLT_MAX : md[i];
            const float m = (d < prev) ? d : prev;
            md[i] = m;
            int l;
            acc = u128_add(acc, to_units(m, l, bad));
            minl = min(minl, l);
        }
        __syncthreads();  // this buffer is refilled two iterations on
        if (base + (j + 1) * BT >= b.n) break;
    }
    // block reduce
    for (int o = 16; o > 0; o >>= 1) {
        u128 other;
        other.lo = __shfl_xor_sync(0xffffffffu, acc.lo, o);
        other.hi = __shfl_xor_sync(0xffffffffu, acc.hi, o);
        acc = u128_add(acc, other);
        minl = min(minl, __shfl_xor_sync(0xffffffffu, minl, o));
        bad |= __shfl_xor_sync(0xffffffffu, bad, o);
    }
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        rlo[w] = acc.lo;
        rhi[w] = acc.hi;
        rl[w] = minl;
        rb[w] = bad;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        u128 s{0ull, 0ull};
        int ml = INT_MAX, bb = 0;
        for (int q = 0; q < BT / 32; ++q) {
            s = u128_add(s, u128{rlo[q], rhi[q]});
            ml = min(ml, rl[q]);
            bb |= rb[q];
        }
        const size_t o = (size_t)t * b.NB + blockIdx.x;
        b.part_lo[o] = s.lo;
        b.part_hi[o] = s.hi;
        b.part_minl[o] = ml;
        b.part_bad[o] = bb;
    }
    // The last block of the task to finish draws centroid c: the block
    // barrier orders every thread's min-distance stores (and thread 0's
    // partial) before thread 0's release; its acquire plus the barrier order
    // the drawing block's loads after all of them.
    __shared__ int s_last;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned old;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;\n" : "=r"(old) : "l"(b.kpp_ticket + t) : "memory");
        s_last = old == (unsigned)(gridDim.x - 1);
    }
    __syncthreads();
    if (!s_last) return;
    kpp_pick_block<BT>(b, t, c, reinterpret_cast<unsigned char*>(kst));
    if (threadIdx.x == 0) b.kpp_ticket[t] = 0;  // re-armed for the next step
}



template <int SUB>
size_t kpp_step_smem(int NB) {
    const size_t stage = (size_t)2 * BT * (SUB + 8) * 2, pick = (size_t)16 * NB;
    return stage > pick ? stage : pick;
}

// ---------------------------------------------------------------------------
// Lloyd E-step: first-min argmin over the task's centroids
// ---------------------------------------------------------------------------
template <int SUB>
__global__ void __launch_bounds__(BT) estep_kernel(Dev b) {
    const int t = blockIdx.y;
    if (b.done[t]) return;
    extern __shared__ __align__(16) float cs[];
    const int k = b.ks[task_s(b, t)];
    const int chunk = min(k, 32768 / SUB);
    const int i = blockIdx.x * BT + threadIdx.x;
    float x[SUB];
    if (i < b.n) load_sample<SUB>(b, t, i, x);
    float best = FLT_MAX;
    int bi = 0;
    const float* cg = b.cent + (size_t)t * b.kmax * SUB;
    for (int c0 = 0; c0 < k; c0 += chunk) {
        const int cn = min(chunk, k - c0);
        __syncthreads();
        for (int e = threadIdx.x; e < cn * SUB / 4; e += BT)
            reinterpret_cast<float4*>(cs)[e] = reinterpret_cast<const float4*>(cg + (size_t)c0 * SUB)[e];
        __syncthreads();
        if (i < b.n) {
            for (int c = 0; c < cn; ++c) {
                const float d = dist_lanes8<SUB>(x, cs + c * SUB);
                if (d < best) {
                    best = d;
                    bi = c0 + c;
                }
            }
        }
    }
    if (i < b.n) {
        b.labels[(size_t)t * b.n + i] = bi;
        b.md[(size_t)t * b.n + i] = best;
    }
}

// Sequential fp32 inertia and the early-stop test (kmeans_core.cpp:216-262).
// The sum is one chain in sample order (thread 0); the other threads stage
// the next 4096 distances in shared memory meanwhile, so the chain never
// waits on memory.
constexpr int IN_THREADS = 256;
constexpr int IN_CHUNK = 4096;
__global__ void __launch_bounds__(IN_THREADS) inertia_kernel(Dev b, int it, int max_iters, int min_iter, float tol,
                                                             float rel_tol, int eval) {
    const int t = blockIdx.x;
    if (b.done[t]) return;
    __shared__ __align__(16) float buf[2][IN_CHUNK];
    float inertia = 0.0f;
    if (eval) {
        const float* md = b.md + (size_t)t * b.n;
        const int nch = (b.n + IN_CHUNK - 1) / IN_CHUNK;
        auto stage = [&](int ch) {
            const int i0 = ch * IN_CHUNK;
            float* dst = buf[ch & 1];
            for (int e = threadIdx.x; e < IN_CHUNK; e += IN_THREADS) {
                const int i = i0 + e;
                asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(
                                 static_cast<uint32_t>(__cvta_generic_to_shared(dst + e))),
                             "l"(md + (i < b.n ? i : 0)), "r"(i < b.n ? 4 : 0)
                             : "memory");
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
        };
        stage(0);
        for (int ch = 0; ch < nch; ++ch) {
            if (ch + 1 < nch) {
                stage(ch + 1);
                asm volatile("cp.async.wait_group 1;" ::: "memory");
            } else {
                asm volatile("cp.async.wait_group 0;" ::: "memory");
            }
            __syncthreads();
            if (threadIdx.x == 0) {
                const float* v = buf[ch & 1];
                const int cnt = min(IN_CHUNK, b.n - ch * IN_CHUNK);
                int e = 0;
                for (; e + 8 <= cnt; e += 8) {
                    const float4 a = *reinterpret_cast<const float4*>(v + e);
                    const float4 c = *reinterpret_cast<const float4*>(v + e + 4);
                    inertia = __fadd_rn(inertia, a.x);
                    inertia = __fadd_rn(inertia, a.y);
                    inertia = __fadd_rn(inertia, a.z);
                    inertia = __fadd_rn(inertia, a.w);
                    inertia = __fadd_rn(inertia, c.x);
                    inertia = __fadd_rn(inertia, c.y);
                    inertia = __fadd_rn(inertia, c.z);
                    inertia = __fadd_rn(inertia, c.w);
                }
                for (; e < cnt; ++e) inertia = __fadd_rn(inertia, v[e]);
            }
            __syncthreads();  // this buffer is refilled two chunks on
        }
    }
    if (threadIdx.x != 0) return;
    const int iters = it + 1;
    if (eval) {
        const float prev = b.prev_inertia[t];
        const float change = fabsf(__fsub_rn(prev, inertia));
        const float rel = (prev > 0.0f) ? __fdiv_rn(change, prev) : 0.0f;
        if (iters >= max(1, min_iter) && (rel <= fmaxf(0.0f, rel_tol) || change <= fmaxf(0.0f, tol))) {
            b.done[t] = 1;
            b.iters_run[t] = iters;
            return;
        }
        b.prev_inertia[t] = inertia;
    }
    b.iters_run[t] = iters;
}

// ---------------------------------------------------------------------------
// Tensor-core E-step (tcgen05 MMA into TMEM) with an exact recheck.
//
// The reference's labels come from exact fp32 distances in its 8-lane order.
// Here a 128-sample tile meets every centroid on the tensor cores and TMEM
// receives an approximate d~(x, c) = ||c||^2 - 2 x.c: the samples are bf16
// (exact), extended by a [1, 1] column pair; the centroids go in as -2c split
// into bf16 hi + lo halves, extended by ||c||^2 split the same way; fp32
// accumulation.  The splits leave under 2^-18 relative of each term, the fp32
// accumulation of the exact products under 2^-16 of sum |x_i c_i|, and the
// exact routine's own rounding under 2^-19 of the distance, so every centroid
// with d~ within 2^-11 (||x||^2 + max ||c||^2) of the minimum d~ is
// recomputed with the exact 8-lane routine and the exact minimum wins (the
// lowest index on ties): labels and minimum distances are those of the exact
// E-step.  Usually only one centroid lies in that band: it is the winner, and
// its exact distance is only needed when the inertia is evaluated.
//
// Operands sit in shared memory in the K-major, no-swizzle core-matrix
// layout (8 rows x 16 bytes per core matrix).  Centroid rows: core matrices
// 128 B apart along K, 8-row groups KC*16 B apart (KC = SUB + 16 columns).
// Sample tiles: chunk-major as the TMA writes them (below).
// ---------------------------------------------------------------------------
constexpr int TC_M = 128;                 // samples per tile = TMEM lanes
constexpr int TC_WAIT_LIMIT = 1 << 20;    // polls of the MMA-done barrier before giving up
constexpr float TC_PAD_NORM = 3.0e38f;    // ||c||^2 of a padding row: never the minimum, still finite

template <int KC>
IMI_DEV int core_off(int r, int d) {
    return (r >> 3) * (KC * 8) + (d >> 3) * 64 + (r & 7) * 8 + (d & 7);
}

IMI_DEV uint32_t tc_smem(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// shared-memory matrix descriptor: start address, leading / stride byte
// offsets (16-byte units), descriptor version 1 (sm_100), no swizzle
IMI_DEV uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

IMI_DEV void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

IMI_DEV bool tc_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

IMI_DEV bool tc_wait(uint32_t bar, uint32_t parity) {
    for (int i = 0; i < TC_WAIT_LIMIT; ++i)
        if (tc_try_wait(bar, parity)) return true;
    return false;
}

IMI_DEV void tc_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}

IMI_DEV void tc_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

// minimum of W accumulator words (a tree, so the compares overlap)
template <int W>
IMI_DEV float tc_min(const uint32_t (&r)[W]) {
    float v[W];
#pragma unroll
    for (int j = 0; j < W; ++j) v[j] = __uint_as_float(r[j]);
#pragma unroll
    for (int h = W / 2; h > 0; h >>= 1)
#pragma unroll
        for (int j = 0; j < h; ++j) v[j] = fminf(v[j], v[j + h]);
    return v[0];
}

// bit j set where word j is at most thr
template <int W>
IMI_DEV uint32_t tc_le(const uint32_t (&r)[W], float thr) {
    uint32_t m = 0u;
#pragma unroll
    for (int j = 0; j < W; ++j) m |= (__uint_as_float(r[j]) <= thr) ? (1u << j) : 0u;
    return m;
}

// the low `live` bits (all 32 when live >= 32, none when live <= 0): the
// columns below k; padding columns never win, even when the band is infinite
IMI_DEV uint32_t col_mask(int live) { return live >= 32 ? 0xffffffffu : (live <= 0 ? 0u : (1u << live) - 1u); }

// squared norm of every sample of every task (fp32; it only scales the error
// band of the tensor-core E-step), rows padded to whole tiles
template <int SUB>
__global__ void __launch_bounds__(BT) xnorm_kernel(Dev b) {
    const int t = blockIdx.y;
    const int i = blockIdx.x * BT + threadIdx.x;
    if (i >= b.nx) return;
    float s = 0.0f;
    if (i < b.n) {
        float x[SUB];
        load_sample<SUB>(b, t, i, x);
#pragma unroll
        for (int d = 0; d < SUB; ++d) s = fmaf(x[d], x[d], s);
    }
    b.xn[(size_t)t * b.nx + i] = s;
}

IMI_DEV uint16_t bf16_bits_rn(float v) { return __bfloat16_as_ushort(__float2bfloat16_rn(v)); }

// centroid c of task t -> B rows of the two MMA chains (core-matrix layout,
// KC = SUB + 16 columns): hi row = [bf16(-2c), hi(||c||^2), lo(||c||^2), 0..],
// lo row = [bf16(-2c - hi), 0..]; padding rows carry only a huge norm
template <int SUB>
__global__ void cent_split_kernel(Dev b) {
    constexpr int KC = SUB + 16;
    const int t = blockIdx.y, c = blockIdx.x;
    if (b.done[t]) return;
    const int k = b.ks[task_s(b, t)];
    const float* src = b.cent + ((size_t)t * b.kmax + c) * SUB;
    uint16_t* hi = b.chi + (size_t)t * b.npad * KC;
    uint16_t* lo = b.clo + (size_t)t * b.npad * KC;
    float sq = 0.0f;
    for (int d = threadIdx.x; d < SUB; d += 32) {
        const float v = c < k ? src[d] : 0.0f;
        const float m2 = -2.0f * v;  // exact (power of two)
        const uint16_t h = bf16_bits_rn(m2);
        hi[core_off<KC>(c, d)] = h;
        lo[core_off<KC>(c, d)] = bf16_bits_rn(m2 - bf16_bits_to_f32(h));
        sq = fmaf(v, v, sq);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    if (threadIdx.x < 16) {
        const float nrm = c < k ? sq : TC_PAD_NORM;
        const uint16_t nh = bf16_bits_rn(nrm);
        const uint16_t nl = bf16_bits_rn(nrm - bf16_bits_to_f32(nh));
        const int d = SUB + threadIdx.x;
        hi[core_off<KC>(c, d)] = threadIdx.x == 0 ? nh : (threadIdx.x == 1 ? nl : (uint16_t)0);
        lo[core_off<KC>(c, d)] = 0;
        if (threadIdx.x == 0) b.cn[(size_t)t * b.npad + c] = c < k ? sq : 0.0f;
    }
}

// Lloyd E-step on the tensor cores, warp-specialised.  One CTA per SM walks
// a run of 128-sample tiles of one task:
//  * a producer thread keeps up to `stages` tiles in flight with TMA (a 4-D
//    tensor map over the keys writes each tile chunk-major: 16-byte column
//    chunk c of row r at c * 2 KB + r * 16 B, the no-swizzle K-major
//    core-matrix layout with LBO = 2 KB, SBO = 128 B) plus the tile's 128
//    sample norms;
//  * an MMA thread (another warp) issues the hi, norm and lo MMA chains of
//    tile j into TMEM accumulator j % 4 (npad fp32 columns,
//    d~(c) = ||c||^2 - 2 x.c) once the tile has landed and the accumulator
//    is free (each role waits on its own barriers);
//  * two groups of eight epilogue warps take alternate tiles; sample r (TMEM
//    lane r) of a tile is shared by two warps of the group, each scanning one
//    half of the columns: the minimum m1, then the centroids with
//    d~ <= m1 + band, band = 2^-11 (||x||^2 + max ||c||^2) bounding the
//    bf16-split error.  One centroid in that set is the exact first-min
//    argmin; otherwise every centroid of the set is re-measured exactly and
//    the lowest distance (then the lowest index) wins.  The exact distance of
//    the winner is only computed for iterations whose inertia is evaluated.
// Stages and accumulators are handed over with mbarriers (full / empty per
// stage, full / empty per accumulator); every wait is bounded and a timeout
// sets the status flag and drains the copies and MMAs in flight.
constexpr int TC_MAX_STAGES = 8;
constexpr int TC_GROUP = 256;                       // eight epilogue warps
constexpr int TC_CTA_THREADS = 2 * TC_GROUP + 64;   // two groups, the MMA warp and the TMA warp (18 warps:
                                                    // at most 96 registers, five warps share one SM quarter)

// element (r, d) of a staged sample tile (chunk-major, see above)
IMI_DEV int a_off(int r, int d) { return (d >> 3) * (TC_M * 8) + r * 8 + (d & 7); }

IMI_DEV void mb_init(uint32_t bar, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
IMI_DEV bool mb_test(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
IMI_DEV void mb_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
IMI_DEV void mb_expect(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
IMI_DEV void group_sync(int id) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(TC_GROUP) : "memory"); }
IMI_DEV bool group_any(int id, bool v) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(id), "r"(TC_GROUP)
        : "memory");
    return r != 0;
}

// Exact squared distance between sample row `row` of a staged tile and an
// fp32 centroid: the same eight-lane accumulation order as dist_lanes8.
template <int SUB>
IMI_DEV float dist_tile(const uint16_t* A, int row, const float* __restrict__ c) {
    float lane[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) lane[l] = 0.0f;
#pragma unroll
    for (int i = 0; i < SUB; i += 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(A + a_off(row, i));
        const float4 c0 = *reinterpret_cast<const float4*>(c + i);
        const float4 c1 = *reinterpret_cast<const float4*>(c + i + 4);
        float d;
        d = __fsub_rn(bf16lo(v.x), c0.x); lane[0] = __fmaf_rn(d, d, lane[0]);
        d = __fsub_rn(bf16hi(v.x), c0.y); lane[1] = __fmaf_rn(d, d, lane[1]);
        d = __fsub_rn(bf16lo(v.y), c0.z); lane[2] = __fmaf_rn(d, d, lane[2]);
        d = __fsub_rn(bf16hi(v.y), c0.w); lane[3] = __fmaf_rn(d, d, lane[3]);
        d = __fsub_rn(bf16lo(v.z), c1.x); lane[4] = __fmaf_rn(d, d, lane[4]);
        d = __fsub_rn(bf16hi(v.z), c1.y); lane[5] = __fmaf_rn(d, d, lane[5]);
        d = __fsub_rn(bf16lo(v.w), c1.z); lane[6] = __fmaf_rn(d, d, lane[6]);
        d = __fsub_rn(bf16hi(v.w), c1.w); lane[7] = __fmaf_rn(d, d, lane[7]);
    }
    float t = __fadd_rn(lane[0], lane[1]);
#pragma unroll
    for (int l = 2; l < 8; ++l) t = __fadd_rn(t, lane[l]);
    return t;
}

template <int SUB>
__global__ void __launch_bounds__(TC_CTA_THREADS, 1)
    estep_tc_kernel(Dev b, const __grid_constant__ CUtensorMap tmap, int tiles_per_cta, int acc_cols, int stages,
                    int want_md) {
    constexpr int KC = SUB + 16;   // K columns of the hi chain of B (the lo chain uses the first SUB)
    constexpr int CPR = SUB / 8;   // 16-byte chunks per sample row
    constexpr int CFLD = SUB + 4;  // row stride of the exact centroids (spreads the banks)
    const int t = blockIdx.y;
    if (b.done[t]) return;  // the whole CTA, before any TMEM is allocated
    const int k = b.ks[task_s(b, t)], npad = b.npad;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ntiles = (b.n + TC_M - 1) / TC_M;
    const int tile0 = blockIdx.x * tiles_per_cta;
    const int nt = max(0, min(ntiles, tile0 + tiles_per_cta) - tile0);

    extern __shared__ __align__(1024) unsigned char tsm[];
    uint16_t* As = reinterpret_cast<uint16_t*>(tsm);  // [stages][CPR][TC_M][8] sample tiles
    uint16_t* Ae = As + stages * TC_M * SUB;           // [TC_M][16] constant norm columns
    uint16_t* Bh = Ae + TC_M * 16;                     // [npad][KC]
    uint16_t* Bl = Bh + npad * KC;
    float* xs = reinterpret_cast<float*>(Bl + npad * KC);  // [stages][TC_M] sample norms
    unsigned long long* bars = reinterpret_cast<unsigned long long*>(xs + stages * TC_M);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 24);
    float* cf = reinterpret_cast<float*>(bars + 64);   // [k][CFLD] exact centroids
    const uint32_t full0 = tc_smem(bars), empty0 = tc_smem(bars + 8);
    const uint32_t accf0 = tc_smem(bars + 16), acce0 = tc_smem(bars + 20);
    __shared__ float xm[2][2][TC_M];  // per group and half: partial minimum, then partial exact best
    __shared__ int xc[2][2][TC_M];    // per group and half: candidates in the band, then best index
    __shared__ int xf[2][2][TC_M];    // per group and half: first candidate
    __shared__ float red[TC_CTA_THREADS / 32];
    __shared__ volatile int s_fail;
    __shared__ int s_issued, s_mma;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc_smem(tslot)),
                     "r"(4 * acc_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    for (int e = tid; e < TC_M * 16; e += TC_CTA_THREADS)  // bf16 1.0 in columns 0 and 1
        Ae[core_off<16>(e >> 4, e & 15)] = (e & 15) < 2 ? (uint16_t)0x3F80u : (uint16_t)0;
    {  // this task's B rows (both chains) and its exact centroids
        const uint4* sh = reinterpret_cast<const uint4*>(b.chi + (size_t)t * npad * KC);
        const uint4* sl = reinterpret_cast<const uint4*>(b.clo + (size_t)t * npad * KC);
        uint4* dh = reinterpret_cast<uint4*>(Bh);
        uint4* dl = reinterpret_cast<uint4*>(Bl);
        for (int e = tid; e < npad * KC / 8; e += TC_CTA_THREADS) {
            dh[e] = sh[e];
            dl[e] = sl[e];
        }
        const float* sc = b.cent + (size_t)t * b.kmax * SUB;
        for (int e = tid; e < k * SUB / 4; e += TC_CTA_THREADS) {
            const int c = e / (SUB / 4), q = e - c * (SUB / 4);
            *reinterpret_cast<float4*>(cf + c * CFLD + 4 * q) = *reinterpret_cast<const float4*>(sc + 4 * e);
        }
        float cm = 0.0f;  // max ||c||^2 of the task's centroids (the band's scale)
        for (int c = tid; c < k; c += TC_CTA_THREADS) cm = fmaxf(cm, __ldg(b.cn + (size_t)t * npad + c));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
        if (lane == 0) red[warp] = cm;
    }
    if (tid == 0) {
        for (int q = 0; q < stages; ++q) {
            mb_init(full0 + 8 * q, 1);   // the control thread's expect_tx; the copies complete it
            mb_init(empty0 + 8 * q, 2);  // the MMAs' commit and the epilogue group
        }
        for (int q = 0; q < 4; ++q) {
            mb_init(accf0 + 8 * q, 1);   // the MMAs' commit
            mb_init(acce0 + 8 * q, 1);   // the epilogue group
        }
        s_fail = 0;
        s_issued = 0;
        s_mma = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes above -> MMA operand reads
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tslot;
    float cmax = red[0];
#pragma unroll
    for (int w = 1; w < TC_CTA_THREADS / 32; ++w) cmax = fmaxf(cmax, red[w]);

    if (warp == 2 * TC_GROUP / 32) {
        // ---- MMA issuer (one thread): tile j once it has landed and its accumulator is free
        if (lane == 0) {
            // instruction descriptor: fp32 accumulator, bf16 A and B, both K-major, N = npad, M = 128
            const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(npad >> 3) << 17) |
                                   ((uint32_t)(TC_M >> 4) << 24);
            const uint32_t bh0 = tc_smem(Bh), bl0 = tc_smem(Bl);
            constexpr uint32_t LBO_A = TC_M * 16, SBO_A = 128, LBO_B = 128, SBO_B = KC * 16;
            const uint64_t ext_desc = umma_desc(tc_smem(Ae), 128, 256);
            const uint64_t a_desc0 = umma_desc(tc_smem(As), LBO_A, SBO_A);
            const uint64_t bh_desc = umma_desc(bh0, LBO_B, SBO_B), bl_desc = umma_desc(bl0, LBO_B, SBO_B);
            int jm = 0;
            for (; jm < nt; ++jm) {
                const int q = jm % stages, ac = jm & 3;
                if (!tc_wait(full0 + 8 * q, (uint32_t)(jm / stages) & 1u) ||
                    (jm >= 4 && !tc_wait(acce0 + 8 * ac, (uint32_t)((jm >> 2) - 1) & 1u))) {
                    s_fail = 1;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t acc = tmem + (uint32_t)(ac * acc_cols);
                // descriptor start addresses sit in the low bits (16-byte units):
                // a K step is a plain add
                const uint64_t ad = a_desc0 + (uint64_t)(q * (TC_M * SUB * 2 / 16));
#pragma unroll
                for (int kk = 0; kk < SUB / 16; ++kk)
                    umma_bf16(acc, ad + (uint64_t)(kk * (2 * LBO_A / 16)), bh_desc + (uint64_t)(kk * (2 * LBO_B / 16)),
                              idesc, kk > 0 ? 1u : 0u);
                umma_bf16(acc, ext_desc, bh_desc + (uint64_t)((SUB / 16) * (2 * LBO_B / 16)), idesc, 1u);
#pragma unroll
                for (int kk = 0; kk < SUB / 16; ++kk)
                    umma_bf16(acc, ad + (uint64_t)(kk * (2 * LBO_A / 16)), bl_desc + (uint64_t)(kk * (2 * LBO_B / 16)),
                              idesc, 1u);
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 accf0 + 8 * ac)
                             : "memory");
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 empty0 + 8 * q)
                             : "memory");
            }
            s_mma = jm;
        }
    } else if (warp == 2 * TC_GROUP / 32 + 1) {
        // ---- TMA producer (one thread): tile j into its stage once that stage is free
        if (lane == 0) {
            const uint32_t stage_bytes = TC_M * SUB * 2;
            const int h = task_h(b, t), s0 = task_s(b, t) * CPR;
            const float* xn_t = b.xn + (size_t)t * b.nx;
            int issued = 0;
            for (; issued < nt; ++issued) {
                const int q = issued % stages;
                if (issued >= stages && !tc_wait(empty0 + 8 * q, (uint32_t)((issued / stages) - 1) & 1u)) {
                    s_fail = 1;
                    break;
                }
                const uint32_t fb = full0 + 8 * q;
                const int row0 = (tile0 + issued) * TC_M;
                mb_expect(fb, stage_bytes + TC_M * 4);
                asm volatile(
                    "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
                    "[%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(tc_smem(As + q * TC_M * SUB)),
                    "l"(reinterpret_cast<uint64_t>(&tmap)), "r"(0), "r"(row0), "r"(s0), "r"(h), "r"(fb)
                    : "memory");
                asm volatile(
                    "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                        tc_smem(xs + q * TC_M)),
                    "l"(xn_t + row0), "r"(TC_M * 4), "r"(fb)
                    : "memory");
            }
            s_issued = issued;
        }
    } else {
        // ---- epilogue (warps 0-15): group g takes tiles g, g + 2, ...
        const int g = warp >> 3, lw = warp & 7, half = lw >> 2;
        const int row = (lw & 3) * 32 + lane;            // this thread's sample (TMEM lane) in a tile
        const int gid = 1 + g;                           // the group's named barrier
        const int hsplit = ((npad / 2 + 15) / 16) * 16;  // columns [0, hsplit) and [hsplit, npad)
        const int cbeg = half ? hsplit : 0, cend = half ? npad : hsplit;
        const uint32_t lane_base = (uint32_t)((lw & 3) * 32) << 16;
        for (int j = g; j < nt; j += 2) {
            const int q = j % stages, ac = j & 3;
            // one thread polls the barriers; the group waits at its named barrier
            bool ok = true;
            if ((tid & (TC_GROUP - 1)) == 0)
                ok = tc_wait(accf0 + 8 * ac, (uint32_t)(j >> 2) & 1u) && tc_wait(full0 + 8 * q, (uint32_t)(j / stages) & 1u);
            if (group_any(gid, !ok)) {
                s_fail = 1;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t taddr = tmem + lane_base + (uint32_t)(ac * acc_cols);
            const uint16_t* Ap = As + q * TC_M * SUB;
            const float xn = xs[q * TC_M + row];
            const int i = (tile0 + j) * TC_M + row;
            // pass 1: the approximate minimum over this half of the row
            float m1 = INFINITY;
            int c0 = cbeg;
            for (; c0 + 32 <= cend; c0 += 32) {
                uint32_t r[32];
                tc_ld32(taddr + (uint32_t)c0, r);
                m1 = fminf(m1, tc_min<32>(r));
            }
            if (c0 < cend) {
                uint32_t r[16];
                tc_ld16(taddr + (uint32_t)c0, r);
                m1 = fminf(m1, tc_min<16>(r));
            }
            xm[g][half][row] = m1;
            group_sync(gid);
            m1 = fminf(xm[g][0][row], xm[g][1][row]);
            // pass 2: the real centroids of this half within the band
            const float thr = m1 + ldexpf(xn + cmax, -11);
            int cnt = 0, first = 0;
            for (c0 = cbeg; c0 + 32 <= cend; c0 += 32) {
                uint32_t r[32];
                tc_ld32(taddr + (uint32_t)c0, r);
                const uint32_t m = tc_le<32>(r, thr) & col_mask(k - c0);
                if (cnt == 0 && m) first = c0 + __ffs(m) - 1;
                cnt += __popc(m);
            }
            if (c0 < cend) {
                uint32_t r[16];
                tc_ld16(taddr + (uint32_t)c0, r);
                const uint32_t m = tc_le<16>(r, thr) & col_mask(k - c0);
                if (cnt == 0 && m) first = c0 + __ffs(m) - 1;
                cnt += __popc(m);
            }
            xc[g][half][row] = cnt;
            xf[g][half][row] = first;
            group_sync(gid);
            const int c_lo = xc[g][0][row];
            const bool single = c_lo + xc[g][1][row] <= 1;
            int bi = c_lo ? xf[g][0][row] : xf[g][1][row];
            float best = 0.0f;
            // several within the band: each half re-measures its own, in index
            // order; the TMEM loads are warp-wide, so a warp walks its chunks
            // when any of its lanes needs them
            if (group_any(gid, !single)) {
                float pb = FLT_MAX;
                int pi = 0;
                if (__any_sync(0xffffffffu, !single)) {
                    const float th2 = single ? -INFINITY : thr;
                    for (c0 = cbeg; c0 < cend; c0 += 16) {
                        uint32_t r[16];
                        tc_ld16(taddr + (uint32_t)c0, r);
                        uint32_t cand = tc_le<16>(r, th2) & col_mask(k - c0);
                        while (cand) {
                            const int c = c0 + __ffs(cand) - 1;
                            cand &= cand - 1u;
                            const float dd = dist_tile<SUB>(Ap, row, cf + c * CFLD);
                            if (dd < pb) {
                                pb = dd;
                                pi = c;
                            }
                        }
                    }
                }
                xm[g][half][row] = pb;  // (the partials of pass 2 were read before the vote)
                xc[g][half][row] = pi;
                group_sync(gid);
                if (!single) {
                    const bool lo_wins = xm[g][0][row] <= xm[g][1][row];  // ties: the lower index
                    best = lo_wins ? xm[g][0][row] : xm[g][1][row];
                    bi = lo_wins ? xc[g][0][row] : xc[g][1][row];
                }
            }
            if (half == 0) {
                if (single && want_md) best = dist_tile<SUB>(Ap, row, cf + bi * CFLD);
                if (i < b.n) {
                    b.labels[(size_t)t * b.n + i] = bi;
                    if (want_md) b.md[(size_t)t * b.n + i] = best;
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            group_sync(gid);  // the accumulator, the tile and the exchange arrays are free again
            if ((tid & (TC_GROUP - 1)) == 0) {
                mb_arrive(acce0 + 8 * ac);
                mb_arrive(empty0 + 8 * q);
            }
        }
    }
    __syncthreads();
    if (s_fail) {
        // a wait gave up: the CTA's labels are not valid.  Leave every row of its
        // tiles with an in-range label (0) so that the kernels that index by
        // label (counts, M-step, reorganize) stay in bounds; the status bit
        // tells the caller the build is void.
        const int r0 = tile0 * TC_M, r1 = min(b.n, (tile0 + nt) * TC_M);
        for (int i = r0 + tid; i < r1; i += TC_CTA_THREADS) {
            b.labels[(size_t)t * b.n + i] = 0;
            if (want_md) b.md[(size_t)t * b.n + i] = 0.0f;
        }
    }
    if (tid == 2 * TC_GROUP && s_fail) {
        // report, then let the copies and MMAs in flight finish (bounded) before TMEM and shared memory go
        if (b.status) atomicOr(b.status, 1);
        const int issued = s_issued, jm = s_mma;
        for (int j = max(0, jm - 4); j < jm; ++j) (void)tc_wait(accf0 + 8 * (j & 3), (uint32_t)(j >> 2) & 1u);
        for (int j = jm; j < issued; ++j) (void)tc_wait(full0 + 8 * (j % stages), (uint32_t)(j / stages) & 1u);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(4 * acc_cols) : "memory");
}

// The keys as a 4-D TMA tensor: (8 bf16 of a chunk, token, chunk of the head
// dim, head), so that a box of (8, 128, sub / 8, 1) lands chunk-major.  False
// when the driver entry point is missing or the strides do not qualify.
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static bool encode_sample_map(const Dev& d, CUtensorMap* m) {
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
        else
            (void)cudaGetLastError();
    }
    if (!fn) return false;
    const unsigned long long tb = (unsigned long long)d.tstride * 2;
    const unsigned long long hb = d.heads > 1 ? (unsigned long long)d.hstride * 2 : tb * (unsigned long long)d.n;
    if ((reinterpret_cast<uintptr_t>(d.keys) & 15) || (tb & 15) || (hb & 15) || d.dim % 8 || d.sub % 16) return false;
    const cuuint64_t dims[4] = {8, (cuuint64_t)d.n, (cuuint64_t)(d.dim / 8), (cuuint64_t)d.heads};
    const cuuint64_t strides[3] = {tb, 16, hb};
    const cuuint32_t box[4] = {8, (cuuint32_t)TC_M, (cuuint32_t)(d.sub / 8), 1};
    const cuuint32_t elem[4] = {1, 1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<uint16_t*>(d.keys), dims, strides, box, elem,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// ---------------------------------------------------------------------------
// Stable counting sort by an 8-bit digit (one LSD radix pass).
//   key(t, i) = (keys[t*key_tstride + i] >> shift) & 255
//   element at position p is perm_in[t][p] (or p when perm_in is null)
// ---------------------------------------------------------------------------
struct Radix {
    int T, n, NB, shift;
    const int32_t* keys;
    long long key_tstride;
    const int32_t* perm_in;   // [T][n] or null
    int32_t* perm_out;        // [T][n]
    int32_t* hist;            // [T][NB][256]
    int32_t* dig_off;         // [T][256]
    int32_t* dig_tot;         // [T][256]
    const int32_t* gate;      // [T] skip tasks with gate[t] != 0 (may be null)
};

__global__ void __launch_bounds__(BT) radix_hist_kernel(Radix r) {
    const int t = blockIdx.y;
    if (r.gate && r.gate[t]) return;
    __shared__ int h[256];
    h[threadIdx.x] = 0;
    __syncthreads();
    for (int j = 0; j < SPB / BT; ++j) {
        const int p = blockIdx.x * SPB + j * BT + threadIdx.x;
        if (p >= r.n) break;
        const int i = r.perm_in ? r.perm_in[(size_t)t * r.n + p] : p;
        const int v = (r.keys[(size_t)t * r.key_tstride + i] >> r.shift) & 255;
        atomicAdd(&h[v], 1);
    }
    __syncthreads();
    r.hist[((size_t)t * r.NB + blockIdx.x) * 256 + threadIdx.x] = h[threadIdx.x];
}

__global__ void __launch_bounds__(256) radix_scan_kernel(Radix r) {
    const int t = blockIdx.x;
    if (r.gate && r.gate[t]) return;
    const int v = threadIdx.x;
    int run = 0;
    for (int q = 0; q < r.NB; ++q) {
        const size_t o = ((size_t)t * r.NB + q) * 256 + v;
        const int x = r.hist[o];
        r.hist[o] = run;
        run += x;
    }
    __shared__ int tot[256];
    tot[v] = run;
    __syncthreads();
    if (v == 0) {
        int acc = 0;
        for (int q = 0; q < 256; ++q) {
            r.dig_off[(size_t)t * 256 + q] = acc;
            r.dig_tot[(size_t)t * 256 + q] = tot[q];
            acc += tot[q];
        }
    }
}

__global__ void __launch_bounds__(BT) radix_scatter_kernel(Radix r) {
    const int t = blockIdx.y;
    if (r.gate && r.gate[t]) return;
    __shared__ int run[256];
    __shared__ int wc[BT / 32][257];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    run[threadIdx.x] = 0;
    for (int q = 0; q < BT / 32; ++q) wc[q][threadIdx.x] = 0;
    if (threadIdx.x < BT / 32) wc[threadIdx.x][256] = 0;
    __syncthreads();
    const int32_t* hb = r.hist + ((size_t)t * r.NB + blockIdx.x) * 256;
    const int32_t* doff = r.dig_off + (size_t)t * 256;
    for (int j = 0; j < SPB / BT; ++j) {
        const int p = blockIdx.x * SPB + j * BT + threadIdx.x;
        const bool valid = p < r.n;
        int i = 0, v = 256;
        if (valid) {
            i = r.perm_in ? r.perm_in[(size_t)t * r.n + p] : p;
            v = (r.keys[(size_t)t * r.key_tstride + i] >> r.shift) & 255;
        }
        const unsigned peers = __match_any_sync(0xffffffffu, v);
        const int rank = __popc(peers & ((1u << lane) - 1u));
        if (rank == 0) wc[w][v] = __popc(peers);
        __syncthreads();
        if (valid) {
            int before = run[v];
            for (int q = 0; q < w; ++q) before += wc[q][v];
            r.perm_out[(size_t)t * r.n + doff[v] + hb[v] + before + rank] = i;
        }
        __syncthreads();
        {
            int add = 0;
            for (int q = 0; q < BT / 32; ++q) {
                add += wc[q][threadIdx.x];
                wc[q][threadIdx.x] = 0;
            }
            run[threadIdx.x] += add;
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// M-step
// ---------------------------------------------------------------------------
// Label counts for k > 256 (one smem histogram per block, then global adds).
__global__ void __launch_bounds__(BT) label_count_kernel(Dev b) {
    const int t = blockIdx.y;
    if (b.done[t]) return;
    const int k = b.ks[task_s(b, t)];
    for (int e = blockIdx.x * BT + threadIdx.x; e < b.n; e += gridDim.x * BT)
        atomicAdd(&b.counts[(size_t)t * b.kst + b.labels[(size_t)t * b.n + e]], 1);
    (void)k;
}

// offsets, empty ranks (one CTA per task).  When from_radix, counts are the
// single-pass digit totals.
__global__ void __launch_bounds__(1024) cell_prefix_kernel(Dev b, int from_radix) {
    const int t = blockIdx.x;
    if (b.done[t]) return;
    const int k = b.ks[task_s(b, t)];
    __shared__ int carry_c, carry_e;
    if (threadIdx.x == 0) {
        carry_c = 0;
        carry_e = 0;
    }
    __syncthreads();
    for (int base = 0; base < k; base += blockDim.x) {
        const int c = base + threadIdx.x;
        int cnt = 0;
        if (c < k) {
            cnt = from_radix ? b.dig_tot[(size_t)t * 256 + c] : b.counts[(size_t)t * b.kst + c];
            if (from_radix) b.counts[(size_t)t * b.kst + c] = cnt;
        }
        // two block scans (counts, empties)
        int tot;
        int x = cnt, e = (c < k && cnt == 0) ? 1 : 0;
        const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
        int xs = x, es = e;
        for (int o = 1; o < 32; o <<= 1) {
            const int a1 = __shfl_up_sync(0xffffffffu, xs, o);
            const int a2 = __shfl_up_sync(0xffffffffu, es, o);
            if (lane >= o) {
                xs += a1;
                es += a2;
            }
        }
        __shared__ int wsx[32], wse[32];
        if (lane == 31) {
            wsx[w] = xs;
            wse[w] = es;
        }
        __syncthreads();
        if (w == 0) {
            int y1 = wsx[lane], y2 = wse[lane];
            for (int o = 1; o < 32; o <<= 1) {
                const int a1 = __shfl_up_sync(0xffffffffu, y1, o);
                const int a2 = __shfl_up_sync(0xffffffffu, y2, o);
                if (lane >= o) {
                    y1 += a1;
                    y2 += a2;
                }
            }
            wsx[lane] = y1;
            wse[lane] = y2;
        }
        __syncthreads();
        const int bx = (w ? wsx[w - 1] : 0) + carry_c;
        const int be = (w ? wse[w - 1] : 0) + carry_e;
        if (c < k) {
            b.offs[(size_t)t * (b.kst + 1) + c] = bx + xs - x;
            b.erank[(size_t)t * b.kst + c] = be + es - e;
        }
        tot = wsx[31];
        const int tote = wse[31];
        __syncthreads();
        if (threadIdx.x == 0) {
            carry_c += tot;
            carry_e += tote;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) b.offs[(size_t)t * (b.kst + 1) + k] = carry_c;
    // the M-step's launch order: cells by member count, largest first (ties by
    // index), so the longest sequential sums start in the first wave; by rank
    // against every other cell when k fits the block, in index order otherwise
    __shared__ int scnt[1024];
    __syncthreads();
    const int* cn = b.counts + (size_t)t * b.kst;
    int* ord = b.order + (size_t)t * b.kst;
    if (k <= (int)blockDim.x) {
        const int c = threadIdx.x;
        if (c < k) scnt[c] = cn[c];
        __syncthreads();
        if (c < k) {
            const int mine = scnt[c];
            int rank = 0;
            for (int c2 = 0; c2 < k; ++c2) {
                const int o = scnt[c2];
                rank += (o > mine || (o == mine && c2 < c)) ? 1 : 0;
            }
            ord[rank] = c;
        }
    } else {
        for (int c = threadIdx.x; c < k; c += blockDim.x) ord[c] = c;
    }
}

// centroid[c][d] = (sum over members in sample order) * (1 / size); empty cells
// take the iteration's next reseed draw (kmeans_core.cpp:268-311).
// One CTA per (task, centroid), the centroids of each task launched largest
// first (cell_prefix_kernel ranks them by member count) and the tasks
// interleaved, so the longest sums start in the first wave.  Each dim's sum
// is one chain of fp32 adds in sample order, so a cell's time is its member
// count times one add; the
// member rows are gathered by all four warps with 16-byte cp.async into a
// ring of MS_STAGES chunks (MS_CHUNK bf16 each), far enough ahead that warp 0,
// which owns the chains (lane l: bf16 pairs l and, for sub 128, l + 32),
// never waits on DRAM.
constexpr int MS_THREADS = 128;
constexpr int MS_STAGES = 4;
constexpr int MS_CHUNK = 8192;  // bf16 per stage: 256 / 128 / 64 rows of sub 32 / 64 / 128
template <int SUB>
__global__ void __launch_bounds__(MS_THREADS) msum_kernel(Dev b, int it, const int32_t* perm) {
    constexpr int NPAIR = SUB / 2;       // bf16 pairs per subvector (16, 32 or 64)
    constexpr bool TWO = NPAIR > 32;     // sub = 128: each lane owns pairs l and l + 32
    constexpr int ROWS = MS_CHUNK / SUB; // rows per stage
    constexpr int CPR = SUB / 8;         // 16-byte pieces per row
    const int t = blockIdx.x;  // tasks vary fastest: every task's largest cells launch first
    if (b.done[t]) return;
    const int k = b.ks[task_s(b, t)];
    if ((int)blockIdx.y >= k) return;
    const int c = b.order[(size_t)t * b.kst + blockIdx.y];
    extern __shared__ __align__(16) uint16_t mring[];  // [MS_STAGES][ROWS][SUB]
    const int tid = threadIdx.x, lane = tid & 31;
    const int cnt = b.counts[(size_t)t * b.kst + c];
    float* out = b.cent + ((size_t)t * b.kmax + c) * SUB;
    if (cnt == 0) {
        if (tid < 32) {
            const int r = b.erank[(size_t)t * b.kst + c];
            const uint16_t* row = sample_ptr(b, t, b.reseed[(size_t)it * b.kst + r]);
            for (int d = lane; d < SUB; d += 32) out[d] = bf16_bits_to_f32(row[d]);
        }
        return;
    }
    const int32_t* pm = perm + (size_t)t * b.n + b.offs[(size_t)t * (b.kst + 1) + c];
    const int nch = (cnt + ROWS - 1) / ROWS;
    auto stage = [&](int ch) {
        uint16_t* dst = mring + (size_t)(ch % MS_STAGES) * MS_CHUNK;
        const int m0 = ch * ROWS;
#pragma unroll
        for (int q = 0; q < ROWS * CPR / MS_THREADS; ++q) {
            const int e = tid + MS_THREADS * q;
            const int r = e / CPR, j = e - r * CPR;
            const bool live = m0 + r < cnt;
            const uint16_t* src = sample_ptr(b, t, live ? __ldg(pm + m0 + r) : 0) + 8 * j;
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(
                             static_cast<uint32_t>(__cvta_generic_to_shared(dst + r * SUB + 8 * j))),
                         "l"(src), "r"(live ? 16 : 0)
                         : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    // MS_STAGES - 1 chunks ahead; empty groups keep the group count uniform
#pragma unroll
    for (int ch = 0; ch < MS_STAGES - 1; ++ch) {
        if (ch < nch) stage(ch);
        else asm volatile("cp.async.commit_group;" ::: "memory");
    }
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
    const bool own = tid < 32 && (NPAIR >= 32 || lane < NPAIR);
    for (int ch = 0; ch < nch; ++ch) {
        asm volatile("cp.async.wait_group %0;" ::"n"(MS_STAGES - 2) : "memory");
        __syncthreads();  // chunk ch landed for every thread; chunk ch - 1's slot is free
        if (ch + MS_STAGES - 1 < nch) stage(ch + MS_STAGES - 1);
        else asm volatile("cp.async.commit_group;" ::: "memory");
        if (own) {
            const uint32_t* src = reinterpret_cast<const uint32_t*>(mring + (size_t)(ch % MS_STAGES) * MS_CHUNK) + lane;
            const int nb = min(ROWS, cnt - ch * ROWS);
            if (nb == ROWS) {
#pragma unroll 16
                for (int r = 0; r < ROWS; ++r) {
                    const uint32_t v = src[r * NPAIR];
                    s0 = __fadd_rn(s0, bf16lo(v));
                    s1 = __fadd_rn(s1, bf16hi(v));
                    if (TWO) {
                        const uint32_t w = src[r * NPAIR + 32];
                        s2 = __fadd_rn(s2, bf16lo(w));
                        s3 = __fadd_rn(s3, bf16hi(w));
                    }
                }
            } else {
                for (int r = 0; r < nb; ++r) {
                    const uint32_t v = src[r * NPAIR];
                    s0 = __fadd_rn(s0, bf16lo(v));
                    s1 = __fadd_rn(s1, bf16hi(v));
                    if (TWO) {
                        const uint32_t w = src[r * NPAIR + 32];
                        s2 = __fadd_rn(s2, bf16lo(w));
                        s3 = __fadd_rn(s3, bf16hi(w));
                    }
                }
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    if (own) {
        const float inv = __fdiv_rn(1.0f, (float)cnt);
        out[2 * lane] = __fmul_rn(s0, inv);
        out[2 * lane + 1] = __fmul_rn(s1, inv);
        if (TWO) {
            out[64 + 2 * lane] = __fmul_rn(s2, inv);
            out[65 + 2 * lane] = __fmul_rn(s3, inv);
        }
    }
}

// ---------------------------------------------------------------------------
// Reorganize (per head; reorganize_core.cpp:18-311)
// ---------------------------------------------------------------------------
IMI_DEV int comb_id(const Dev& b, const int32_t* sl, int h, int i) {
    int g = 0;
    for (int s = 0; s < b.S; ++s) g = g * b.ks[s] + sl[((size_t)h * b.S + s) * b.n + i];
    return g;
}

__global__ void reorg_mark_kernel(Dev b) {
    const int h = blockIdx.y;
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= b.n) return;
    b.used[(size_t)h * b.G + comb_id(b, b.labels, h, i)] = 1;
}

// compact ids in ascending Cartesian order; cell codes; n_active
__global__ void __launch_bounds__(1024) reorg_compact_kernel(Dev b, BuildArgs a) {
    const int h = blockIdx.x;
    __shared__ int wsum[32];
    __shared__ int carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    for (int base = 0; base < b.G; base += blockDim.x) {
        const int g = base + threadIdx.x;
        const int f = (g < b.G) ? b.used[(size_t)h * b.G + g] : 0;
        int x = f;
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) wsum[w] = x;
        __syncthreads();
        if (w == 0) {
            int y = wsum[lane];
            for (int o = 1; o < 32; o <<= 1) {
                const int z = __shfl_up_sync(0xffffffffu, y, o);
                if (lane >= o) y += z;
            }
            wsum[lane] = y;
        }
        __syncthreads();
        const int cidx = carry + (w ? wsum[w - 1] : 0) + x - f;
        if (g < b.G) {
            b.g2c[(size_t)h * b.G + g] = f ? cidx : -1;
            if (f && cidx < a.n_slots) {
                // packed digits, byte s = digit of subspace s
                int rem = g, code = 0;
                for (int s = b.S - 1; s >= 0; --s) {
                    const int dg = rem % b.ks[s];
                    rem /= b.ks[s];
                    code |= dg << (8 * s);
                }
                a.cell_code[(size_t)h * a.n_slots + cidx] = (b.S == 1) ? g : code;
            }
        }
        const int tot = wsum[31];
        __syncthreads();
        if (threadIdx.x == 0) carry += tot;
        __syncthreads();
    }
    if (threadIdx.x == 0) a.n_active[h] = carry;
}

// CSR offsets from the sorted member list: a new compact id starts at p
__global__ void reorg_offsets_kernel(Dev b, BuildArgs a, const int32_t* perm) {
    const int h = blockIdx.y;
    const int p = blockIdx.x * blockDim.x + threadIdx.x;
    if (p >= b.n) return;
    const int32_t* pm = perm + (size_t)h * b.n;
    const int f = b.g2c[(size_t)h * b.G + comb_id(b, b.labels, h, pm[p])];
    const int pf = p ? b.g2c[(size_t)h * b.G + comb_id(b, b.labels, h, pm[p - 1])] : -1;
    if (f != pf && f < a.n_slots) a.cell_offsets[(size_t)h * (a.n_slots + 1) + f] = p;
}

// padded per-slot metadata (indexing.py:108-174 layout)
__global__ void reorg_meta_kernel(Dev b, BuildArgs a) {
    const int h = blockIdx.y;
    const int na = a.n_active[h];
    const int c = blockIdx.x;
    if (c > a.n_slots) return;
    int32_t* offs = a.cell_offsets + (size_t)h * (a.n_slots + 1);
    if (c == a.n_slots || c >= na) {
        if (threadIdx.x == 0) offs[c] = b.n;
    }
    if (c == a.n_slots) return;
    const bool active = c < na;
    if (threadIdx.x == 0) {
        const int next = (c + 1 < na) ? offs[c + 1] : b.n;
        a.cell_sizes[(size_t)h * a.n_slots + c] = active ? next - offs[c] : 0;
        a.cell_mask[(size_t)h * a.n_slots + c] = active ? 0 : 1;
        if (!active) a.cell_code[(size_t)h * a.n_slots + c] = -1;
    }
    float* row = a.centroids + ((size_t)h * a.n_slots + c) * b.dim;
    const int code = active ? a.cell_code[(size_t)h * a.n_slots + c] : 0;
    for (int d = threadIdx.x; d < b.dim; d += blockDim.x) {
        float v = 0.0f;
        if (active) {
            const int s = d / b.sub, dd = d - s * b.sub;
            const int dg = (b.S == 1) ? code : ((code >> (8 * s)) & 0xff);
            v = b.cent[(((size_t)h * b.S + s) * b.kmax + dg) * b.sub + dd];
        }
        row[d] = v;
    }
}

// list rows in member order (reorganize_core.cpp:298-308)
__global__ void reorg_gather_kernel(Dev b, BuildArgs a, const int32_t* perm) {
    const int h = blockIdx.y;
    const int row = blockIdx.x * (blockDim.x / 16) + (threadIdx.x >> 4);
    const int q = threadIdx.x & 15;
    if (row >= b.n) return;
    const int src = perm[(size_t)h * b.n + row];
    const int n16 = b.dim * 2 / 16;
    for (int qq = q; qq < n16; qq += 16) {
        const uint4* sk = reinterpret_cast<const uint4*>(a.keys + (size_t)h * a.head_stride + (size_t)src * a.token_stride);
        const uint4* sv = reinterpret_cast<const uint4*>(a.values + (size_t)h * a.head_stride + (size_t)src * a.token_stride);
        reinterpret_cast<uint4*>(a.list_keys + ((size_t)h * a.list_rows + row) * b.dim)[qq] = __ldg(sk + qq);
        reinterpret_cast<uint4*>(a.list_values + ((size_t)h * a.list_rows + row) * b.dim)[qq] = __ldg(sv + qq);
    }
}

// device timestamp of a point in the build's stream order (per-stage times)
__global__ void stamp_kernel(unsigned long long* out) {
    if (threadIdx.x == 0) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        *out = t;
    }
}

// ---------------------------------------------------------------------------
// host orchestration
// ---------------------------------------------------------------------------
namespace {

struct Layout {
    size_t labels, md, perm_a, perm_b, part_lo, part_hi, part_minl, part_bad, hist, dig_off, dig_tot, counts, offs,
        erank, order, draws_u, first, reseed, done, prev, iters, used, g2c, chi, clo, cn, xn, tick, total;
    int npad;
};

// centroids per task rounded up to the MMA's N granularity; 0 when k > 256
// (the tensor-core E-step then is not used)
int tc_npad(int kmax) { return kmax <= 256 ? ((kmax + 15) / 16) * 16 : 0; }

Layout layout(int heads, int n, int dim, int parts, const int* ks, int max_iters, bool own_labels) {
    const int S = parts == 0 ? 1 : parts;
    const int T = heads * S;
    int kmax = 1;
    long long G = 1;
    for (int s = 0; s < S; ++s) {
        kmax = std::max(kmax, ks[s]);
        G *= ks[s];
    }
    const int NB = (n + SPB - 1) / SPB;
    Layout L{};
    size_t o = 0;
    auto take = [&](size_t bytes) {
        size_t r = o;
        o += (bytes + 255) & ~size_t(255);
        return r;
    };
    L.labels = own_labels ? take((size_t)T * n * 4) : 0;
    L.md = take((size_t)T * n * 4);
    L.perm_a = take((size_t)T * n * 4);
    L.perm_b = take((size_t)T * n * 4);
    L.part_lo = take((size_t)T * NB * 8);
    L.part_hi = take((size_t)T * NB * 8);
    L.part_minl = take((size_t)T * NB * 4);
    L.part_bad = take((size_t)T * NB * 4);
    L.hist = take((size_t)T * NB * 256 * 4);
    L.dig_off = take((size_t)T * 256 * 4);
    L.dig_tot = take((size_t)T * 256 * 4);
    L.counts = take((size_t)T * kmax * 4);
    L.offs = take((size_t)T * (kmax + 1) * 4);
    L.erank = take((size_t)T * kmax * 4);
    L.order = take((size_t)T * kmax * 4);
    L.draws_u = take((size_t)S * kmax * 8);
    L.first = take((size_t)S * 4);
    L.reseed = take((size_t)std::max(1, max_iters) * kmax * 4);
    L.done = take((size_t)T * 4);
    L.prev = take((size_t)T * 4);
    L.iters = take((size_t)T * 4);
    L.used = take((size_t)heads * G);
    L.g2c = take((size_t)heads * G * 4);
    L.npad = tc_npad(kmax);
    const size_t sub = (size_t)dim / S;
    L.chi = take((size_t)T * L.npad * (sub + 16) * 2);
    L.clo = take((size_t)T * L.npad * (sub + 16) * 2);
    L.cn = take((size_t)T * L.npad * 4);
    L.xn = take(L.npad > 0 ? (size_t)T * ((n + 127) / 128 * 128) * 4 : 0);
    L.tick = take((size_t)T * 4);
    L.total = o;
    return L;
}

}  // namespace

size_t build_workspace_bytes(int heads, int n, int dim, int parts, const int* ks) {
    // sized for up to 64 Lloyd iterations of reseed draws
    return layout(heads, n, dim, parts, ks, 64, true).total;
}

template <int SUB>
static cudaError_t run_kmeans_sub(Dev& d, const BuildArgs& a, cudaStream_t st) {
    cudaError_t e;
    // ---- k-means++
    kpp_first_kernel<<<d.T, 128, 0, st>>>(d);
    int kmax_all = 0;
    for (int s = 0; s < d.S; ++s) kmax_all = std::max(kmax_all, d.ks[s]);
    const size_t step_smem = kpp_step_smem<SUB>(d.NB);
    if ((e = cudaFuncSetAttribute(kpp_step_kernel<SUB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)step_smem)) != cudaSuccess)
        return e;
    // One launch per step over every task.  (Steps over groups of tasks whose
    // samples stay resident in L2 were measured slower: 4 groups of 4 tasks
    // took 148.7 ms against 116.3 ms for 8 config-1 layers -- the per-step
    // launch and draw latency outweighs the saved HBM traffic.)
    for (int c = 1; c < kmax_all; ++c)
        if ((e = launch_pdl(kpp_step_kernel<SUB>, dim3(d.NB, d.T), dim3(BT), step_smem, st, d, c, 0)) != cudaSuccess)
            return e;
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    // ---- Lloyd
    const int chunk = std::min(kmax_all, 32768 / SUB);
    const size_t es_smem = (size_t)chunk * SUB * 4;
    if ((e = cudaFuncSetAttribute(estep_kernel<SUB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)es_smem)) !=
        cudaSuccess)
        return e;
    const int two_pass = kmax_all > 256;
    // tensor-core E-step when every task's k fits one MMA (N <= 256)
    // tensor-core E-step when every task's k fits one MMA (N <= 256), the
    // operands fit shared memory and the keys can be described to the TMA unit
    int tc_acc = 32, tc_ctas = 1, tc_tiles = 1, tc_stages = 0;
    size_t tc_smem_bytes = 0;
    CUtensorMap tmap;
    bool tc = d.npad > 0 && encode_sample_map(d, &tmap);
    if (tc) {
        while (tc_acc < d.npad) tc_acc <<= 1;  // four accumulators of tc_acc columns
        const size_t fixed = (size_t)TC_M * 16 * 2 + 2 * (size_t)d.npad * (SUB + 16) * 2 + 64 * 8 +
                             (size_t)kmax_all * (SUB + 4) * 4;
        const size_t per_stage = (size_t)TC_M * SUB * 2 + TC_M * 4;
        const size_t room = 232448 - 8192;  // less the static exchange arrays
        tc_stages = (int)std::min<size_t>(TC_MAX_STAGES, room > fixed ? (room - fixed) / per_stage : 0);
        tc = tc_acc * 4 <= 512 && tc_stages >= 2;
        if (tc) {
            tc_smem_bytes = fixed + (size_t)tc_stages * per_stage + 1024;
            // more than half the SM's shared memory: one CTA (and its 512
            // TMEM columns) per SM
            tc_smem_bytes = std::max(tc_smem_bytes, (size_t)120 * 1024);
            if ((e = cudaFuncSetAttribute(estep_tc_kernel<SUB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)tc_smem_bytes)) != cudaSuccess)
                return e;
            const int ntiles = (d.n + TC_M - 1) / TC_M;
            tc_ctas = std::max(1, std::min(ntiles, 148 / d.T));
            tc_tiles = (ntiles + tc_ctas - 1) / tc_ctas;
            tc_ctas = (ntiles + tc_tiles - 1) / tc_tiles;
        }
    }
    const size_t ms_smem = (size_t)MS_STAGES * MS_CHUNK * 2;
    if ((e = cudaFuncSetAttribute(msum_kernel<SUB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ms_smem)) !=
        cudaSuccess)
        return e;
    if (tc) xnorm_kernel<SUB><<<dim3((d.nx + BT - 1) / BT, d.T), BT, 0, st>>>(d);
    for (int it = 0; it < a.max_iters; ++it) {
        // the inertia (and so the exact min distances) is only needed from
        // two iterations before the first one allowed to stop
        const int eval = it >= std::max(0, a.early_stop_min_iter - 2) ? 1 : 0;
        if (tc) {
            cent_split_kernel<SUB><<<dim3(d.npad, d.T), 32, 0, st>>>(d);
            estep_tc_kernel<SUB><<<dim3(tc_ctas, d.T), TC_CTA_THREADS, tc_smem_bytes, st>>>(d, tmap, tc_tiles, tc_acc,
                                                                                            tc_stages, eval);
        } else {
            estep_kernel<SUB><<<dim3((d.n + BT - 1) / BT, d.T), BT, es_smem, st>>>(d);
        }
        inertia_kernel<<<d.T, IN_THREADS, 0, st>>>(d, it, a.max_iters, a.early_stop_min_iter, a.tol, a.early_stop_rel_tol,
                                            eval);
        Radix r{};
        r.T = d.T;
        r.n = d.n;
        r.NB = d.NB;
        r.keys = d.labels;
        r.key_tstride = d.n;
        r.hist = d.hist;
        r.dig_off = d.dig_off;
        r.dig_tot = d.dig_tot;
        r.gate = d.done;
        r.shift = 0;
        r.perm_in = nullptr;
        r.perm_out = d.perm_a;
        radix_hist_kernel<<<dim3(d.NB, d.T), BT, 0, st>>>(r);
        radix_scan_kernel<<<d.T, 256, 0, st>>>(r);
        radix_scatter_kernel<<<dim3(d.NB, d.T), BT, 0, st>>>(r);
        const int32_t* perm = d.perm_a;
        if (two_pass) {
            r.shift = 8;
            r.perm_in = d.perm_a;
            r.perm_out = d.perm_b;
            radix_hist_kernel<<<dim3(d.NB, d.T), BT, 0, st>>>(r);
            radix_scan_kernel<<<d.T, 256, 0, st>>>(r);
            radix_scatter_kernel<<<dim3(d.NB, d.T), BT, 0, st>>>(r);
            perm = d.perm_b;
            cudaMemsetAsync(d.counts, 0, (size_t)d.T * d.kst * 4, st);
            label_count_kernel<<<dim3(std::min(d.NB, 64), d.T), BT, 0, st>>>(d);
        }
        cell_prefix_kernel<<<d.T, 1024, 0, st>>>(d, two_pass ? 0 : 1);
        msum_kernel<SUB><<<dim3(d.T, kmax_all), MS_THREADS, ms_smem, st>>>(d, it, perm);
    }
    return cudaGetLastError();
}

cudaError_t run_build(const BuildArgs& a, cudaStream_t st, const char** why) {
    const int S = a.parts == 0 ? 1 : a.parts;
    if (!(a.parts == 0 || a.parts == 2 || a.parts == 4)) {
        *why = "parts must be 0, 2 or 4";
        return cudaErrorInvalidValue;
    }
    if (a.dim % (8 * S) != 0 || a.dim != 128) {
        *why = "dim must be 128";
        return cudaErrorInvalidValue;
    }
    const int sub = a.dim / S;
    int kmax = 1;
    long long G = 1;
    for (int s = 0; s < S; ++s) {
        if (a.ks[s] < 1 || (S > 1 && a.ks[s] > 255) || a.ks[s] > 65536) {
            *why = "k per subspace must be in [1, 255] (IMI) or [1, 65536] (IVF)";
            return cudaErrorInvalidValue;
        }
        kmax = std::max(kmax, a.ks[s]);
        G *= a.ks[s];
    }
    if (G > (1ll << 26)) {
        *why = "product of k over subspaces too large";
        return cudaErrorInvalidValue;
    }
    if (a.n_tokens < 1 || a.n_tokens > (1 << 23)) {
        *why = "token count must be in [1, 2^23]";
        return cudaErrorInvalidValue;
    }
    if (a.kmax < kmax) {
        *why = "sub_centroids stride kmax smaller than max k";
        return cudaErrorInvalidValue;
    }
    if (a.max_iters < 1 || a.max_iters > 64) {
        *why = "max_iters must be in [1, 64]";
        return cudaErrorInvalidValue;
    }
    if ((a.token_stride * 2) % 16 != 0 || (a.head_stride * 2) % 16 != 0 ||
        (reinterpret_cast<uintptr_t>(a.keys) & 15) || (reinterpret_cast<uintptr_t>(a.values) & 15)) {
        *why = "keys/values and their strides must be 16-byte aligned";
        return cudaErrorInvalidValue;
    }
    const bool own_labels = a.sub_labels == nullptr;
    const Layout L = layout(a.heads, a.n_tokens, a.dim, a.parts, a.ks, 64, own_labels);
    if (a.workspace_bytes < L.total || a.workspace == nullptr) {
        *why = "workspace too small (see imi_build_workspace_size)";
        return cudaErrorInvalidValue;
    }
    unsigned char* ws = static_cast<unsigned char*>(a.workspace);
    Dev d{};
    d.heads = a.heads;
    d.n = a.n_tokens;
    d.dim = a.dim;
    d.S = S;
    d.sub = sub;
    d.T = a.heads * S;
    d.kmax = a.kmax;
    d.kst = kmax;
    d.NB = (a.n_tokens + SPB - 1) / SPB;
    for (int s = 0; s < 4; ++s) d.ks[s] = s < S ? a.ks[s] : 1;
    d.keys = a.keys;
    d.hstride = a.head_stride;
    d.tstride = a.token_stride;
    d.cent = a.sub_centroids;
    d.labels = own_labels ? reinterpret_cast<int32_t*>(ws + L.labels) : a.sub_labels;
    d.md = reinterpret_cast<float*>(ws + L.md);
    d.perm_a = reinterpret_cast<int32_t*>(ws + L.perm_a);
    d.perm_b = reinterpret_cast<int32_t*>(ws + L.perm_b);
    d.part_lo = reinterpret_cast<unsigned long long*>(ws + L.part_lo);
    d.part_hi = reinterpret_cast<unsigned long long*>(ws + L.part_hi);
    d.part_minl = reinterpret_cast<int32_t*>(ws + L.part_minl);
    d.part_bad = reinterpret_cast<int32_t*>(ws + L.part_bad);
    d.hist = reinterpret_cast<int32_t*>(ws + L.hist);
    d.dig_off = reinterpret_cast<int32_t*>(ws + L.dig_off);
    d.dig_tot = reinterpret_cast<int32_t*>(ws + L.dig_tot);
    d.counts = reinterpret_cast<int32_t*>(ws + L.counts);
    d.offs = reinterpret_cast<int32_t*>(ws + L.offs);
    d.erank = reinterpret_cast<int32_t*>(ws + L.erank);
    d.order = reinterpret_cast<int32_t*>(ws + L.order);
    d.draws_u = reinterpret_cast<const double*>(ws + L.draws_u);
    d.first = reinterpret_cast<const int32_t*>(ws + L.first);
    d.reseed = reinterpret_cast<const int32_t*>(ws + L.reseed);
    d.done = reinterpret_cast<int32_t*>(ws + L.done);
    d.prev_inertia = reinterpret_cast<float*>(ws + L.prev);
    d.iters_run = reinterpret_cast<int32_t*>(ws + L.iters);
    d.used = ws + L.used;
    d.g2c = reinterpret_cast<int32_t*>(ws + L.g2c);
    d.npad = L.npad;
    d.chi = reinterpret_cast<uint16_t*>(ws + L.chi);
    d.clo = reinterpret_cast<uint16_t*>(ws + L.clo);
    d.cn = reinterpret_cast<float*>(ws + L.cn);
    d.xn = reinterpret_cast<float*>(ws + L.xn);
    d.nx = (d.n + 127) / 128 * 128;
    d.status = a.status;
    d.kpp_ticket = reinterpret_cast<uint32_t*>(ws + L.tick);
    d.G = (int)G;
    // per-cell work arrays use stride d.kst (max k); sub-centroids use a.kmax
    // ---- host draws (the reference's seeds, the same <random> algorithms)
    {
        const int dkmax = kmax;
        std::vector<double> du((size_t)S * dkmax, 0.0);
        std::vector<int32_t> first(S, 0);
        for (int s = 0; s < S; ++s) {
            std::mt19937_64 rng(42 + s);
            std::uniform_int_distribution<int32_t> pick(0, a.n_tokens - 1);
            first[s] = pick(rng);
            for (int c = 1; c < a.ks[s]; ++c) {
                std::uniform_real_distribution<double> ud(0.0, 1.0);
                du[(size_t)s * dkmax + c] = ud(rng);
            }
        }
        std::vector<int32_t> rs((size_t)a.max_iters * dkmax, 0);
        for (int it = 0; it < a.max_iters; ++it) {
            std::mt19937 rng(it + 12345);
            std::uniform_int_distribution<int32_t> pick(0, a.n_tokens - 1);
            for (int r = 0; r < dkmax; ++r) rs[(size_t)it * dkmax + r] = pick(rng);
        }
        cudaError_t e;
        if ((e = cudaMemcpyAsync(ws + L.draws_u, du.data(), du.size() * 8, cudaMemcpyHostToDevice, st)) != cudaSuccess)
            return e;
        if ((e = cudaMemcpyAsync(ws + L.first, first.data(), first.size() * 4, cudaMemcpyHostToDevice, st)) !=
            cudaSuccess)
            return e;
        if ((e = cudaMemcpyAsync(ws + L.reseed, rs.data(), rs.size() * 4, cudaMemcpyHostToDevice, st)) != cudaSuccess)
            return e;
        // prev_inertia = FLT_MAX
        std::vector<float> pv(d.T, FLT_MAX);
        if ((e = cudaMemcpyAsync(d.prev_inertia, pv.data(), pv.size() * 4, cudaMemcpyHostToDevice, st)) !=
            cudaSuccess)
            return e;
        // A copy from pageable host memory returns once the data is staged, so
        // the vectors may go out of scope here.  It also waits for the work
        // already in `st` (the previous build on that stream), but not for the
        // ready event below: the producer of the keys keeps running.
    }
    if (a.ready_event) {  // the keys / values are produced on another stream
        cudaError_t e = cudaStreamWaitEvent(st, static_cast<cudaEvent_t>(a.ready_event), 0);
        if (e != cudaSuccess) return e;
    }
    cudaMemsetAsync(d.done, 0, (size_t)d.T * 4, st);
    cudaMemsetAsync(d.kpp_ticket, 0, (size_t)d.T * 4, st);
    cudaMemsetAsync(d.iters_run, 0, (size_t)d.T * 4, st);
    cudaError_t e;
    if (a.phase_ns) stamp_kernel<<<1, 32, 0, st>>>(a.phase_ns);
    if (sub == 64) e = run_kmeans_sub<64>(d, a, st);
    else if (sub == 32) e = run_kmeans_sub<32>(d, a, st);
    else e = run_kmeans_sub<128>(d, a, st);
    if (e != cudaSuccess) return e;
    if (a.iters_run) cudaMemcpyAsync(a.iters_run, d.iters_run, (size_t)d.T * 4, cudaMemcpyDeviceToDevice, st);
    if (a.phase_ns) stamp_kernel<<<1, 32, 0, st>>>(a.phase_ns + 1);
    // ---- reorganize
    cudaMemsetAsync(d.used, 0, (size_t)a.heads * G, st);
    reorg_mark_kernel<<<dim3((a.n_tokens + 255) / 256, a.heads), 256, 0, st>>>(d);
    reorg_compact_kernel<<<a.heads, 1024, 0, st>>>(d, a);
    // stable sort of token indices by (digit_0, ..., digit_{S-1}): LSD passes
    Radix r{};
    r.T = a.heads;
    r.n = a.n_tokens;
    r.NB = d.NB;
    r.hist = d.hist;
    r.dig_off = d.dig_off;
    r.dig_tot = d.dig_tot;
    r.gate = nullptr;
    const int32_t* perm = nullptr;
    int32_t* bufs[2] = {d.perm_a, d.perm_b};
    int which = 0;
    auto pass = [&](const int32_t* keys, long long tstride, int shift) {
        r.keys = keys;
        r.key_tstride = tstride;
        r.shift = shift;
        r.perm_in = perm;
        r.perm_out = bufs[which];
        radix_hist_kernel<<<dim3(d.NB, a.heads), BT, 0, st>>>(r);
        radix_scan_kernel<<<a.heads, 256, 0, st>>>(r);
        radix_scatter_kernel<<<dim3(d.NB, a.heads), BT, 0, st>>>(r);
        perm = bufs[which];
        which ^= 1;
    };
    if (S == 1) {
        pass(d.labels, a.n_tokens, 0);
        if (kmax > 256) pass(d.labels, a.n_tokens, 8);
    } else {
        for (int s = S - 1; s >= 0; --s) pass(d.labels + (size_t)s * a.n_tokens, (long long)S * a.n_tokens, 0);
    }
    reorg_offsets_kernel<<<dim3((a.n_tokens + 255) / 256, a.heads), 256, 0, st>>>(d, a, perm);
    reorg_meta_kernel<<<dim3(a.n_slots + 1, a.heads), 128, 0, st>>>(d, a);
    reorg_gather_kernel<<<dim3((a.n_tokens + 15) / 16, a.heads), 256, 0, st>>>(d, a, perm);
    if (a.phase_ns) stamp_kernel<<<1, 32, 0, st>>>(a.phase_ns + 2);
    return cudaGetLastError();
}

}  // namespace imi
