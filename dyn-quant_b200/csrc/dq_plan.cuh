// dq_plan.cuh -- the activation plan shared by the GEMV kernels: block scan,
// the statistics of x and the outlier mask with the reference's capacity rule
// (src/outlier_detect.cuh:104-205).  Every kernel that derives a mask from an
// activation vector runs this code with the same fixed partition, so the
// batch-1 split GEMV, the batched split GEMV's plan kernel and the standalone
// detector agree bit for bit.
#pragma once

#include "dq_common.cuh"
#include "dq_internal.h"

namespace dq {

// ---------------------------------------------------------------------------
// Block-wide helpers (NT threads)
// ---------------------------------------------------------------------------

// Exclusive prefix sums over the threads (in thread order) of NV ints per
// thread, plus the totals.  scratch: NW * NV ints used by nothing else; one
// barrier.
template <int NT, int NV>
__device__ __forceinline__ void block_scan(const int (&v)[NV], int (&pre)[NV], int (&tot)[NV], int* scratch) {
    constexpr int NW = NT / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int incl[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) incl[i] = v[i];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int n = __shfl_up_sync(0xffffffffu, incl[i], o);
            if (lane >= o) incl[i] += n;
        }
    }
    if (lane == 31)
#pragma unroll
        for (int i = 0; i < NV; ++i) scratch[warp * NV + i] = incl[i];
    __syncthreads();
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        int before = 0, all = 0;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            const int s = scratch[w * NV + i];
            before += (w < warp) ? s : 0;
            all += s;
        }
        pre[i] = before + incl[i] - v[i];
        tot[i] = all;
    }
}

__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
    return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

// ---------------------------------------------------------------------------
// Activation plan (per CTA, NT threads)
//
// The outlier mask follows the reference's detector definition
// (src/outlier_detect.cuh:104-205): mean and unbiased variance of x in FP32,
// thresh = k * sqrt(max(var, 1e-8)), outlier iff |x - mean| > thresh, and at
// most (d_in/4)/4 outliers kept per stripe class (columns c with
// (c/32) % 4 == w, the first ones in ascending order), as the reference's
// per-warp capacity does (src/outlier_detect.cuh:160-178).  Mean and variance
// are merged from per-thread two-pass summaries in a fixed order, so every CTA
// (and the standalone detector, which runs the same code with the same thread
// count) derives the same mask.
// ---------------------------------------------------------------------------

// x (d_in = 8 * n8 halves) from global memory into xs, natural order, as
// 16-byte cp.async copies (completed by cp_async_wait_all + a barrier).
template <int NT>
__device__ __forceinline__ void load_x_async(const uint16_t* __restrict__ x, int n8, uint4* xs) {
    for (int ch = threadIdx.x; ch < n8; ch += NT) cp_async16(smem_u32(xs + ch), x + 8 * static_cast<size_t>(ch));
    cp_async_commit();
}

struct XStats {
    float mean, thresh, var, m2;
};

// Sum of the 16 floats at p (16-byte aligned shared memory), fixed tree.
__device__ __forceinline__ float sum16_tree(const float* p) {
    const uint32_t a = smem_u32(p);
    const uint4 q0 = lds_v4(a), q1 = lds_v4(a + 16), q2 = lds_v4(a + 32), q3 = lds_v4(a + 48);
    auto f = [](uint32_t u) { return __uint_as_float(u); };
    const float s0 = (f(q0.x) + f(q0.y)) + (f(q0.z) + f(q0.w));
    const float s1 = (f(q1.x) + f(q1.y)) + (f(q1.z) + f(q1.w));
    const float s2 = (f(q2.x) + f(q2.y)) + (f(q2.z) + f(q2.w));
    const float s3 = (f(q3.x) + f(q3.y)) + (f(q3.z) + f(q3.w));
    return (s0 + s1) + (s2 + s3);
}

// Mean and unbiased variance of x (in xs), threshold k * sqrt(max(var, 1e-8)),
// reading x from shared memory (detector, batched plan kernel, streaming
// kernel).  The same
// partition and summation order as x_stats_regs: bit-identical statistics.
// Two passes (sum, then sum of squared deviations) over a fixed partition of
// kStatThreads virtual threads (virtual thread v: pieces v, v + 512, ...;
// xor butterfly within each virtual warp; virtual-warp totals summed in
// order), run by the NT real threads: every CTA of a launch, whatever its warp
// count, and the standalone detector get bit-identical statistics.
// inv_n = 1/d_in and inv_n1 = 1/(d_in - 1) come from the host.
// red: >= 32 floats, 16-byte aligned, not in use; two barriers.
// bar() synchronises the NT threads (warps 0 .. NT/32 - 1) running it.
template <int NT, class Bar>
__device__ __forceinline__ XStats x_stats_bar(const uint4* xs, int n8, int d_in, float k, float inv_n, float inv_n1,
                                              float* red, Bar bar) {
    constexpr int NW = NT / 32;
    constexpr int NWV = kStatThreads / 32;
    static_assert(NT <= kStatThreads && NT % 32 == 0, "statistics partition");
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int vw = warp; vw < NWV; vw += NW) {
        float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
        for (int ch = 32 * vw + lane; ch < n8; ch += kStatThreads) {
            const uint4 v = xs[ch];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t w = word_of(v, i);
                s[i] = add_f16_f32(hi16(w), add_f16_f32(lo16(w), s[i]));
            }
        }
        const float ws = warp_sum((s[0] + s[1]) + (s[2] + s[3]));
        if (lane == 0) red[vw] = ws;
    }
    bar();
    const float total = sum16_tree(red);
    XStats r;
    r.mean = __fmul_rn(total, inv_n);
    for (int vw = warp; vw < NWV; vw += NW) {
        float m[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
        for (int ch = 32 * vw + lane; ch < n8; ch += kStatThreads) {
            const uint4 v = xs[ch];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t w = word_of(v, i);
                const float d0 = sub_f16_f32(lo16(w), r.mean);
                const float d1 = sub_f16_f32(hi16(w), r.mean);
                m[i] = __fmaf_rn(d1, d1, __fmaf_rn(d0, d0, m[i]));
            }
        }
        const float wq = warp_sum((m[0] + m[1]) + (m[2] + m[3]));
        if (lane == 0) red[NWV + vw] = wq;
    }
    bar();
    const float m2 = sum16_tree(red + NWV);
    r.m2 = m2;
    r.var = (d_in > 1) ? __fmul_rn(m2, inv_n1) : 0.f;
    r.thresh = __fmul_rn(k, __fsqrt_rn(fmaxf(r.var, 1e-8f)));
    return r;
}

template <int NT>
__device__ __forceinline__ XStats x_stats(const uint4* xs, int n8, int d_in, float k, float inv_n, float inv_n1,
                                          float* red) {
    return x_stats_bar<NT>(xs, n8, d_in, k, inv_n, inv_n1, red, []() { __syncthreads(); });
}

// Outlier mask with the reference's capacity rule, and the ascending outlier
// list (column | FP16 bits of x << 16).  Thread tid owns the 32-column stripe
// words [w0, w1) (at most 4; word wj = columns 32 wj .. 32 wj + 31, stripe
// class wj % 4): it computes their bits, the block scan of the per-class
// counts gives each class's count before it, and the capacity keeps the first
// (d_in/4)/4 of each class in column order.  Writes mask32 and list; returns
// the outlier count.  Barrier-synchronised; the list and mask are complete
// after the caller's next barrier.  scratch: >= NW * 5 ints used by nothing
// else.  list may be null (the mask only).
template <int NT>
__device__ int x_mask_list(const uint4* xs, int d_in, float mean, float thresh, uint32_t* mask32, uint32_t* list,
                           int* scratch) {
    constexpr int kMaxWords = 4;
    static_assert(kMaxDIn / 32 <= kMaxWords * NT, "stripe words per thread");
    const int nw = d_in / 32;
    const int tid = threadIdx.x;
    const int w0 = static_cast<int>(static_cast<long long>(tid) * nw / NT);
    const int w1 = static_cast<int>(static_cast<long long>(tid + 1) * nw / NT);
    uint32_t bits[kMaxWords];
    int cnt[4] = {0, 0, 0, 0};
#pragma unroll
    for (int q = 0; q < kMaxWords; ++q) {
        bits[q] = 0;
        const int wj = w0 + q;
        if (wj < w1) {
#pragma unroll
            for (int p = 0; p < 4; ++p) {
                const uint4 v = xs[4 * wj + p];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint32_t w = word_of(v, i);
                    bits[q] |= (fabsf(sub_f16_f32(lo16(w), mean)) > thresh ? 1u : 0u) << (8 * p + 2 * i);
                    bits[q] |= (fabsf(sub_f16_f32(hi16(w), mean)) > thresh ? 1u : 0u) << (8 * p + 2 * i + 1);
                }
            }
            const int c = __popc(bits[q]);
#pragma unroll
            for (int i = 0; i < 4; ++i) cnt[i] += (wj & 3) == i ? c : 0;
        }
    }
    int pre[4], tot[4];
    block_scan<NT, 4>(cnt, pre, tot, scratch);
    const int cap = (d_in / 4) / 4;
    int pos;
    if (tot[0] > cap || tot[1] > cap || tot[2] > cap || tot[3] > cap) {
        int kept[1] = {0};
#pragma unroll
        for (int q = 0; q < kMaxWords; ++q) {
            const int wj = w0 + q;
            if (wj < w1) {
                uint32_t m = bits[q];
                const int c = __popc(m);
                const int w = wj & 3;
                const int before = w == 0 ? pre[0] : (w == 1 ? pre[1] : (w == 2 ? pre[2] : pre[3]));
                if (before + c > cap) {
                    int keep = cap - before;
                    uint32_t out = 0;
                    for (; keep > 0 && m; --keep) {
                        out |= m & (~m + 1u);
                        m &= m - 1u;
                    }
                    bits[q] = out;
                }
                kept[0] += __popc(bits[q]);
#pragma unroll
                for (int i = 0; i < 4; ++i) pre[i] += w == i ? c : 0;
            }
        }
        int p1[1], t1[1];
        block_scan<NT, 1>(kept, p1, t1, scratch + (NT / 32) * 4);
        pos = p1[0];
        tot[0] = t1[0];
        tot[1] = tot[2] = tot[3] = 0;
    } else {
        pos = (pre[0] + pre[1]) + (pre[2] + pre[3]);
    }
    const uint16_t* xh = reinterpret_cast<const uint16_t*>(xs);
#pragma unroll
    for (int q = 0; q < kMaxWords; ++q) {
        const int wj = w0 + q;
        if (wj < w1) {
            mask32[wj] = bits[q];
            uint32_t m = list ? bits[q] : 0u;
            while (m) {
                const int col = 32 * wj + (__ffs(m) - 1);
                list[pos++] = static_cast<uint32_t>(col) | (static_cast<uint32_t>(xh[col]) << 16);
                m &= m - 1u;
            }
        }
    }
    return (tot[0] + tot[1]) + (tot[2] + tot[3]);
}

// ---------------------------------------------------------------------------
// The rest of the batch-1 kernel's plan, in a balanced partition.
//
// x sits in natural order in xb (shared memory; the statistics came from
// x_stats over it).  Thread tid takes pieces p = tid + NT r (r < R), so every
// thread holds at most one piece more than any other, and the 16 pieces of a
// group are the 16 lanes of one half-warp in one round.  From its pieces each
// thread derives the outlier bits; a ballot prefix within each warp and the
// warp totals give the list positions.  After one barrier (every piece of x
// is in registers) xb is overwritten with the MMA B fragments of x', the
// per-group sums go to xp4 and the list is written.
// ---------------------------------------------------------------------------

// Outlier bits of one piece: bit 2i (2i + 1) for the low (high) half of word i.
__device__ __forceinline__ uint32_t piece_bits(const uint4& v, float mean, float thresh) {
    uint32_t b = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t w = word_of(v, i);
        b |= (fabsf(sub_f16_f32(lo16(w), mean)) > thresh ? 1u : 0u) << (2 * i);
        b |= (fabsf(sub_f16_f32(hi16(w), mean)) > thresh ? 1u : 0u) << (2 * i + 1);
    }
    return b;
}

// Block total of a per-thread count (every thread gets it).  wcnt: NT/32 ints
// not in use until the caller's next barrier; one barrier.
template <int NT>
__device__ __forceinline__ int block_count(int cnt, int* wcnt) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    cnt = static_cast<int>(__reduce_add_sync(0xffffffffu, static_cast<unsigned>(cnt)));
    if (lane == 0) wcnt[warp] = cnt;
    __syncthreads();
    int total = 0;
#pragma unroll
    for (int w = 0; w < NT / 32; ++w) total += wcnt[w];
    return total;
}

// Exclusive prefix of this thread's cnt over the block in (warp, lane) order
// and the block total (cnt < 2^8).  wcnt: NT/32 ints, 16-byte aligned, not in
// use; one barrier.
template <int NT>
__device__ __forceinline__ int plan_prefix(int cnt, int* wcnt, int& total) {
    constexpr int NW = NT / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const unsigned lt = (1u << lane) - 1u;
    int before = 0, wtot = 0;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
        const unsigned bal = __ballot_sync(0xffffffffu, (cnt >> b) & 1);
        before += __popc(bal & lt) << b;
        wtot += __popc(bal) << b;
    }
    if (lane == 0) wcnt[warp] = wtot;
    __syncthreads();
    int base = 0;
    total = 0;
    const uint32_t wa = smem_u32(wcnt);
#pragma unroll
    for (int w4 = 0; w4 < NW / 4; ++w4) {
        const uint4 c4 = lds_v4(wa + 16 * w4);
        const int c[4] = {static_cast<int>(c4.x), static_cast<int>(c4.y), static_cast<int>(c4.z), static_cast<int>(c4.w)};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            base += 4 * w4 + i < warp ? c[i] : 0;
            total += c[i];
        }
    }
    return base + before;
}

// The plan after the statistics (kMask) or the fragments of x alone (INT4
// GEMV).  R: rounds, at least ceil(64 NC / NT).
//   xb   in: x in natural order (n8 pieces); out: [NC][64] 16-byte pieces in
//        MMA B order [word wi][slice sl][group jj], the f16 pairs (x0,x4),
//        (x2,x6), (x1,x5), (x3,x7) of each piece of x'; pieces past d_in (to
//        the end of the last chunk) are zero
//   xp4  [4 NC] per group (1024 sum x' even columns, 1024 sum x' odd columns,
//        sum x', 0); groups past d_in are zero
//   list the outliers (column | FP16 bits of x << 16) in (warp, lane, round)
//        order; with more than d_in/16 outliers the reference's capacity
//        rule decides the mask (x_mask_list over all of x; mask32 receives
//        it)
// red: kB1RedBytes of shared memory not in use.  Returns the outlier count
// (every thread); everything is complete on return (ends with a barrier).
// Column slabs (kSlab): xb holds only the pieces [piece0, piece0 + n8) of x
// (a slab of NC chunks); xfull is all of x in natural order in shared memory
// and total_all the outlier count over all of x.  The list then holds the
// slab's outliers (columns of x) in (warp, lane, round) order also under the
// capacity rule, and the return value is their number.
template <int NT, int R, bool kMask, bool kSlab = false>
__device__ __forceinline__ int plan_balanced(uint4* xb, int n8, int NC, int d_in, float mean, float thresh,
                                             float4* xp4, uint32_t* list, uint32_t* mask32, int* red,
                                             const uint4* xfull = nullptr, int piece0 = 0, int total_all = 0) {
    static_assert(NT % 32 == 0 && NT <= 512, "plan threads");
    const int tid = threadIdx.x;
    const int npc = 64 * NC;
    uint4 v[R];
    uint32_t bits[R];
    int cnt = 0;
#pragma unroll
    for (int rr = 0; rr < R; ++rr) {
        const int p = tid + NT * rr;
        v[rr] = p < n8 ? xb[p] : make_uint4(0, 0, 0, 0);
        bits[rr] = (kMask && p < n8) ? piece_bits(v[rr], mean, thresh) : 0u;
        cnt += __popc(bits[rr]);
    }
    int total = 0, pos = 0;
    bool capacity = false;
    if (kMask && !kSlab) {
        pos = plan_prefix<NT>(cnt, red, total);
        if (total > d_in / 16) {
            // No stripe class can exceed its capacity ((d_in/4)/4) below this
            // total; above it the reference's rule may drop outliers.
            capacity = true;
            total = x_mask_list<NT>(xb, d_in, mean, thresh, mask32, list, red + 16);
            __syncthreads();
#pragma unroll
            for (int rr = 0; rr < R; ++rr) {
                const int p = tid + NT * rr;
                if (p < n8) bits[rr] = (mask32[p >> 2] >> (8 * (p & 3))) & 0xFFu;
            }
        }
    }
    if (kMask && kSlab) {
        pos = plan_prefix<NT>(cnt, red, total);
        if (total_all > d_in / 16) {
            // Under the capacity rule: the mask from all of x in column
            // order, then this thread's bits from it and the list positions
            // again.
            __syncthreads();  // every thread has read the warp counts (x_mask_list's scratch follows them)
            x_mask_list<NT>(xfull, d_in, mean, thresh, mask32, nullptr, red + 16);
            __syncthreads();
            cnt = 0;
#pragma unroll
            for (int rr = 0; rr < R; ++rr) {
                const int p = tid + NT * rr, pg = piece0 + p;
                bits[rr] = p < n8 ? (mask32[pg >> 2] >> (8 * (pg & 3))) & 0xFFu : 0u;
                cnt += __popc(bits[rr]);
            }
            pos = plan_prefix<NT>(cnt, red, total);
        }
    }
    __syncthreads();  // every piece of x is in registers: xb may be overwritten
#pragma unroll
    for (int rr = 0; rr < R; ++rr) {
        if (NT * rr >= npc) break;  // uniform
        const int p = tid + NT * rr;
        uint4 w = v[rr];
        const uint32_t b = bits[rr];
        if (b) {
            uint32_t keep[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
                keep[i] = ((b >> (2 * i)) & 1u ? 0u : 0x0000FFFFu) | ((b >> (2 * i + 1)) & 1u ? 0u : 0xFFFF0000u);
            w.x &= keep[0];
            w.y &= keep[1];
            w.z &= keep[2];
            w.w &= keep[3];
        }
        float pe = add_f16_f32(lo16(w.w), add_f16_f32(lo16(w.z), add_f16_f32(lo16(w.y), add_f16_f32(lo16(w.x), 0.f))));
        float po = add_f16_f32(hi16(w.w), add_f16_f32(hi16(w.z), add_f16_f32(hi16(w.y), add_f16_f32(hi16(w.x), 0.f))));
        if (p < npc) {
            const int c = p >> 6, i = p & 63;
            const int jj = i >> 4, sl = (i >> 2) & 3, wi = i & 3;
            xb[64 * c + (wi * 4 + sl) * 4 + jj] =
                make_uint4((w.x & 0xFFFFu) | (w.z << 16), (w.y & 0xFFFFu) | (w.w << 16),
                           (w.x >> 16) | (w.z & 0xFFFF0000u), (w.y >> 16) | (w.w & 0xFFFF0000u));
        }
        // the 16 pieces of a group are the 16 lanes of one half-warp
#pragma unroll
        for (int o = 8; o >= 1; o >>= 1) {
            pe += __shfl_xor_sync(0xffffffffu, pe, o);
            po += __shfl_xor_sync(0xffffffffu, po, o);
        }
        if ((p & 15) == 0 && p < npc) xp4[p >> 4] = make_float4(1024.f * pe, 1024.f * po, pe + po, 0.f);
    }
    if (kMask && !capacity) {
#pragma unroll
        for (int rr = 0; rr < R; ++rr) {
            uint32_t b = bits[rr];
            const int p = (kSlab ? piece0 : 0) + tid + NT * rr;
            while (b) {
                const int e = __ffs(b) - 1;
                const uint32_t word = word_of(v[rr], e >> 1);
                const uint32_t h = (e & 1) ? (word >> 16) : (word & 0xFFFFu);
                list[pos++] = static_cast<uint32_t>(8 * p + e) | (h << 16);
                b &= b - 1u;
            }
        }
    }
    __syncthreads();
    return total;
}

}  // namespace dq
