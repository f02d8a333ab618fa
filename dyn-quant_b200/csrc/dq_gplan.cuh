// dq_gplan.cuh -- the activation plan of the streaming kernel in the group
// partition: the outlier mask with the reference's capacity rule
// (src/outlier_detect.cuh:104-205), the MMA B fragments of the masked
// activation x', its per-group sums and the outlier list, computed by up to
// kPlanThreads threads from registers.  (The statistics themselves come from
// x_stats_bar of dq_plan.cuh, the partition every kernel shares, so that all
// kernels derive the same mask bit for bit.)
//
// Partition.  x (d_in = 128 G columns) is G groups of 16 pieces (a piece is 8
// consecutive columns, 16 bytes).  Plan thread tau = TPG j + h (TPG threads per
// group, the largest of 16, 8, 4, 2, 1 with G TPG <= kPlanThreads) holds the
// PPT = 16 / TPG consecutive pieces 16 j + PPT h .. 16 j + PPT h + PPT - 1 of
// group j.  The per-group sums of x' run in a fixed order (per thread over its
// pieces, then a xor butterfly over the group's TPG lanes).
#pragma once

#include "dq_common.cuh"
#include "dq_internal.h"

namespace dq {

constexpr int kPlanThreads = 480;  // plan threads of the partition (15 warps)
constexpr int kPlanWarps = kPlanThreads / 32;

// Threads per group of the partition for G groups.
__host__ __device__ inline int gp_tpg(int G) {
    int p = 16;
    while (p > 1 && G * p > kPlanThreads) p >>= 1;
    return p;
}

__device__ __forceinline__ uint32_t gp_word(const uint4& v, int i) {
    return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

// The pieces of plan thread tau (tau < G TPG), or zeros.
template <int kPPT>
struct GpRegs {
    uint4 v[kPPT];
};

template <int kPPT>
__device__ __forceinline__ void gp_load(const uint16_t* __restrict__ x, int G, int tau, GpRegs<kPPT>& r) {
    constexpr int TPG = 16 / kPPT;
#pragma unroll
    for (int i = 0; i < kPPT; ++i) r.v[i] = make_uint4(0, 0, 0, 0);
    if (tau < G * TPG) {
        const int j = tau / TPG, h = tau % TPG;
        const uint4* src = reinterpret_cast<const uint4*>(x) + 16 * j + kPPT * h;
#pragma unroll
        for (int i = 0; i < kPPT; ++i) r.v[i] = ldcg_v4(src + i);
    }
}

// Same pieces from x in shared memory (natural order).
template <int kPPT>
__device__ __forceinline__ void gp_load_smem(const uint4* xs, int G, int tau, GpRegs<kPPT>& r) {
    constexpr int TPG = 16 / kPPT;
#pragma unroll
    for (int i = 0; i < kPPT; ++i) r.v[i] = make_uint4(0, 0, 0, 0);
    if (tau < G * TPG) {
        const int j = tau / TPG, h = tau % TPG;
#pragma unroll
        for (int i = 0; i < kPPT; ++i) r.v[i] = xs[16 * j + kPPT * h + i];
    }
}

// Outlier bits of one piece: bit 2i (2i + 1) for the low (high) half of word i.
__device__ __forceinline__ uint32_t gp_piece_bits(const uint4& v, float mean, float thresh) {
    uint32_t b = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t w = gp_word(v, i);
        b |= (fabsf(sub_f16_f32(lo16(w), mean)) > thresh ? 1u : 0u) << (2 * i);
        b |= (fabsf(sub_f16_f32(hi16(w), mean)) > thresh ? 1u : 0u) << (2 * i + 1);
    }
    return b;
}

// Exclusive prefix of v over plan threads 0 .. 32 NW - 1 in thread order, and
// the total.  scratch: NW ints (16-byte aligned, multiple of 4) not in use;
// one bar().
template <int NW, class Bar>
__device__ __forceinline__ int gp_scan(int v, int* scratch, int& total, Bar bar) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
    }
    if (lane == 31) scratch[warp] = incl;
    bar();
    int before = 0, all = 0;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
        const int sw = scratch[w];
        before += w < warp ? sw : 0;
        all += sw;
    }
    total = all;
    return before + incl - v;
}

// The mask of the reference's capacity rule (at most (d_in/4)/4 outliers per
// stripe class (c/32) % 4, the first ones in column order), from the
// unlimited bits of every piece: mask32[d_in/32] in shared memory.  Plan
// thread tau owns the stripe words [tau nw / NT, (tau + 1) nw / NT) of xs
// (x in natural order in shared memory); scratch: 4 x 16 ints.  Five bar().
template <int NW, class Bar>
__device__ void gp_capacity_mask(const uint4* xs, int d_in, float mean, float thresh, uint32_t* mask32, int* scratch,
                                 Bar bar) {
    constexpr int NT = 32 * NW;
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
            for (int p = 0; p < 4; ++p) bits[q] |= gp_piece_bits(xs[4 * wj + p], mean, thresh) << (8 * p);
            const int c = __popc(bits[q]);
#pragma unroll
            for (int i = 0; i < 4; ++i) cnt[i] += (wj & 3) == i ? c : 0;
        }
    }
    int pre[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        int tot;
        pre[i] = gp_scan<NW>(cnt[i], scratch + i * 16, tot, bar);
    }
    const int cap = (d_in / 4) / 4;
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
#pragma unroll
            for (int i = 0; i < 4; ++i) pre[i] += w == i ? c : 0;
            mask32[wj] = bits[q];
        }
    }
    bar();
}

// The MMA B fragments of x' (x with the outliers zeroed), its per-group sums
// and the outlier list, from the registers of the partition.
//   xb   [NC][64] 16-byte pieces in MMA B order [word wi][slice sl][group jj]:
//        the f16 pairs (x0,x4), (x2,x6), (x1,x5), (x3,x7) of each piece; the
//        caller zeroes the pieces of the groups past d_in in the last chunk
//        (they lie interleaved with the real groups' pieces)
//   xp4  [G] per group (1024 sum x' even columns, 1024 sum x' odd columns,
//        sum x', 0)
//   list the outliers in column order, column | FP16 bits of x << 16
// kMask false: no mask (the INT4 GEMV).  mask32: null to derive the mask
// from (mean, thresh), else the mask words to apply (the capacity rule).
// Returns the outlier count (every thread).  scratch: NW ints not in use.
// When the count exceeds cap the list is not written (the caller applies the
// capacity rule and calls again with its mask).  One bar() (kMask).
template <int kPPT, int NW, bool kMask, class Bar>
__device__ __forceinline__ int gp_frags(const GpRegs<kPPT>& r, int G, float mean, float thresh,
                                        const uint32_t* mask32, int cap, uint4* xb, float4* xp4, uint32_t* list,
                                        int* scratch, Bar bar) {
    constexpr int TPG = 16 / kPPT;
    const int tau = threadIdx.x;
    const bool mine = tau < G * TPG;
    const int j = tau / TPG, h = tau % TPG;
    uint32_t bits[kPPT];
    int cnt = 0;
    float pe = 0.f, po = 0.f;
#pragma unroll
    for (int i = 0; i < kPPT; ++i) {
        bits[i] = 0;
        uint4 w = r.v[i];
        const int p = 16 * j + kPPT * h + i;  // piece index
        if (kMask && mine) {
            bits[i] = mask32 ? (mask32[p >> 2] >> (8 * (p & 3))) & 0xFFu : gp_piece_bits(w, mean, thresh);
            cnt += __popc(bits[i]);
            const uint32_t b = bits[i];
            if (b) {
                uint32_t keep[4];
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    keep[e] = ((b >> (2 * e)) & 1u ? 0u : 0x0000FFFFu) | ((b >> (2 * e + 1)) & 1u ? 0u : 0xFFFF0000u);
                w.x &= keep[0];
                w.y &= keep[1];
                w.z &= keep[2];
                w.w &= keep[3];
            }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const uint32_t u = gp_word(w, e);
            pe = add_f16_f32(lo16(u), pe);
            po = add_f16_f32(hi16(u), po);
        }
        if (mine) {
            const int c = p >> 6, q = p & 63;
            const int jj = q >> 4, sl = (q >> 2) & 3, wi = q & 3;
            xb[64 * c + (wi * 4 + sl) * 4 + jj] =
                make_uint4((w.x & 0xFFFFu) | (w.z << 16), (w.y & 0xFFFFu) | (w.w << 16),
                           (w.x >> 16) | (w.z & 0xFFFF0000u), (w.y >> 16) | (w.w & 0xFFFF0000u));
        }
    }
    // the TPG threads of a group are consecutive lanes: fixed butterfly
#pragma unroll
    for (int o = 1; o < TPG; o <<= 1) {
        pe += __shfl_xor_sync(0xffffffffu, pe, o);
        po += __shfl_xor_sync(0xffffffffu, po, o);
    }
    if (mine && h == 0) xp4[j] = make_float4(1024.f * pe, 1024.f * po, pe + po, 0.f);
    if (!kMask) return 0;
    int total;
    int pos = gp_scan<NW>(cnt, scratch, total, bar);
    if (total > cap) return total;
#pragma unroll
    for (int i = 0; i < kPPT; ++i) {
        uint32_t b = bits[i];
        const int p = 16 * j + kPPT * h + i;
        while (b) {
            const int e = __ffs(b) - 1;
            const uint32_t word = gp_word(r.v[i], e >> 1);
            const uint32_t hv = (e & 1) ? (word >> 16) : (word & 0xFFFFu);
            list[pos++] = static_cast<uint32_t>(8 * p + e) | (hv << 16);
            b &= b - 1u;
        }
    }
    return total;
}

}  // namespace dq
