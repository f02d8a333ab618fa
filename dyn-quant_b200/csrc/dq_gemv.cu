// dq_gemv.cu -- batch-1 GEMV kernels for sm_100a: fused split (INT4 + FP16
// outlier columns), dense INT4, dense FP16, and the standalone detector.
//
// Reference path (dyn-quant): src/split_gemv.cu:25-198, src/int4_gemv.cu:12-100,
// src/reference_gemv.cu:9-78, src/outlier_detect.cuh:104-205.
//
// Design (one launch per GEMV, no global scratch):
//   * Persistent grid, one 512-thread CTA per SM.  CTA c owns a contiguous
//     range of 16-row blocks; its (row-block, 128-column group) "units" are
//     split into equal contiguous ranges, one per warp.  All of a CTA's units
//     are read exactly once from HBM with 16-byte streaming loads.
//   * Every CTA first issues the packed-weight loads of its first units, then
//     runs the activation prologue (mean / variance / threshold / mask /
//     per-group tables) on its own copy of x while those loads are in flight.
//     All CTAs run the identical deterministic prologue, so all see one mask.
//   * The contraction runs on the tensor cores: mma.sync.m16n8k16 with the
//     dequantised codes q (exact small integers in f16) as A and the masked
//     activation as B (column 0; the other 7 columns are zero), FP32
//     accumulate.  Per (row, group): y += s * (sum_c q_c x'_c - z * sum_c x'_c)
//     where x' has the outlier channels zeroed -- the same value as the
//     reference's sum of s*(q-z)*x over non-outlier channels.
//   * Outlier channels add W16[r][c] * x[c] from the FP16 weights (column-major
//     mirror: 16 rows of one column = one 32-byte sector), prefetched with the
//     unit they belong to.
//   * Row sums are combined across warps through shared memory in a fixed
//     order and written once as FP16.
#include <cfloat>
#include <climits>

#include "dq_common.cuh"
#include "dq_internal.h"

namespace dq {

namespace {

constexpr int kNW = kGemvWarps;     // warps per CTA
constexpr int kNT = kNW * 32;       // threads per CTA
constexpr int kDepth = 4;           // units in flight per warp

// ---------------------------------------------------------------------------
// Activation prologue
// ---------------------------------------------------------------------------

// Loads x into shared memory and, for the split path, computes the outlier
// mask the way the reference's detector defines it (src/outlier_detect.cuh):
// mean and unbiased variance of x (two-pass, FP32, fixed reduction order),
// thresh = k * sqrt(max(var, 1e-8)), outlier iff |x - mean| > thresh, and at
// most (d_in/4)/4 outliers kept per stripe class (columns c with
// (c/32) % 4 == w; the first ones in ascending order), as the reference's
// per-warp capacity does (src/outlier_detect.cuh:160-178).
// Then builds, per 128-column group j:
//   Bsm[j][wi][t]  the MMA B fragments of x' (outliers zeroed)
//   Xp[j]          sum of x' over the group (FP32)
//   goff[j]        start of the group's outliers in `list` (ascending columns)
// misc[0..3] = mean, thresh, var, M2 (split path).
template <bool kSplit>
__device__ void activation_prologue(const uint16_t* __restrict__ x, int d_in, float k, char* smem,
                                    const SmemLayout& L) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = d_in / kGroup;
    const int n8 = d_in >> 3;
    uint4* sx4 = reinterpret_cast<uint4*>(smem + L.sx);
    uint8_t* smask = reinterpret_cast<uint8_t*>(smem + L.mask);
    float* red = reinterpret_cast<float*>(smem + L.misc);           // [0..31] reduction
    float* stat = red + 32;                                          // [32..35] stats
    int* stripe = reinterpret_cast<int*>(red + 40);                  // [40..43] counts

    if (tid < 4) stripe[tid] = 0;
    float sum = 0.f;
    for (int ch = tid; ch < n8; ch += kNT) {
        uint4 v = ldg_v4(x + 8 * static_cast<size_t>(ch));
        sx4[ch] = v;
        if (kSplit) {
            const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                sum += h2f_bits(static_cast<uint16_t>(wv[i] & 0xFFFFu));
                sum += h2f_bits(static_cast<uint16_t>(wv[i] >> 16));
            }
        }
    }

    if (kSplit) {
        const float total = block_sum<kNT>(sum, red);
        const float mean = __fdiv_rn(total, static_cast<float>(d_in));
        float m2 = 0.f;
        for (int ch = tid; ch < n8; ch += kNT) {
            const uint4 v = sx4[ch];
            const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float d0 = __fsub_rn(h2f_bits(static_cast<uint16_t>(wv[i] & 0xFFFFu)), mean);
                float d1 = __fsub_rn(h2f_bits(static_cast<uint16_t>(wv[i] >> 16)), mean);
                m2 = __fmaf_rn(d0, d0, m2);
                m2 = __fmaf_rn(d1, d1, m2);
            }
        }
        const float M2 = block_sum<kNT>(m2, red);
        const float var = (d_in > 1) ? __fdiv_rn(M2, static_cast<float>(d_in - 1)) : 0.f;
        const float thresh = __fmul_rn(k, __fsqrt_rn(fmaxf(var, 1e-8f)));
        if (tid == 0) {
            stat[0] = mean;
            stat[1] = thresh;
            stat[2] = var;
            stat[3] = M2;
        }
        for (int ch = tid; ch < n8; ch += kNT) {
            const uint4 v = sx4[ch];
            const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
            uint32_t byte = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float a = h2f_bits(static_cast<uint16_t>(wv[i] & 0xFFFFu));
                float b = h2f_bits(static_cast<uint16_t>(wv[i] >> 16));
                byte |= (fabsf(__fsub_rn(a, mean)) > thresh ? 1u : 0u) << (2 * i);
                byte |= (fabsf(__fsub_rn(b, mean)) > thresh ? 1u : 0u) << (2 * i + 1);
            }
            smask[ch] = static_cast<uint8_t>(byte);
            if (byte) atomicAdd(&stripe[(ch >> 2) & 3], __popc(byte));
        }
        __syncthreads();
        // Capacity rule (rare): keep the first warp_cap outliers of each stripe class.
        const int warp_cap = (d_in / 4) / 4;
        const bool over = stripe[0] > warp_cap || stripe[1] > warp_cap || stripe[2] > warp_cap ||
                          stripe[3] > warp_cap;
        if (over) {
            if (warp == 0 && lane < 4) {
                uint32_t* words = reinterpret_cast<uint32_t*>(smask);
                int kept = 0;
                for (int wj = lane; wj < d_in / 32; wj += 4) {
                    uint32_t m = words[wj];
                    int c = __popc(m);
                    if (kept + c > warp_cap) {
                        int keep = warp_cap - kept;
                        uint32_t out = 0;
                        for (int b = 0; b < 32 && keep > 0; ++b)
                            if (m & (1u << b)) { out |= 1u << b; --keep; }
                        m = out;
                        c = __popc(m);
                    }
                    words[wj] = m;
                    kept += c;
                }
            }
            __syncthreads();
        }
    } else {
        __syncthreads();
    }

    // Per-group B fragments, masked group sums and outlier counts.
    uint4* bsm = reinterpret_cast<uint4*>(smem + L.bsm);
    float* xp = reinterpret_cast<float*>(smem + L.xp);
    int* goff = reinterpret_cast<int*>(smem + L.goff);
    for (int j = warp; j < G; j += kNW) {
        float ps = 0.f;
        int cnt = 0;
        if (lane < 16) {
            const int t = lane >> 2, wi = lane & 3;
            const int ch = 16 * j + 4 * t + wi;
            const uint4 v = sx4[ch];
            const uint32_t mb = kSplit ? smask[ch] : 0u;
            uint16_t h[8];
            h[0] = v.x & 0xFFFFu; h[1] = v.x >> 16; h[2] = v.y & 0xFFFFu; h[3] = v.y >> 16;
            h[4] = v.z & 0xFFFFu; h[5] = v.z >> 16; h[6] = v.w & 0xFFFFu; h[7] = v.w >> 16;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                if (mb & (1u << i)) h[i] = 0;
                ps += h2f_bits(h[i]);
            }
            // word wi of chunk t feeds k-steps 2wi (pairs (0,4),(1,5)) and 2wi+1 ((2,6),(3,7))
            bsm[(j * 4 + wi) * 4 + t] = make_uint4(pack_h2(h[0], h[4]), pack_h2(h[1], h[5]),
                                                   pack_h2(h[2], h[6]), pack_h2(h[3], h[7]));
            cnt = __popc(mb);
        }
        ps = warp_sum(ps);
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
        if (lane == 0) {
            xp[j] = ps;
            goff[j] = cnt;
        }
    }
    __syncthreads();
    if (!kSplit) return;

    // Exclusive scan of the per-group counts (one warp).
    if (warp == 0) {
        const int per = (G + 31) / 32;
        const int b = lane * per;
        int local = 0;
        for (int i = 0; i < per; ++i)
            if (b + i < G) local += goff[b + i];
        int incl = local;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int n = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += n;
        }
        int run = incl - local;
        for (int i = 0; i < per; ++i)
            if (b + i < G) {
                int c = goff[b + i];
                goff[b + i] = run;
                run += c;
            }
        if (lane == 31) goff[G] = incl;
    }
    __syncthreads();
    // Ascending outlier list per group.
    int* list = reinterpret_cast<int*>(smem + L.list);
    for (int j = warp; j < G; j += kNW) {
        const int c0 = kGroup * j + 4 * lane;
        const uint32_t bits = (smask[c0 >> 3] >> (c0 & 7)) & 0xFu;
        const int n = __popc(bits);
        int incl = n;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        int pos = goff[j] + incl - n;
#pragma unroll
        for (int i = 0; i < 4; ++i)
            if (bits & (1u << i)) list[pos++] = c0 + i;
    }
    __syncthreads();
}

// ---------------------------------------------------------------------------
// Fused batch-1 GEMV
// ---------------------------------------------------------------------------
struct GemvArgs {
    const uint8_t* packed;
    const uint16_t* scales;
    const uint16_t* zeros;
    const uint16_t* w16;     // row-major FP16 (split path without mirror)
    const uint16_t* w16_cm;  // column-major FP16 mirror
    const uint16_t* x;
    uint16_t* y;
    int d_out, d_in, n_rb, nrb_max;
    float k;
};

struct Stage {
    uint4 ag, ag8;      // packed words of rows g and g+8 (32 columns each)
    uint32_t sz0, sz8;  // (scale, zero) of rows g and g+8 (lanes t == 0)
    uint32_t ow0, ow1;  // FP16 outlier weights (row g | row g+8 << 16) for outliers t and t+4
    uint32_t xo;        // x of those two outliers (lo, hi)
};

template <bool kSplit, bool kCM>
__device__ __forceinline__ uint16_t load_w16(const GemvArgs& a, int row, int c) {
    if (kCM) return ldg_u16(a.w16_cm + static_cast<size_t>(c) * a.d_out + row);
    return ldg_u16(a.w16 + static_cast<size_t>(row) * a.d_in + c);
}

template <bool kSplit, bool kCM>
__global__ void __launch_bounds__(kNT, 1) gemv_m1_kernel(const GemvArgs a) {
    extern __shared__ __align__(16) char smem[];
    const SmemLayout L = smem_layout(a.d_in, a.nrb_max, kNW, kSplit);
    const int G = a.d_in / kGroup;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;

    const int rb0 = static_cast<int>(static_cast<long long>(blockIdx.x) * a.n_rb / gridDim.x);
    const int rb1 = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * a.n_rb / gridDim.x);
    const int nrb = rb1 - rb0;
    const int U = nrb * G;
    const int u0 = static_cast<int>(static_cast<long long>(warp) * U / kNW);
    const int u1 = static_cast<int>(static_cast<long long>(warp + 1) * U / kNW);
    const size_t row_bytes = static_cast<size_t>(a.d_in) / 2;

    float* part = reinterpret_cast<float*>(smem + L.part);
    for (int i = tid; i < nrb * kNW * 16; i += kNT) part[i] = 0.f;

    const int* goff = reinterpret_cast<const int*>(smem + L.goff);
    const int* list = reinterpret_cast<const int*>(smem + L.list);
    const uint16_t* sxh = reinterpret_cast<const uint16_t*>(smem + L.sx);
    const uint4* bsm = reinterpret_cast<const uint4*>(smem + L.bsm);
    const float* xp = reinterpret_cast<const float*>(smem + L.xp);

    auto prefetch_a = [&](Stage& s, int rbl, int j) {
        const int r0 = (rb0 + rbl) * kRowBlock + g, r8 = r0 + 8;
        const uint8_t* base = a.packed + 64 * j + 16 * t;
        s.ag = r0 < a.d_out ? ldg_stream_v4(base + r0 * row_bytes) : make_uint4(0, 0, 0, 0);
        s.ag8 = r8 < a.d_out ? ldg_stream_v4(base + r8 * row_bytes) : make_uint4(0, 0, 0, 0);
        s.sz0 = 0;
        s.sz8 = 0;
        if (t == 0) {
            if (r0 < a.d_out)
                s.sz0 = pack_h2(ldg_u16(a.scales + static_cast<size_t>(r0) * G + j),
                                ldg_u16(a.zeros + static_cast<size_t>(r0) * G + j));
            if (r8 < a.d_out)
                s.sz8 = pack_h2(ldg_u16(a.scales + static_cast<size_t>(r8) * G + j),
                                ldg_u16(a.zeros + static_cast<size_t>(r8) * G + j));
        }
    };
    auto prefetch_o = [&](Stage& s, int rbl, int j) {
        s.ow0 = 0;
        s.ow1 = 0;
        s.xo = 0;
        if (!kSplit) return;
        const int r0 = (rb0 + rbl) * kRowBlock + g, r8 = r0 + 8;
        const int o0 = goff[j], nj = goff[j + 1] - o0;
        if (t < nj) {
            const int c = list[o0 + t];
            uint16_t w0 = r0 < a.d_out ? load_w16<kSplit, kCM>(a, r0, c) : 0;
            uint16_t w8 = r8 < a.d_out ? load_w16<kSplit, kCM>(a, r8, c) : 0;
            s.ow0 = pack_h2(w0, w8);
            s.xo = sxh[c];
        }
        if (t + 4 < nj) {
            const int c = list[o0 + t + 4];
            uint16_t w0 = r0 < a.d_out ? load_w16<kSplit, kCM>(a, r0, c) : 0;
            uint16_t w8 = r8 < a.d_out ? load_w16<kSplit, kCM>(a, r8, c) : 0;
            s.ow1 = pack_h2(w0, w8);
            s.xo |= static_cast<uint32_t>(sxh[c]) << 16;
        }
    };

    Stage ring[kDepth];
    // Issue the first weight loads before the prologue so they overlap it.
    int p_rb = (U > 0) ? u0 / G : 0, p_j = (U > 0) ? u0 % G : 0;
#pragma unroll
    for (int s = 0; s < kDepth; ++s) {
        if (u0 + s < u1) prefetch_a(ring[s], p_rb, p_j);
        if (++p_j == G) { p_j = 0; ++p_rb; }
    }

    activation_prologue<kSplit>(a.x, a.d_in, a.k, smem, L);

    {
        int q_rb = (U > 0) ? u0 / G : 0, q_j = (U > 0) ? u0 % G : 0;
#pragma unroll
        for (int s = 0; s < kDepth; ++s) {
            if (u0 + s < u1) prefetch_o(ring[s], q_rb, q_j);
            if (++q_j == G) { q_j = 0; ++q_rb; }
        }
    }

    float acc0 = 0.f, acc8 = 0.f, cor0 = 0.f, cor8 = 0.f;
    int c_rb = (U > 0) ? u0 / G : 0, c_j = (U > 0) ? u0 % G : 0;
    for (int ub = u0; ub < u1; ub += kDepth) {
#pragma unroll
        for (int s = 0; s < kDepth; ++s) {
            const int u = ub + s;
            if (u < u1) {
                Stage& st = ring[s];
                const int j = c_j;
                uint4 bq[4];
#pragma unroll
                for (int wi = 0; wi < 4; ++wi)
                    bq[wi] = (g == 0) ? bsm[(j * 4 + wi) * 4 + t] : make_uint4(0, 0, 0, 0);
                float d[4] = {0.f, 0.f, 0.f, 0.f};
                const uint32_t wa[4] = {st.ag.x, st.ag.y, st.ag.z, st.ag.w};
                const uint32_t wb[4] = {st.ag8.x, st.ag8.y, st.ag8.z, st.ag8.w};
#pragma unroll
                for (int wi = 0; wi < 4; ++wi) {
                    const Deq4 qa = dequant_word(wa[wi]);
                    const Deq4 qb = dequant_word(wb[wi]);
                    mma_16816(d, qa.p04, qb.p04, qa.p15, qb.p15, bq[wi].x, bq[wi].y);
                    mma_16816(d, qa.p26, qb.p26, qa.p37, qb.p37, bq[wi].z, bq[wi].w);
                }
                if (t == 0) {
                    const float xs = xp[j];
                    const float s0 = h2f_bits(st.sz0 & 0xFFFFu), z0 = h2f_bits(st.sz0 >> 16);
                    const float s8 = h2f_bits(st.sz8 & 0xFFFFu), z8 = h2f_bits(st.sz8 >> 16);
                    acc0 = fmaf(s0, fmaf(-z0, xs, d[0]), acc0);
                    acc8 = fmaf(s8, fmaf(-z8, xs, d[2]), acc8);
                }
                if (kSplit) {
                    const int o0 = goff[j], nj = goff[j + 1] - o0;
                    if (t < nj) {
                        const float xv = h2f_bits(st.xo & 0xFFFFu);
                        cor0 = fmaf(h2f_bits(st.ow0 & 0xFFFFu), xv, cor0);
                        cor8 = fmaf(h2f_bits(st.ow0 >> 16), xv, cor8);
                    }
                    if (t + 4 < nj) {
                        const float xv = h2f_bits(st.xo >> 16);
                        cor0 = fmaf(h2f_bits(st.ow1 & 0xFFFFu), xv, cor0);
                        cor8 = fmaf(h2f_bits(st.ow1 >> 16), xv, cor8);
                    }
                    if (nj > 8) {  // groups with more than 8 outliers: the rest unprefetched
                        const int r0 = (rb0 + c_rb) * kRowBlock + g, r8 = r0 + 8;
                        for (int i = 8 + t; i < nj; i += 4) {
                            const int c = list[o0 + i];
                            const float xv = h2f_bits(sxh[c]);
                            if (r0 < a.d_out) cor0 = fmaf(h2f_bits(load_w16<kSplit, kCM>(a, r0, c)), xv, cor0);
                            if (r8 < a.d_out) cor8 = fmaf(h2f_bits(load_w16<kSplit, kCM>(a, r8, c)), xv, cor8);
                        }
                    }
                }
                // End of this warp's segment of the row-block: publish its partial sums.
                if (c_j == G - 1 || u == u1 - 1) {
                    if (kSplit) {
                        cor0 += __shfl_xor_sync(0xffffffffu, cor0, 1);
                        cor0 += __shfl_xor_sync(0xffffffffu, cor0, 2);
                        cor8 += __shfl_xor_sync(0xffffffffu, cor8, 1);
                        cor8 += __shfl_xor_sync(0xffffffffu, cor8, 2);
                    }
                    if (t == 0) {
                        float* pp = part + (c_rb * kNW + warp) * 16;
                        pp[g] = acc0 + cor0;
                        pp[g + 8] = acc8 + cor8;
                    }
                    acc0 = acc8 = cor0 = cor8 = 0.f;
                }
                if (++c_j == G) { c_j = 0; ++c_rb; }
                // Refill this slot with the unit kDepth ahead.
                if (u + kDepth < u1) {
                    prefetch_a(st, p_rb, p_j);
                    prefetch_o(st, p_rb, p_j);
                }
                if (++p_j == G) { p_j = 0; ++p_rb; }
            }
        }
    }
    __syncthreads();
    for (int r = tid; r < nrb * 16; r += kNT) {
        const int rbl = r >> 4, rr = r & 15;
        const int row = (rb0 + rbl) * kRowBlock + rr;
        if (row < a.d_out) {
            float s = 0.f;
#pragma unroll
            for (int w = 0; w < kNW; ++w) s += part[(rbl * kNW + w) * 16 + rr];
            a.y[row] = __half_as_ushort(__float2half_rn(s));
        }
    }
}

// ---------------------------------------------------------------------------
// Dense FP16 GEMV (the reference's correctness oracle, also an API call)
// ---------------------------------------------------------------------------
struct RefArgs {
    const uint16_t* w16;
    const uint16_t* x;
    uint16_t* y;
    int d_out, d_in, n_rb, nrb_max;
};

constexpr int kRefDepth = 2;

__global__ void __launch_bounds__(kNT, 1) reference_gemv_kernel(const RefArgs a) {
    extern __shared__ __align__(16) char smem[];
    const int G = a.d_in / kGroup;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int rb0 = static_cast<int>(static_cast<long long>(blockIdx.x) * a.n_rb / gridDim.x);
    const int rb1 = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * a.n_rb / gridDim.x);
    const int nrb = rb1 - rb0;
    const int U = nrb * G;
    const int u0 = static_cast<int>(static_cast<long long>(warp) * U / kNW);
    const int u1 = static_cast<int>(static_cast<long long>(warp + 1) * U / kNW);

    uint4* bsm = reinterpret_cast<uint4*>(smem);                       // [G][4][4] uint4
    float* part = reinterpret_cast<float*>(smem + G * 256);            // [nrb][NW][16]

    struct RStage { uint4 r0[4], r8[4]; };
    auto prefetch = [&](RStage& s, int rbl, int j) {
        const int r0 = (rb0 + rbl) * kRowBlock + g, r8 = r0 + 8;
        const uint16_t* b = a.w16 + kGroup * j + 32 * t;
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
            s.r0[wi] = r0 < a.d_out ? ldg_stream_v4(b + static_cast<size_t>(r0) * a.d_in + 8 * wi)
                                    : make_uint4(0, 0, 0, 0);
            s.r8[wi] = r8 < a.d_out ? ldg_stream_v4(b + static_cast<size_t>(r8) * a.d_in + 8 * wi)
                                    : make_uint4(0, 0, 0, 0);
        }
    };

    RStage ring[kRefDepth];
    int p_rb = (U > 0) ? u0 / G : 0, p_j = (U > 0) ? u0 % G : 0;
#pragma unroll
    for (int s = 0; s < kRefDepth; ++s) {
        if (u0 + s < u1) prefetch(ring[s], p_rb, p_j);
        if (++p_j == G) { p_j = 0; ++p_rb; }
    }
    // x in fragment order: chunk ch = 16j + 4t + wi -> bsm[(j*4 + wi)*4 + t]
    for (int ch = tid; ch < a.d_in / 8; ch += kNT) {
        const int j = ch >> 4, t_ = (ch >> 2) & 3, wi = ch & 3;
        bsm[(j * 4 + wi) * 4 + t_] = ldg_v4(a.x + 8 * static_cast<size_t>(ch));
    }
    for (int i = tid; i < nrb * kNW * 16; i += kNT) part[i] = 0.f;
    __syncthreads();

    float d[4] = {0.f, 0.f, 0.f, 0.f};
    int c_rb = (U > 0) ? u0 / G : 0, c_j = (U > 0) ? u0 % G : 0;
    for (int ub = u0; ub < u1; ub += kRefDepth) {
#pragma unroll
        for (int s = 0; s < kRefDepth; ++s) {
            const int u = ub + s;
            if (u < u1) {
                RStage& st = ring[s];
#pragma unroll
                for (int wi = 0; wi < 4; ++wi) {
                    const uint4 bq = (g == 0) ? bsm[(c_j * 4 + wi) * 4 + t] : make_uint4(0, 0, 0, 0);
                    mma_16816(d, st.r0[wi].x, st.r8[wi].x, st.r0[wi].y, st.r8[wi].y, bq.x, bq.y);
                    mma_16816(d, st.r0[wi].z, st.r8[wi].z, st.r0[wi].w, st.r8[wi].w, bq.z, bq.w);
                }
                if (c_j == G - 1 || u == u1 - 1) {
                    if (t == 0) {
                        float* pp = part + (c_rb * kNW + warp) * 16;
                        pp[g] = d[0];
                        pp[g + 8] = d[2];
                    }
                    d[0] = d[1] = d[2] = d[3] = 0.f;
                }
                if (++c_j == G) { c_j = 0; ++c_rb; }
                if (u + kRefDepth < u1) prefetch(st, p_rb, p_j);
                if (++p_j == G) { p_j = 0; ++p_rb; }
            }
        }
    }
    __syncthreads();
    for (int r = tid; r < nrb * 16; r += kNT) {
        const int rbl = r >> 4, rr = r & 15;
        const int row = (rb0 + rbl) * kRowBlock + rr;
        if (row < a.d_out) {
            float s = 0.f;
#pragma unroll
            for (int w = 0; w < kNW; ++w) s += part[(rbl * kNW + w) * 16 + rr];
            a.y[row] = __half_as_ushort(__float2half_rn(s));
        }
    }
}

// ---------------------------------------------------------------------------
// Standalone detector: the GEMV prologue, exported.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kNT, 1) detect_kernel(const uint16_t* x, int d_in, float k,
                                                        uint32_t* mask_words, int32_t* indices,
                                                        int32_t* count, float* stats) {
    extern __shared__ __align__(16) char smem[];
    const SmemLayout L = smem_layout(d_in, 1, kNW, true);
    activation_prologue<true>(x, d_in, k, smem, L);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = d_in / kGroup;
    const uint32_t* words = reinterpret_cast<const uint32_t*>(smem + L.mask);
    const int* goff = reinterpret_cast<const int*>(smem + L.goff);
    const int* list = reinterpret_cast<const int*>(smem + L.list);
    const float* stat = reinterpret_cast<const float*>(smem + L.misc) + 32;
    if (mask_words)
        for (int i = tid; i < d_in / 32; i += kNT) mask_words[i] = words[i];
    const int total = goff[G];
    if (tid == 0) {
        if (count) *count = total;
        if (stats)
            for (int i = 0; i < 4; ++i) stats[i] = stat[i];
    }
    if (indices && warp < 4) {
        // The reference's list order: stripe class 0 ascending, then 1, 2, 3.
        // Count the classes before this one, then ballot-compact this class.
        int before = 0;
        for (int i = lane; i < total; i += 32) before += (((list[i] >> 5) & 3) < warp) ? 1 : 0;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) before += __shfl_xor_sync(0xffffffffu, before, o);
        int pos = before;
        for (int base = 0; base < total; base += 32) {
            const int i = base + lane;
            const bool mine = i < total && ((list[i] >> 5) & 3) == warp;
            const unsigned bal = __ballot_sync(0xffffffffu, mine);
            if (mine) indices[pos + __popc(bal & ((1u << lane) - 1u))] = list[i];
            pos += __popc(bal);
        }
    }
}

// ---------------------------------------------------------------------------
// Bit-exact quantizer (src/quant_format.cuh:48-53, 58-97), one thread per
// (row, group), scanning the group in column order exactly as the host loop
// does so that ties (+0/-0) and NaNs resolve identically.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int trunc_to_int_x86(float t) {
    // (int)t as the reference's x86-64 host build computes it: out-of-range and NaN give INT_MIN
    if (!(t >= -2147483648.0f && t < 2147483648.0f)) return INT_MIN;
    return __float2int_rz(t);
}

__device__ __forceinline__ uint32_t quant_code(uint16_t h, float gmin, float inv) {
    const float v = h2f_bits(h);
    const float s = __fadd_rn(__fmul_rn(__fsub_rn(v, gmin), inv), 0.5f);
    int c = trunc_to_int_x86(s);
    c = c < 0 ? 0 : (c > 15 ? 15 : c);
    return static_cast<uint32_t>(c);
}

__global__ void quantize_kernel(const uint16_t* __restrict__ w, int d_out, int d_in,
                                uint8_t* __restrict__ packed, uint16_t* __restrict__ scales,
                                uint16_t* __restrict__ zeros) {
    const int G = d_in / kGroup;
    const long long gid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (gid >= static_cast<long long>(d_out) * G) return;
    const int row = static_cast<int>(gid / G), grp = static_cast<int>(gid % G);
    const uint4* src = reinterpret_cast<const uint4*>(w + static_cast<size_t>(row) * d_in + kGroup * grp);
    float gmin = FLT_MAX, gmax = -FLT_MAX;
    for (int i = 0; i < 16; ++i) {
        const uint4 v = ldg_v4(src + i);
        const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float f = h2f_bits(static_cast<uint16_t>(wv[q >> 1] >> (16 * (q & 1))));
            if (f < gmin) gmin = f;
            if (f > gmax) gmax = f;
        }
    }
    const float range = __fsub_rn(gmax, gmin);
    const float scale_f = (range < 1e-8f) ? 1.0f : __fdiv_rn(range, 15.0f);
    const float inv = __fdiv_rn(1.0f, scale_f);
    const float zero_f = __fmul_rn(-gmin, inv);
    scales[gid] = __half_as_ushort(__float2half_rn(scale_f));
    zeros[gid] = __half_as_ushort(__float2half_rn(zero_f));
    uint4* dst = reinterpret_cast<uint4*>(packed + static_cast<size_t>(row) * (d_in / 2) + 64 * grp);
    for (int i = 0; i < 4; ++i) {
        uint32_t outw[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint4 v = ldg_v4(src + 4 * i + k);
            const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
            uint32_t word = 0;
#pragma unroll
            for (int q = 0; q < 8; ++q)
                word |= quant_code(static_cast<uint16_t>(wv[q >> 1] >> (16 * (q & 1))), gmin, inv) << (4 * q);
            outw[k] = word;
        }
        dst[i] = make_uint4(outw[0], outw[1], outw[2], outw[3]);
    }
}

// Column-major mirror: cm[c][r] = w[r][c], 64x64 tiles through shared memory.
__global__ void colmajor_kernel(const uint16_t* __restrict__ w, int d_out, int d_in,
                                uint16_t* __restrict__ cm) {
    __shared__ uint16_t tile[64][66];
    const int c0 = blockIdx.x * 64, r0 = blockIdx.y * 64;
    for (int i = threadIdx.x; i < 64 * 8; i += blockDim.x) {
        const int rr = i >> 3, cc = (i & 7) * 8;
        const int r = r0 + rr;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < d_out) v = ldg_v4(w + static_cast<size_t>(r) * d_in + c0 + cc);
        const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 8; ++q) tile[rr][cc + q] = static_cast<uint16_t>(wv[q >> 1] >> (16 * (q & 1)));
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 64 * 64; i += blockDim.x) {
        const int cc = i >> 6, rr = i & 63;
        const int r = r0 + rr;
        if (r < d_out) cm[static_cast<size_t>(c0 + cc) * d_out + r] = tile[rr][cc];
    }
}

// Per-device, per-kernel "max dynamic shared memory" opt-in, done once.
constexpr int kMaxDevices = 64;
enum KernelId { kSplitRM, kSplitCM, kInt4, kRef, kDetect, kNumKernels };
int g_smem_set[kMaxDevices][kNumKernels];  // bytes already opted in (0 = none)

template <class K>
dq_status_t ensure_smem(K kernel, KernelId id, int bytes) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
    if (dev >= 0 && dev < kMaxDevices && __atomic_load_n(&g_smem_set[dev][id], __ATOMIC_ACQUIRE) >= bytes)
        return DQ_OK;
    int want = bytes < 48 * 1024 ? 48 * 1024 : bytes;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, want);
    if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
    if (dev >= 0 && dev < kMaxDevices) {
        int cur = __atomic_load_n(&g_smem_set[dev][id], __ATOMIC_ACQUIRE);
        while (cur < want && !__atomic_compare_exchange_n(&g_smem_set[dev][id], &cur, want, false,
                                                          __ATOMIC_ACQ_REL, __ATOMIC_ACQUIRE)) {
        }
    }
    return DQ_OK;
}

dq_status_t check_launch() {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
    return DQ_OK;
}

}  // namespace

dq_status_t launch_gemv_m1(const dq_weights_t& w, const uint16_t* x, uint16_t* y, float k,
                           bool split, cudaStream_t stream) {
    DeviceInfo di;
    dq_status_t st = device_info(&di);
    if (st != DQ_OK) return st;
    GemvArgs a;
    a.packed = w.packed;
    a.scales = w.scales;
    a.zeros = w.zeros;
    a.w16 = w.fp16;
    a.w16_cm = w.fp16_cm;
    a.x = x;
    a.y = y;
    a.d_out = w.d_out;
    a.d_in = w.d_in;
    a.k = k;
    a.n_rb = (w.d_out + kRowBlock - 1) / kRowBlock;
    const int grid = a.n_rb < di.sm_count ? a.n_rb : di.sm_count;
    a.nrb_max = (a.n_rb + grid - 1) / grid;
    const SmemLayout L = smem_layout(a.d_in, a.nrb_max, kNW, split);
    if (L.total > di.smem_optin) return DQ_ERR_UNSUPPORTED;
    if (split && w.fp16_cm) {
        if ((st = ensure_smem(gemv_m1_kernel<true, true>, kSplitCM, L.total)) != DQ_OK) return st;
        gemv_m1_kernel<true, true><<<grid, kNT, L.total, stream>>>(a);
    } else if (split) {
        if ((st = ensure_smem(gemv_m1_kernel<true, false>, kSplitRM, L.total)) != DQ_OK) return st;
        gemv_m1_kernel<true, false><<<grid, kNT, L.total, stream>>>(a);
    } else {
        if ((st = ensure_smem(gemv_m1_kernel<false, false>, kInt4, L.total)) != DQ_OK) return st;
        gemv_m1_kernel<false, false><<<grid, kNT, L.total, stream>>>(a);
    }
    return check_launch();
}

dq_status_t launch_reference_gemv(const uint16_t* w16, const uint16_t* x, uint16_t* y, int d_out,
                                  int d_in, cudaStream_t stream) {
    DeviceInfo di;
    dq_status_t st = device_info(&di);
    if (st != DQ_OK) return st;
    RefArgs a;
    a.w16 = w16;
    a.x = x;
    a.y = y;
    a.d_out = d_out;
    a.d_in = d_in;
    a.n_rb = (d_out + kRowBlock - 1) / kRowBlock;
    const int grid = a.n_rb < di.sm_count ? a.n_rb : di.sm_count;
    a.nrb_max = (a.n_rb + grid - 1) / grid;
    const int smem = (d_in / kGroup) * 256 + a.nrb_max * kNW * 16 * 4;
    if (smem > di.smem_optin) return DQ_ERR_UNSUPPORTED;
    if ((st = ensure_smem(reference_gemv_kernel, kRef, smem)) != DQ_OK) return st;
    reference_gemv_kernel<<<grid, kNT, smem, stream>>>(a);
    return check_launch();
}

dq_status_t launch_detect(const uint16_t* x, int d_in, float k, uint32_t* mask_words,
                          int32_t* indices, int32_t* count, float* stats, cudaStream_t stream) {
    DeviceInfo di;
    dq_status_t st = device_info(&di);
    if (st != DQ_OK) return st;
    const SmemLayout L = smem_layout(d_in, 1, kNW, true);
    if (L.total > di.smem_optin) return DQ_ERR_UNSUPPORTED;
    if ((st = ensure_smem(detect_kernel, kDetect, L.total)) != DQ_OK) return st;
    detect_kernel<<<1, kNT, L.total, stream>>>(x, d_in, k, mask_words, indices, count, stats);
    return check_launch();
}

dq_status_t launch_quantize(const uint16_t* w16, int d_out, int d_in, uint8_t* packed,
                            uint16_t* scales, uint16_t* zeros, cudaStream_t stream) {
    const long long n = static_cast<long long>(d_out) * (d_in / kGroup);
    if (n == 0) return DQ_OK;
    const int threads = 128;
    const long long blocks = (n + threads - 1) / threads;
    quantize_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(w16, d_out, d_in, packed,
                                                                            scales, zeros);
    return check_launch();
}

dq_status_t launch_colmajor(const uint16_t* w16, int d_out, int d_in, uint16_t* cm,
                            cudaStream_t stream) {
    if (d_out == 0) return DQ_OK;
    dim3 grid(d_in / 64, (d_out + 63) / 64);
    colmajor_kernel<<<grid, 256, 0, stream>>>(w16, d_out, d_in, cm);
    return check_launch();
}

}  // namespace dq
