// dq_gemv.cu -- batch-1 GEMV kernels for sm_100a: fused split (INT4 + FP16
// outlier columns), dense INT4, dense FP16, the activation plan / standalone
// detector, the bit-exact quantizer and the layout builders.
//
// Reference path (dyn-quant): src/split_gemv.cu:25-198, src/int4_gemv.cu:12-100,
// src/reference_gemv.cu:9-78, src/outlier_detect.cuh:104-205,
// src/quant_format.cuh:48-97.
//
// One split GEMV call = two kernels on the stream:
//   1. plan_kernel (one 1024-thread CTA): statistics of x, the outlier mask
//      (with the reference's capacity rule), the outlier list, the MMA B
//      fragments of the masked activation and per-group sums -- computed once
//      into the workspace.  It triggers the dependent launch at its start.
//   2. gemv_kernel (persistent, one 256-thread CTA per SM, launched as a
//      programmatic dependent of the plan): each warp starts streaming its
//      weight units through a 3-stage shared-memory ring (cp.async.bulk, the
//      non-tensor TMA form, completing on per-stage mbarriers) BEFORE it waits
//      for the plan (griddepcontrol.wait); then one bulk copy brings the plan
//      into shared memory and the warps run the dequant + tensor-core loop.
//   * A unit is 16 rows x 4 groups of 128 columns (4 KB of packed INT4).  The
//     units are split evenly across CTAs (and across the 8 warps of a CTA) in
//     (row-block, column-chunk) order; a 16-row block that straddles two CTAs
//     is finished by whichever of them arrives last, summing the partial row
//     sums in CTA order (fixed order: results are bit-reproducible).
//   * The contraction runs on the tensor cores: mma.sync.m16n8k16 with the
//     packed codes as A (f16 1024+q or 1024+16q, exact) and the masked
//     activation x' as column 0 of B, FP32 accumulate; the exponent bias is
//     removed per group in FP32 from the plan's per-group sums.  Per
//     (row, group): y += s * (sum_c q_c x'_c - z * sum_c x'_c), the value of
//     the reference's sum of s*(q-z)*x over the non-outlier channels.
//   * Outlier channels add W16[r][c] * x[c]: with the column-major mirror the
//     16 rows of one outlier column (32 bytes) are fetched by cp.async into the
//     unit's stage and complete on the same mbarrier as the weights.
#include <cfloat>
#include <climits>

#include "dq_common.cuh"
#include "dq_internal.h"

namespace dq {

namespace {

constexpr int kW = kB1Warps;
constexpr int kT = kB1Threads;
constexpr int kStages = kB1Stages;
constexpr int kCG = kB1ChunkGroups;
constexpr int kStageBytes = kB1StageBytes;

// Set (bit 0) by a kernel whose bounded wait on its own copies gave up.
__device__ unsigned int g_error_word;

// ---------------------------------------------------------------------------
// Activation plan
// ---------------------------------------------------------------------------

// Computes the plan of x into shared memory laid out by plan_layout, with NT
// threads.  The outlier mask follows the reference's detector definition
// (src/outlier_detect.cuh): mean and unbiased variance of x (two-pass, FP32,
// fixed reduction order), thresh = k * sqrt(max(var, 1e-8)), outlier iff
// |x - mean| > thresh, and at most (d_in/4)/4 outliers kept per stripe class
// (columns c with (c/32) % 4 == w, the first ones in ascending order), as the
// reference's per-warp capacity does (src/outlier_detect.cuh:160-178).
// red: >= 64 floats of scratch.
template <int NT, bool kSplit>
__device__ void build_plan(const uint16_t* __restrict__ x, int d_in, float k, char* smem, float* red) {
    constexpr int NW = NT / 32;
    const PlanLayout P = plan_layout(d_in);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = d_in / kGroup;
    const int n8 = d_in >> 3;
    uint4* xb = reinterpret_cast<uint4*>(smem + P.bsm);  // natural order, then B fragments
    uint8_t* smask = reinterpret_cast<uint8_t*>(smem + P.mask);
    float* stat = reinterpret_cast<float*>(smem + P.stats);
    int* stripe = reinterpret_cast<int*>(red + 40);
    float4* xp4 = reinterpret_cast<float4*>(smem + P.xp);
    int* goff = reinterpret_cast<int*>(smem + P.goff);
    uint32_t* list = reinterpret_cast<uint32_t*>(smem + P.list);

    if (tid < 4) stripe[tid] = 0;
    float sum = 0.f;
    for (int ch = tid; ch < n8; ch += NT) {
        const uint4 v = ldg_v4(x + 8 * static_cast<size_t>(ch));
        xb[ch] = v;
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
        const float total = block_sum<NT>(sum, red);
        const float mean = __fdiv_rn(total, static_cast<float>(d_in));
        float m2 = 0.f;
        for (int ch = tid; ch < n8; ch += NT) {
            const uint4 v = xb[ch];
            const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float d0 = __fsub_rn(h2f_bits(static_cast<uint16_t>(wv[i] & 0xFFFFu)), mean);
                const float d1 = __fsub_rn(h2f_bits(static_cast<uint16_t>(wv[i] >> 16)), mean);
                m2 = __fmaf_rn(d0, d0, m2);
                m2 = __fmaf_rn(d1, d1, m2);
            }
        }
        const float M2 = block_sum<NT>(m2, red);
        const float var = (d_in > 1) ? __fdiv_rn(M2, static_cast<float>(d_in - 1)) : 0.f;
        const float thresh = __fmul_rn(k, __fsqrt_rn(fmaxf(var, 1e-8f)));
        if (tid == 0) {
            stat[0] = mean;
            stat[1] = thresh;
            stat[2] = var;
            stat[3] = M2;
        }
        for (int ch = tid; ch < n8; ch += NT) {
            const uint4 v = xb[ch];
            const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
            uint32_t byte = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float a = h2f_bits(static_cast<uint16_t>(wv[i] & 0xFFFFu));
                const float b = h2f_bits(static_cast<uint16_t>(wv[i] >> 16));
                byte |= (fabsf(__fsub_rn(a, mean)) > thresh ? 1u : 0u) << (2 * i);
                byte |= (fabsf(__fsub_rn(b, mean)) > thresh ? 1u : 0u) << (2 * i + 1);
            }
            smask[ch] = static_cast<uint8_t>(byte);
            if (byte) atomicAdd(&stripe[(ch >> 2) & 3], __popc(byte));
        }
        __syncthreads();
        // Capacity rule (rare): keep the first warp_cap outliers of each stripe class.
        const int warp_cap = (d_in / 4) / 4;
        if (stripe[0] > warp_cap || stripe[1] > warp_cap || stripe[2] > warp_cap || stripe[3] > warp_cap) {
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
        // Per-group outlier counts (4 mask words per group).
        const uint32_t* words = reinterpret_cast<const uint32_t*>(smask);
        for (int j = warp; j < G; j += NW) {
            int c = (lane < 4) ? __popc(words[4 * j + lane]) : 0;
            c += __shfl_xor_sync(0xffffffffu, c, 1);
            c += __shfl_xor_sync(0xffffffffu, c, 2);
            if (lane == 0) goff[j] = c;
        }
        __syncthreads();
        // Exclusive scan of the counts (one warp).
        if (warp == 0) {
            const int per = (G + 31) / 32;
            const int b = lane * per;
            int local = 0;
            for (int i = 0; i < per; ++i)
                if (b + i < G) local += goff[b + i];
            int incl = local;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int n = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += n;
            }
            int run = incl - local;
            for (int i = 0; i < per; ++i)
                if (b + i < G) {
                    const int c = goff[b + i];
                    goff[b + i] = run;
                    run += c;
                }
            if (lane == 31) {
                goff[G] = incl;
                reinterpret_cast<int*>(stat)[4] = incl;
            }
        }
        __syncthreads();
        // Ascending outlier list per group, with the activation value of each.
        const uint16_t* xh = reinterpret_cast<const uint16_t*>(xb);
        for (int j = warp; j < G; j += NW) {
            const int c0 = kGroup * j + 4 * lane;
            const uint32_t bits = (smask[c0 >> 3] >> (c0 & 7)) & 0xFu;
            const int n = __popc(bits);
            int incl = n;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            int pos = goff[j] + incl - n;
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (bits & (1u << i))
                    list[pos++] = static_cast<uint32_t>(c0 + i) | (static_cast<uint32_t>(xh[c0 + i]) << 16);
        }
    } else {
        for (int j = tid; j <= G; j += NT) goff[j] = 0;
        if (tid == 0) reinterpret_cast<int*>(stat)[4] = 0;
    }
    __syncthreads();

    // In place: natural chunk (j, t, wi) -> fragment slot (j, wi, t), outliers
    // zeroed.  Word wi of chunk t feeds two MMAs: the "low" one takes columns
    // (0,4) and (2,6) of the word, the "high" one (1,5) and (3,7) -- the
    // pairs the dequantisation extracts without a shift.  Per group, xp holds
    // (1024 * sum x' over even columns, 1024 * sum over odd columns, sum x', 0).
    for (int j = warp; j < G; j += NW) {
        uint4 out = make_uint4(0, 0, 0, 0);
        float pe = 0.f, po = 0.f;
        const int t = lane >> 2, wi = lane & 3;
        if (lane < 16) {
            const int ch = 16 * j + 4 * t + wi;
            const uint4 v = xb[ch];
            const uint32_t mb = kSplit ? smask[ch] : 0u;
            uint16_t h[8];
            h[0] = v.x & 0xFFFFu; h[1] = v.x >> 16; h[2] = v.y & 0xFFFFu; h[3] = v.y >> 16;
            h[4] = v.z & 0xFFFFu; h[5] = v.z >> 16; h[6] = v.w & 0xFFFFu; h[7] = v.w >> 16;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (mb & (1u << i)) h[i] = 0;
            pe = (h2f_bits(h[0]) + h2f_bits(h[2])) + (h2f_bits(h[4]) + h2f_bits(h[6]));
            po = (h2f_bits(h[1]) + h2f_bits(h[3])) + (h2f_bits(h[5]) + h2f_bits(h[7]));
            out = make_uint4(pack_h2(h[0], h[4]), pack_h2(h[2], h[6]), pack_h2(h[1], h[5]), pack_h2(h[3], h[7]));
        }
        __syncwarp();
        if (lane < 16) xb[16 * j + 4 * wi + t] = out;
        pe = warp_sum(pe);
        po = warp_sum(po);
        if (lane == 0) xp4[j] = make_float4(1024.f * pe, 1024.f * po, pe + po, 0.f);
    }
    __syncthreads();
}

// One CTA builds the plan of x.  Writes it to `plan` (the workspace) when
// non-null, and the detector outputs when requested.  Lets the dependent GEMV
// launch immediately: the GEMV only reads the plan after griddepcontrol.wait.
template <bool kSplit>
__global__ void __launch_bounds__(kPlanThreads, 1)
    plan_kernel(const uint16_t* __restrict__ x, int d_in, float k, uint8_t* __restrict__ plan,
                uint32_t* mask_words, int32_t* indices, int32_t* count, float* stats) {
    pdl_launch_dependents();
    extern __shared__ __align__(128) char smem[];
    const PlanLayout P = plan_layout(d_in);
    float* red = reinterpret_cast<float*>(smem + P.total);
    build_plan<kPlanThreads, kSplit>(x, d_in, k, smem, red);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (plan) {
        const uint4* src = reinterpret_cast<const uint4*>(smem);
        uint4* dst = reinterpret_cast<uint4*>(plan);
        for (int i = tid; i < P.total / 16; i += kPlanThreads) dst[i] = src[i];
    }
    if (!kSplit) return;
    const int G = d_in / kGroup;
    const uint32_t* words = reinterpret_cast<const uint32_t*>(smem + P.mask);
    const int* goff = reinterpret_cast<const int*>(smem + P.goff);
    const uint32_t* list = reinterpret_cast<const uint32_t*>(smem + P.list);
    const float* stat = reinterpret_cast<const float*>(smem + P.stats);
    if (mask_words)
        for (int i = tid; i < d_in / 32; i += kPlanThreads) mask_words[i] = words[i];
    const int total = goff[G];
    if (tid == 0) {
        if (count) *count = total;
        if (stats)
            for (int i = 0; i < 4; ++i) stats[i] = stat[i];
    }
    if (indices && warp < 4) {
        // The reference's list order: stripe class 0 ascending, then 1, 2, 3.
        int before = 0;
        for (int i = lane; i < total; i += 32)
            before += ((static_cast<int>(list[i] & 0xFFFFu) >> 5) & 3) < warp ? 1 : 0;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) before += __shfl_xor_sync(0xffffffffu, before, o);
        int pos = before;
        for (int base = 0; base < total; base += 32) {
            const int i = base + lane;
            const int c = (i < total) ? static_cast<int>(list[i] & 0xFFFFu) : 0;
            const bool mine = i < total && ((c >> 5) & 3) == warp;
            const unsigned bal = __ballot_sync(0xffffffffu, mine);
            if (mine) indices[pos + __popc(bal & ((1u << lane) - 1u))] = c;
            pos += __popc(bal);
        }
    }
}

// ---------------------------------------------------------------------------
// Fused batch-1 GEMV
// ---------------------------------------------------------------------------
struct GemvArgs {
    const uint8_t* packed;    // reference layout [d_out][d_in/2]
    const uint16_t* scales;   // reference layout [d_out][G]
    const uint16_t* zeros;
    const uint8_t* native;    // unit layout (native_bytes), or null
    const uint16_t* w16;      // row-major FP16 (split path without mirror)
    const uint16_t* w16_cm;   // column-major FP16 mirror
    uint16_t* y;
    const uint8_t* plan;      // workspace: activation plan
    float* fix;               // workspace: partial row sums of shared row blocks
    unsigned int* cnt;        // workspace: arrival counters of shared row blocks
    int d_out, d_in, n_rb, NC, U, nrb_max;
};

template <bool kCM>
__device__ __forceinline__ uint32_t load_w16_pair(const GemvArgs& a, int r, int c) {
    // (W16[r][c], W16[r+1][c]) as an f16 pair; rows past d_out read as 0.
    if (kCM) {
        const uint16_t* p = a.w16_cm + static_cast<size_t>(c) * a.d_out + r;
        if (r + 1 < a.d_out) {
            if ((a.d_out & 1) == 0) {
                uint32_t v;
                asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
                return v;
            }
            return pack_h2(ldg_u16(p), ldg_u16(p + 1));
        }
        return (r < a.d_out) ? static_cast<uint32_t>(ldg_u16(p)) : 0u;
    }
    const uint16_t* p = a.w16 + static_cast<size_t>(r) * a.d_in + c;
    const uint16_t lo = (r < a.d_out) ? ldg_u16(p) : static_cast<uint16_t>(0);
    const uint16_t hi = (r + 1 < a.d_out) ? ldg_u16(p + a.d_in) : static_cast<uint16_t>(0);
    return pack_h2(lo, hi);
}

__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
    return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

__host__ __device__ inline int unit_start(long long U, int c, int P) {
    return static_cast<int>(U * c / P);
}
__host__ __device__ inline int unit_owner(long long u, int P, long long U) {
    return static_cast<int>((u * P + P - 1) / U);
}

// kNative: weights in the unit layout (one bulk copy per unit, scale/zero
// inside); otherwise the reference layout (one bulk copy per weight row of the
// unit, scale/zero by plain loads).  kStage: outlier columns staged by cp.async
// (column-major mirror with d_out % 8 == 0); otherwise loaded directly.
template <bool kSplit, bool kCM, bool kNative, bool kStage>
__global__ void __launch_bounds__(kT, 1) gemv_kernel(const GemvArgs a) {
    extern __shared__ __align__(128) char smem[];
    const GemvSmem S = gemv_smem(a.d_in, a.nrb_max);
    const int G = a.d_in / kGroup;
    const int NC = a.NC;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int p = lane & 7, q = lane >> 3;  // outlier lanes: rows 2p, 2p+1 of staged outlier q (+4i)
    const int P = gridDim.x, c = blockIdx.x;
    const long long U = a.U;

    const int cu0 = unit_start(U, c, P), cu1 = unit_start(U, c + 1, P);
    const int rbf = cu0 / NC;                 // first row block touched by this CTA
    const int rbz = (cu1 - 1) / NC;           // last
    const int nrb = rbz - rbf + 1;
    const int wu0 = cu0 + static_cast<int>(static_cast<long long>(cu1 - cu0) * warp / kW);
    const int wu1 = cu0 + static_cast<int>(static_cast<long long>(cu1 - cu0) * (warp + 1) / kW);
    const size_t row_stride = static_cast<size_t>(a.d_in) / 2;

    char* ring_p = smem + S.ring + warp * kStages * kStageBytes;
    const uint32_t ring = smem_u32(ring_p);
    const uint32_t bars = smem_u32(smem + S.bars) + warp * kStages * 8;
    const uint32_t planbar = smem_u32(smem + S.bars) + kW * kStages * 8;
    float* part = reinterpret_cast<float*>(smem + S.part);
    const PlanLayout PL = plan_layout(a.d_in);
    const char* plan_s = smem + S.plan;
    const uint4* bsm = reinterpret_cast<const uint4*>(plan_s + PL.bsm);
    const float4* xp4 = reinterpret_cast<const float4*>(plan_s + PL.xp);
    const int* goff = reinterpret_cast<const int*>(plan_s + PL.goff);
    const uint32_t* list = reinterpret_cast<const uint32_t*>(plan_s + PL.list);
    int* flags = reinterpret_cast<int*>(smem + S.misc);

    if (lane == 0) {
#pragma unroll
        for (int s = 0; s < kStages; ++s) mbar_init(bars + 8 * s, 1);
        if (warp == 0) mbar_init(planbar, 1);
        fence_mbar_init();
    }
    for (int i = tid; i < nrb * kW * 16; i += kT) part[i] = 0.f;
    __syncthreads();

    uint32_t szr0[kStages], szr8[kStages];  // reference-layout (scale, zero): lane t's group

    // Weight bytes of unit u into stage s (the stage's phase still needs the
    // arrival of lane 0, after the outlier copies are registered).
    auto issue_weights = [&](int s, int u) {
        const int rb = u / NC, cc = u % NC;
        const uint32_t bar = bars + 8 * s;
        if (kNative) {
            if (lane == 0) {
                mbar_expect_tx(bar, kB1UnitBytes);
                bulk_g2s(ring + s * kStageBytes, a.native + static_cast<size_t>(u) * kB1UnitBytes, kB1UnitBytes, bar);
            }
        } else {
            const int rbase = rb * kRowBlock;
            const int ng = min(kCG, G - kCG * cc);
            const int vrows = min(kRowBlock, a.d_out - rbase);
            const uint32_t rbytes = static_cast<uint32_t>(ng) * 64u;
            if (lane == 0) mbar_expect_tx(bar, vrows * rbytes);
            __syncwarp();
            if (lane < vrows)
                bulk_g2s(ring + s * kStageBytes + lane * kB1RowPitch,
                         a.packed + static_cast<size_t>(rbase + lane) * row_stride + 256 * static_cast<size_t>(cc),
                         rbytes, bar);
            const int j = kCG * cc + t;
            const int r0 = rbase + g, r8 = r0 + 8;
            szr0[s] = (j < G && r0 < a.d_out)
                          ? pack_h2(ldg_u16(a.scales + static_cast<size_t>(r0) * G + j),
                                    ldg_u16(a.zeros + static_cast<size_t>(r0) * G + j))
                          : 0u;
            szr8[s] = (j < G && r8 < a.d_out)
                          ? pack_h2(ldg_u16(a.scales + static_cast<size_t>(r8) * G + j),
                                    ldg_u16(a.zeros + static_cast<size_t>(r8) * G + j))
                          : 0u;
        }
    };

    // Outlier columns of unit u into stage s (first 16: two 16-byte halves per
    // column, one cp.async per lane), then lane 0's arrival closes the phase.
    auto issue_outliers_and_arrive = [&](int s, int u) {
        const uint32_t bar = bars + 8 * s;
        if (kSplit && kStage) {
            const int rb = u / NC, cc = u % NC;
            const int j0 = kCG * cc, j1 = min(G, j0 + kCG);
            const int ob = goff[j0], n = min(goff[j1] - ob, kB1OutlierSlots);
            const int slot = lane >> 1, half = lane & 1;
            const int r = rb * kRowBlock + 8 * half;
            if (slot < n && r < a.d_out) {
                const int col = static_cast<int>(list[ob + slot] & 0xFFFFu);
                cp_async16(ring + s * kStageBytes + kB1StageOutliers + slot * 32 + half * 16,
                           a.w16_cm + static_cast<size_t>(col) * a.d_out + r);
            }
            cp_async_mbar_arrive(bar);
            __syncwarp();
        }
        if (lane == 0) mbar_arrive(bar);
    };

    float acc0 = 0.f, acc8 = 0.f, cor0 = 0.f, cor1 = 0.f;

    auto consume = [&](int s, int u, bool flush) {
        const char* st = ring_p + s * kStageBytes;
        const int rb = u / NC, cc = u % NC;
        const int j0 = kCG * cc;
        const int ng = min(kCG, G - j0);
        // packed words of rows g and g+8 for the unit's groups
        uint4 aw[kCG][2];
#pragma unroll
        for (int jj = 0; jj < kCG; ++jj)
#pragma unroll
            for (int h = 0; h < 2; ++h)
                aw[jj][h] = kNative
                                ? *reinterpret_cast<const uint4*>(st + ((jj * 2 + h) * 32 + lane) * 16)
                                : *reinterpret_cast<const uint4*>(st + (g + 8 * h) * kB1RowPitch + 64 * jj + 16 * t);
        // Two independent accumulators per group (even / odd columns): 8 chains of 4 MMAs.
        float dl[kCG][4], dh[kCG][4];
#pragma unroll
        for (int jj = 0; jj < kCG; ++jj)
#pragma unroll
            for (int i = 0; i < 4; ++i) dl[jj][i] = dh[jj][i] = 0.f;
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
#pragma unroll
            for (int jj = 0; jj < kCG; ++jj) {
                if (jj < ng) {
                    const uint4 bq = (g == 0) ? bsm[((j0 + jj) * 4 + wi) * 4 + t] : make_uint4(0, 0, 0, 0);
                    const Biased4 qa = biased_word(word_of(aw[jj][0], wi));
                    const Biased4 qb = biased_word(word_of(aw[jj][1], wi));
                    mma_16816(dl[jj], qa.lo0, qb.lo0, qa.lo1, qb.lo1, bq.x, bq.y);
                    mma_16816(dh[jj], qa.hi0, qb.hi0, qa.hi1, qb.hi1, bq.z, bq.w);
                }
            }
        }
        uint32_t sz0[kCG], sz8[kCG];
        if (kNative) {
            const uint4 v0 = *reinterpret_cast<const uint4*>(st + kB1UnitPacked + 16 * g);
            const uint4 v8 = *reinterpret_cast<const uint4*>(st + kB1UnitPacked + 16 * (g + 8));
            sz0[0] = v0.x; sz0[1] = v0.y; sz0[2] = v0.z; sz0[3] = v0.w;
            sz8[0] = v8.x; sz8[1] = v8.y; sz8[2] = v8.z; sz8[3] = v8.w;
        } else {
#pragma unroll
            for (int jj = 0; jj < kCG; ++jj) {
                sz0[jj] = __shfl_sync(0xffffffffu, szr0[s], (lane & ~3) + jj);
                sz8[jj] = __shfl_sync(0xffffffffu, szr8[s], (lane & ~3) + jj);
            }
        }
        if (t == 0) {
            // D_lo = 1024*Xe + S_even, D_hi = 1024*Xo + 16*S_odd  ->  S = S_even + S_odd;
            // y += s * (S - z * X) over the non-outlier columns of the group.
#pragma unroll
            for (int jj = 0; jj < kCG; ++jj) {
                if (jj < ng) {
                    const float4 xq = xp4[j0 + jj];
                    const float s0 = h2f_bits(sz0[jj] & 0xFFFFu), z0 = h2f_bits(sz0[jj] >> 16);
                    const float s8 = h2f_bits(sz8[jj] & 0xFFFFu), z8 = h2f_bits(sz8[jj] >> 16);
                    const float S0 = fmaf(dh[jj][0] - xq.y, 0.0625f, dl[jj][0] - xq.x);
                    const float S8 = fmaf(dh[jj][2] - xq.y, 0.0625f, dl[jj][2] - xq.x);
                    acc0 = fmaf(s0, fmaf(-z0, xq.z, S0), acc0);
                    acc8 = fmaf(s8, fmaf(-z8, xq.z, S8), acc8);
                }
            }
        }
        if (kSplit) {
            const int ob = goff[j0], n = goff[j0 + ng] - ob;
            const int r = rb * kRowBlock + 2 * p;
            int first_direct = 0;
            if (kStage) {
                first_direct = kB1OutlierSlots;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int o = q + 4 * i;
                    if (o < n) {
                        const uint32_t w = *reinterpret_cast<const uint32_t*>(st + kB1StageOutliers + o * 32 + 4 * p);
                        const float xv = h2f_bits(static_cast<uint16_t>(list[ob + o] >> 16));
                        cor0 = fmaf(h2f_bits(w & 0xFFFFu), xv, cor0);
                        cor1 = fmaf(h2f_bits(w >> 16), xv, cor1);
                    }
                }
            }
            for (int o = first_direct + q; o < n; o += 4) {
                const uint32_t e = list[ob + o];
                const float xv = h2f_bits(static_cast<uint16_t>(e >> 16));
                const uint32_t w = load_w16_pair<kCM>(a, r, static_cast<int>(e & 0xFFFFu));
                cor0 = fmaf(h2f_bits(w & 0xFFFFu), xv, cor0);
                cor1 = fmaf(h2f_bits(w >> 16), xv, cor1);
            }
        }
        if (flush) {
            // End of this warp's part of the row block: publish its row sums.
            float* pp = part + ((rb - rbf) * kW + warp) * 16;
            if (t == 0) {
                pp[g] = acc0;
                pp[g + 8] = acc8;
            }
            if (kSplit) {
                cor0 += __shfl_xor_sync(0xffffffffu, cor0, 8);
                cor0 += __shfl_xor_sync(0xffffffffu, cor0, 16);
                cor1 += __shfl_xor_sync(0xffffffffu, cor1, 8);
                cor1 += __shfl_xor_sync(0xffffffffu, cor1, 16);
                __syncwarp();
                if (lane < 8) {
                    pp[2 * lane] += cor0;
                    pp[2 * lane + 1] += cor1;
                }
            }
            acc0 = acc8 = cor0 = cor1 = 0.f;
        }
    };

    // Weights of the first units go out before the plan is ready.
    uint32_t armed = 0;
#pragma unroll
    for (int s = 0; s < kStages; ++s)
        if (wu0 + s < wu1) {
            issue_weights(s, wu0 + s);
            armed |= 1u << s;
        }

    // Wait for the plan kernel (programmatic dependent launch), then bring the plan in.
    pdl_wait();
    if (tid == 0) {
        mbar_arrive_expect_tx(planbar, PL.copy_bytes);
        bulk_g2s(smem_u32(smem + S.plan), a.plan, PL.copy_bytes, planbar);
    }
    bool ok = mbar_wait_bounded(planbar, 0);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok && lane == 0) atomicOr(&g_error_word, 1u);

#pragma unroll
    for (int s = 0; s < kStages; ++s)
        if (wu0 + s < wu1) issue_outliers_and_arrive(s, wu0 + s);

    uint32_t phase = 0;
    for (int ub = wu0; ub < wu1 && ok; ub += kStages) {
#pragma unroll
        for (int s = 0; s < kStages; ++s) {
            const int u = ub + s;
            if (u < wu1 && ok) {
                const bool got = mbar_wait_bounded(bars + 8 * s, (phase >> s) & 1u);
                if (!__all_sync(0xffffffffu, got)) {
                    ok = false;
                    if (lane == 0) atomicOr(&g_error_word, 1u);
                } else {
                    phase ^= 1u << s;
                    armed &= ~(1u << s);
                    consume(s, u, (u % NC) == NC - 1 || u == wu1 - 1);
                    __syncwarp();
                    if (u + kStages < wu1) {
                        issue_weights(s, u + kStages);
                        armed |= 1u << s;
                        issue_outliers_and_arrive(s, u + kStages);
                    }
                }
            }
        }
    }
    if (!ok) {
        // Do not leave copies in flight into shared memory this CTA is about to release.
#pragma unroll
        for (int s = 0; s < kStages; ++s)
            if (armed & (1u << s)) mbar_wait_bounded(bars + 8 * s, (phase >> s) & 1u);
    }
    __syncthreads();

    // Row sums: row blocks owned by this CTA alone are written directly; a row
    // block shared with a neighbour goes through the workspace, and the CTA that
    // arrives last sums the contributions in CTA order.
    for (int r = tid; r < nrb * 16; r += kT) {
        const int rbl = r >> 4, rr = r & 15;
        const int rb = rbf + rbl;
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < kW; ++w) sum += part[(rbl * kW + w) * 16 + rr];
        const bool owned = rb * NC >= cu0 && (rb + 1) * NC <= cu1;
        if (owned) {
            const int row = rb * kRowBlock + rr;
            if (row < a.d_out) a.y[row] = __half_as_ushort(__float2half_rn(sum));
        } else {
            a.fix[(c * 2 + (rb == rbf ? 0 : 1)) * 16 + rr] = sum;
        }
    }
    __threadfence();
    __syncthreads();
    if (tid < 2) {
        const int rb = tid == 0 ? rbf : rbz;
        const bool shared = !(rb * NC >= cu0 && (rb + 1) * NC <= cu1) && (tid == 0 || rbz != rbf);
        int last = 0;
        if (shared) {
            const int c_first = unit_owner(static_cast<long long>(rb) * NC, P, U);
            const int c_last = unit_owner(static_cast<long long>(rb + 1) * NC - 1, P, U);
            const unsigned int ticket = atomicAdd(&a.cnt[rb], 1u);
            last = ticket == static_cast<unsigned int>(c_last - c_first) ? 1 : 0;
        }
        flags[tid] = last;
    }
    __syncthreads();
#pragma unroll
    for (int which = 0; which < 2; ++which) {
        if (flags[which]) {
            __threadfence();
            const int rb = which == 0 ? rbf : rbz;
            const int c_first = unit_owner(static_cast<long long>(rb) * NC, P, U);
            const int c_last = unit_owner(static_cast<long long>(rb + 1) * NC - 1, P, U);
            if (tid < 16) {
                float sum = 0.f;
                for (int cc = c_first; cc <= c_last; ++cc) {
                    const int slot = (rb == unit_start(U, cc, P) / NC) ? 0 : 1;
                    sum += ldcg_f32(a.fix + (cc * 2 + slot) * 16 + tid);
                }
                const int row = rb * kRowBlock + tid;
                if (row < a.d_out) a.y[row] = __half_as_ushort(__float2half_rn(sum));
            }
            if (tid == 0) a.cnt[rb] = 0;
        }
    }
}

// Native unit layout: per (row-block rb, 4-group chunk c) one block of
// kB1UnitBytes = 4096 bytes of packed codes ordered [group jj][half h][lane]
// (16 bytes each: row rb*16 + g + 8h, columns 128(4c+jj) + 32t .. +31, with
// lane = 4g + t) followed by 256 bytes of (scale | zero << 16) for
// [16 rows][4 groups].  Rows past d_out and groups past G are zero.
__global__ void build_native_kernel(const uint8_t* __restrict__ packed, const uint16_t* __restrict__ scales,
                                    const uint16_t* __restrict__ zeros, int d_out, int d_in,
                                    uint8_t* __restrict__ out, long long n_chunks) {
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= n_chunks) return;
    constexpr int kChunks = kB1UnitBytes / 16;  // 272 sixteen-byte chunks per unit
    const int G = d_in / kGroup;
    const int NC = (G + kCG - 1) / kCG;
    const long long unit = idx / kChunks;
    const int i = static_cast<int>(idx % kChunks);
    const int rb = static_cast<int>(unit / NC), c = static_cast<int>(unit % NC);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (i < kB1UnitPacked / 16) {
        const int jj = i >> 6, h = (i >> 5) & 1, ln = i & 31;
        const int row = rb * kRowBlock + (ln >> 2) + 8 * h;
        const int grp = kCG * c + jj;
        if (row < d_out && grp < G)
            v = *reinterpret_cast<const uint4*>(packed + static_cast<size_t>(row) * (d_in / 2) + 64 * grp +
                                                16 * (ln & 3));
    } else {
        const int row = rb * kRowBlock + (i - kB1UnitPacked / 16);
        uint32_t e[4];
#pragma unroll
        for (int jj = 0; jj < kCG; ++jj) {
            const int grp = kCG * c + jj;
            e[jj] = 0;
            if (row < d_out && grp < G) {
                const size_t o = static_cast<size_t>(row) * G + grp;
                e[jj] = pack_h2(scales[o], zeros[o]);
            }
        }
        v = make_uint4(e[0], e[1], e[2], e[3]);
    }
    *reinterpret_cast<uint4*>(out + 16 * idx) = v;
}

// ---------------------------------------------------------------------------
// Dense FP16 GEMV (the reference's correctness oracle, also an API call)
// 512 threads; each warp streams 16-row x 128-column tiles with 16-byte loads.
// ---------------------------------------------------------------------------
constexpr int kRW = 16;
constexpr int kRT = kRW * 32;
constexpr int kRefDepth = 2;

struct RefArgs {
    const uint16_t* w16;
    const uint16_t* x;
    uint16_t* y;
    int d_out, d_in, n_rb, nrb_max;
};

__global__ void __launch_bounds__(kRT, 1) reference_gemv_kernel(const RefArgs a) {
    extern __shared__ __align__(128) char smem[];
    const int G = a.d_in / kGroup;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int rb0 = static_cast<int>(static_cast<long long>(blockIdx.x) * a.n_rb / gridDim.x);
    const int rb1 = static_cast<int>(static_cast<long long>(blockIdx.x + 1) * a.n_rb / gridDim.x);
    const int nrb = rb1 - rb0;
    const int U = nrb * G;
    const int u0 = static_cast<int>(static_cast<long long>(warp) * U / kRW);
    const int u1 = static_cast<int>(static_cast<long long>(warp + 1) * U / kRW);

    uint4* bsm = reinterpret_cast<uint4*>(smem);                       // [G][4][4] uint4
    float* part = reinterpret_cast<float*>(smem + G * 256);            // [nrb][NW][16]

    struct RStage { uint4 r0[4], r8[4]; };
    auto prefetch = [&](RStage& s, int rbl, int j) {
        const int r0 = min((rb0 + rbl) * kRowBlock + g, a.d_out - 1);
        const int r8 = min((rb0 + rbl) * kRowBlock + g + 8, a.d_out - 1);
        const uint16_t* b = a.w16 + kGroup * j + 32 * t;
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
            s.r0[wi] = ldg_stream_v4(b + static_cast<size_t>(r0) * a.d_in + 8 * wi);
            s.r8[wi] = ldg_stream_v4(b + static_cast<size_t>(r8) * a.d_in + 8 * wi);
        }
    };

    RStage ring[kRefDepth];
    int p_rb = (u0 < u1) ? u0 / G : 0, p_j = (u0 < u1) ? u0 % G : 0;
#pragma unroll
    for (int s = 0; s < kRefDepth; ++s) {
        if (u0 + s < u1) prefetch(ring[s], p_rb, p_j);
        if (++p_j == G) { p_j = 0; ++p_rb; }
    }
    // x in fragment order: chunk ch = 16j + 4t + wi -> bsm[(j*4 + wi)*4 + t]
    for (int ch = tid; ch < a.d_in / 8; ch += kRT) {
        const int j = ch >> 4, t_ = (ch >> 2) & 3, wi = ch & 3;
        bsm[(j * 4 + wi) * 4 + t_] = ldg_v4(a.x + 8 * static_cast<size_t>(ch));
    }
    for (int i = tid; i < nrb * kRW * 16; i += kRT) part[i] = 0.f;
    __syncthreads();

    float d[4] = {0.f, 0.f, 0.f, 0.f};
    int c_rb = (u0 < u1) ? u0 / G : 0, c_j = (u0 < u1) ? u0 % G : 0;
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
                        float* pp = part + (c_rb * kRW + warp) * 16;
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
    for (int r = tid; r < nrb * 16; r += kRT) {
        const int rbl = r >> 4, rr = r & 15;
        const int row = (rb0 + rbl) * kRowBlock + rr;
        if (row < a.d_out) {
            float s = 0.f;
#pragma unroll
            for (int w = 0; w < kRW; ++w) s += part[(rbl * kRW + w) * 16 + rr];
            a.y[row] = __half_as_ushort(__float2half_rn(s));
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
        for (int e = 0; e < 8; ++e) {
            const float f = h2f_bits(static_cast<uint16_t>(wv[e >> 1] >> (16 * (e & 1))));
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
            for (int e = 0; e < 8; ++e)
                word |= quant_code(static_cast<uint16_t>(wv[e >> 1] >> (16 * (e & 1))), gmin, inv) << (4 * e);
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
        for (int e = 0; e < 8; ++e) tile[rr][cc + e] = static_cast<uint16_t>(wv[e >> 1] >> (16 * (e & 1)));
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
constexpr int kNumKernels = 32;
int g_smem_set[kMaxDevices][kNumKernels];  // bytes already opted in (0 = none)

template <class K>
dq_status_t ensure_smem(K kernel, int id, int bytes) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
    if (dev >= 0 && dev < kMaxDevices && __atomic_load_n(&g_smem_set[dev][id], __ATOMIC_ACQUIRE) >= bytes)
        return DQ_OK;
    const int want = bytes < 48 * 1024 ? 48 * 1024 : bytes;
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
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
    return DQ_OK;
}

int plan_smem_bytes(int d_in) { return plan_layout(d_in).total + 256; }

template <bool kSplit>
dq_status_t launch_plan(const uint16_t* x, int d_in, float k, uint8_t* plan, uint32_t* mask_words,
                        int32_t* indices, int32_t* count, float* stats, cudaStream_t stream) {
    const int smem = plan_smem_bytes(d_in);
    const dq_status_t st = ensure_smem(plan_kernel<kSplit>, kSplit ? 1 : 2, smem);
    if (st != DQ_OK) return st;
    plan_kernel<kSplit><<<1, kPlanThreads, smem, stream>>>(x, d_in, k, plan, mask_words, indices, count, stats);
    return check_launch();
}

template <bool kSplit, bool kCM, bool kNative, bool kStage>
dq_status_t launch_gemv_pdl(const GemvArgs& a, int grid, int smem, cudaStream_t stream) {
    constexpr int id = 4 + (kSplit ? 8 : 0) + (kCM ? 4 : 0) + (kNative ? 2 : 0) + (kStage ? 1 : 0);
    const dq_status_t st = ensure_smem(gemv_kernel<kSplit, kCM, kNative, kStage>, id, smem);
    if (st != DQ_OK) return st;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, gemv_kernel<kSplit, kCM, kNative, kStage>, a);
    if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
    return check_launch();
}

}  // namespace

dq_status_t launch_gemv_b1(const dq_weights_t& w, const uint16_t* x, uint16_t* y, float k,
                           bool split, void* workspace, cudaStream_t stream) {
    DeviceInfo di;
    dq_status_t st = device_info(&di);
    if (st != DQ_OK) return st;
    const int G = w.d_in / kGroup;
    GemvArgs a;
    a.packed = w.packed;
    a.scales = w.scales;
    a.zeros = w.zeros;
    a.native = w.native;
    a.w16 = w.fp16;
    a.w16_cm = w.fp16_cm;
    a.y = y;
    a.d_out = w.d_out;
    a.d_in = w.d_in;
    a.n_rb = (w.d_out + kRowBlock - 1) / kRowBlock;
    a.NC = (G + kCG - 1) / kCG;
    a.U = a.n_rb * a.NC;
    const WsLayout W = ws_layout(w.d_out, w.d_in);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    a.plan = ws + W.plan;
    a.fix = reinterpret_cast<float*>(ws + W.fix);
    a.cnt = reinterpret_cast<unsigned int*>(ws + W.cnt);
    int grid = di.sm_count < a.U ? di.sm_count : a.U;
    if (grid > kMaxCtas) grid = kMaxCtas;
    int nrb_max = 1;
    for (int c = 0; c < grid; ++c) {
        const int u0 = unit_start(a.U, c, grid), u1 = unit_start(a.U, c + 1, grid);
        const int n = (u1 - 1) / a.NC - u0 / a.NC + 1;
        if (n > nrb_max) nrb_max = n;
    }
    a.nrb_max = nrb_max;
    const GemvSmem S = gemv_smem(a.d_in, a.nrb_max);
    if (S.total > di.smem_optin || plan_smem_bytes(a.d_in) > di.smem_optin) return DQ_ERR_UNSUPPORTED;

    st = split ? launch_plan<true>(x, a.d_in, k, ws + W.plan, nullptr, nullptr, nullptr, nullptr, stream)
               : launch_plan<false>(x, a.d_in, k, ws + W.plan, nullptr, nullptr, nullptr, nullptr, stream);
    if (st != DQ_OK) return st;

    const bool nat = w.native != nullptr;
    if (!split)
        return nat ? launch_gemv_pdl<false, false, true, false>(a, grid, S.total, stream)
                   : launch_gemv_pdl<false, false, false, false>(a, grid, S.total, stream);
    if (w.fp16_cm) {
        const bool stage = (w.d_out % 8) == 0;
        if (stage)
            return nat ? launch_gemv_pdl<true, true, true, true>(a, grid, S.total, stream)
                       : launch_gemv_pdl<true, true, false, true>(a, grid, S.total, stream);
        return nat ? launch_gemv_pdl<true, true, true, false>(a, grid, S.total, stream)
                   : launch_gemv_pdl<true, true, false, false>(a, grid, S.total, stream);
    }
    return nat ? launch_gemv_pdl<true, false, true, false>(a, grid, S.total, stream)
               : launch_gemv_pdl<true, false, false, false>(a, grid, S.total, stream);
}

dq_status_t launch_build_native(const uint8_t* packed, const uint16_t* scales, const uint16_t* zeros,
                                int d_out, int d_in, uint8_t* out, cudaStream_t stream) {
    const long long n_chunks = static_cast<long long>(native_bytes(d_out, d_in) / 16);
    if (n_chunks == 0) return DQ_OK;
    const int threads = 256;
    build_native_kernel<<<static_cast<unsigned>((n_chunks + threads - 1) / threads), threads, 0, stream>>>(
        packed, scales, zeros, d_out, d_in, out, n_chunks);
    return check_launch();
}

dq_status_t read_device_error(uint32_t* word, bool clear) {
    unsigned int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_error_word, sizeof(v));
    if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
    if (clear && v) {
        const unsigned int zero = 0;
        e = cudaMemcpyToSymbol(g_error_word, &zero, sizeof(zero));
        if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
    }
    *word = v;
    return DQ_OK;
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
    const int smem = (d_in / kGroup) * 256 + a.nrb_max * kRW * 16 * 4;
    if (smem > di.smem_optin) return DQ_ERR_UNSUPPORTED;
    if ((st = ensure_smem(reference_gemv_kernel, 3, smem)) != DQ_OK) return st;
    reference_gemv_kernel<<<grid, kRT, smem, stream>>>(a);
    return check_launch();
}

dq_status_t launch_detect(const uint16_t* x, int d_in, float k, uint32_t* mask_words,
                          int32_t* indices, int32_t* count, float* stats, cudaStream_t stream) {
    DeviceInfo di;
    const dq_status_t st = device_info(&di);
    if (st != DQ_OK) return st;
    if (plan_smem_bytes(d_in) > di.smem_optin) return DQ_ERR_UNSUPPORTED;
    return launch_plan<true>(x, d_in, k, nullptr, mask_words, indices, count, stats, stream);
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
    const dim3 grid(d_in / 64, (d_out + 63) / 64);
    colmajor_kernel<<<grid, 256, 0, stream>>>(w16, d_out, d_in, cm);
    return check_launch();
}

}  // namespace dq
