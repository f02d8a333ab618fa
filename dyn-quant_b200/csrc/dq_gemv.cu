// dq_gemv.cu -- batch-1 GEMV kernels for sm_100a: fused split (INT4 + FP16
// outlier columns), dense INT4, dense FP16, the standalone outlier detector,
// the bit-exact quantizer and the layout builders.
//
// Reference path (dyn-quant): src/split_gemv.cu:25-198, src/int4_gemv.cu:12-100,
// src/reference_gemv.cu:9-78, src/outlier_detect.cuh:104-205,
// src/quant_format.cuh:48-97.
//
// One split / INT4 GEMV call is ONE kernel (b1_kernel): a persistent grid of
// one CTA of 16 warps (12 for the longest rows) per SM, launched as a
// programmatic dependent of whatever precedes it on the stream.
//   1. Before griddepcontrol.wait, each CTA pulls its first weight units into
//      L2 (cp.async.bulk.prefetch), so the weight stream overlaps the previous
//      kernel.  After the wait each warp streams its units into a ring of
//      shared-memory stages (cp.async.bulk, the non-tensor TMA form,
//      completing on per-stage mbarriers).
//   2. Each CTA derives the activation plan itself from x (<= 60 KB, an L2
//      hit after the first CTA): the statistics, the outlier mask with the
//      reference's capacity rule, the outlier list, and the MMA B fragments
//      of the masked activation x' with per-group sums (dq_plan.cuh; the
//      pieces of x spread evenly over all threads).
//   3. The warps run dequant + tensor-core MMAs over their units.  A unit is
//      16 rows x 4 groups of 128 columns; the units are split evenly across
//      CTAs (and across the warps of a CTA) in (row block, column chunk)
//      order.  A 16-row block that straddles CTAs is finished by the CTA
//      holding its first chunk, which adds the later CTAs' published partial
//      row sums in CTA order (fixed order: results are bit-reproducible).
//   4. Outlier columns add W16[r][c] * x[c] on the tensor cores as well: tasks
//      of (16-row block, 16 outlier columns) run between a warp's units, their
//      column segments (32 contiguous bytes per row block in the column-major
//      FP16 mirror) brought in by cp.async and read with ldmatrix.trans.
//
// Tensor-core formulation (mma.sync.m16n8k16, f16 x f16 -> f32).  Lane
// (g, t) of a warp holds group t of the unit's 4-group chunk: A comes from the
// packed codes with the exponent bias kept (f16 1024 + q for the even columns
// of a word, 1024 + 16 q for the odd ones: one shift and four lop3 per word,
// all exact).  B holds x' of group t in MMA columns 2t (even columns of the
// words) and 2t + 1 (odd columns); every other lane supplies zeros.  The "lo"
// MMA accumulates D_lo[:, 2t] = 1024 Xe + S_even, the "hi" MMA accumulates
// D_hi[:, 2t + 1] = 1024 Xo + 16 S_odd (the other column of each is not read),
// so lane (g, t) ends with the two sums of group t for rows g and g + 8 and
// removes the bias in FP32 from the per-group sums of x':
//   y += s * ((S_even + S_odd) - z * X),   the reference's sum of s (q - z) x.
#include <cfloat>
#include <climits>

#include "dq_common.cuh"
#include "dq_internal.h"
#include "dq_plan.cuh"

namespace dq {

namespace {

constexpr int kStages = kB1Stages;
constexpr int kCG = kB1ChunkGroups;
constexpr int kStageBytes = kB1StageBytes;

// Set (bit 0) by a kernel whose bounded wait on its own copies gave up.
__device__ unsigned int g_error_word;


// ---------------------------------------------------------------------------
// Fused batch-1 GEMV
// ---------------------------------------------------------------------------
struct B1Args {
    const uint8_t* packed;    // reference layout [d_out][d_in/2]
    const uint16_t* scales;   // reference layout [d_out][G]
    const uint16_t* zeros;
    const uint8_t* native;    // unit layout (native_bytes), or null
    const uint16_t* w16;      // row-major FP16 (split path without mirror)
    const uint16_t* w16_cm;   // column-major FP16 mirror
    const uint16_t* x;
    uint16_t* y;
    unsigned int* hdr;        // workspace: [0] tag of the last completed call, [1] CTAs done in this call
    unsigned long long* fix;  // workspace: per CTA, the published partial sums of its first row block
    unsigned long long* xsl;  // workspace: per row block and slab 1 .. nslab-1, its partial sums
    float k;
    float inv_n, inv_n1;      // 1/d_in, 1/(d_in - 1) for the statistics of x
    int d_out, d_in, NC, U, nrb_max;
    int nslab, NCs;           // column slabs (1: none) and chunks per slab; U = row blocks x NCs
    int depth;                // ring stages per warp (reference layout: kB1Stages)
    B1Smem S;
    // fused gather (kGather): this rank, the ranks, slice height, output rows,
    // every rank's gather region as mapped here
    int g_rank, g_world, g_rows_per, g_total;
    uint8_t* g_region[kMaxGatherRanks];
    GatherLayout g_lay;
};

// How the split path reads the FP16 weights of outlier columns.
enum : int {
    kOutNone = 0,       // INT4 only
    kOutStaged = 1,     // column-major mirror, d_out % 8 == 0: bulk copies of row segments
    kOutColDirect = 2,  // column-major mirror, other d_out: plain loads
    kOutRowDirect = 3,  // row-major FP16 only: plain loads
};

__host__ __device__ inline int unit_start(long long U, int c, int P) {
    return static_cast<int>(U * c / P);
}
__host__ __device__ inline int unit_owner(long long u, int P, long long U) {
    return static_cast<int>((u * P + P - 1) / U);
}

// The fused gather, after this CTA stored its rows (in y and, as tagged
// words, in every other rank's region): the same rows of every other rank's
// slice (rows [r0, r1) of the slice, which that rank's CTA of the same index
// stores, the partition being the same on every rank) are read from this
// rank's own region once their words carry this call's tag, and written
// into y.  Each word is waited for (bounded, about a second in all: on
// timeout bit 4 of the error word is set and the row is left unwritten).
template <int kT>
__device__ void gather_rows(const B1Args& a, uint32_t call, int r0, int r1) {
    const uint32_t tag = call & 0xFFFFu, par = call & 1u;
    const uint32_t* src = reinterpret_cast<const uint32_t*>(a.g_region[a.g_rank] + a.g_lay.yfull + par * a.g_lay.ybytes);
    const int n = r1 - r0, total = (a.g_world - 1) * n;
    const long long t_end = clock64() + (1ll << 31);
    bool ok = true;
    // (other rank, row) pairs spread over all threads, so that every word is
    // waited for at the same time
    for (int i = threadIdx.x; i < total && ok; i += kT) {
        const int qi = i / n, q = qi + (qi >= a.g_rank ? 1 : 0);
        const int grow = q * a.g_rows_per + r0 + (i - qi * n);
        if (grow >= a.g_total) continue;
        uint32_t w = ld_relaxed_sys_u32(src + grow);
        while ((w >> 16) != tag) {
            if (clock64() > t_end) {
                ok = false;
                break;
            }
            __nanosleep(64);
            w = ld_relaxed_sys_u32(src + grow);
        }
        if (ok) a.y[grow] = static_cast<uint16_t>(w & 0xFFFFu);
    }
    if (!ok) atomicOr(&g_error_word, 16u);
}

// Rounds of the balanced plan partition (pieces of x per thread) for the
// longest rows (kMaxDIn) in a CTA of kW warps.
template <int kW>
constexpr int plan_rounds_max() { return (kMaxDIn / 8 + 32 * kW - 1) / (32 * kW); }

// kNative: weights in the unit layout (one bulk copy per unit, scale/zero
// inside); otherwise the reference layout (one bulk copy per weight row of the
// unit, scale/zero by plain loads).  kR: rounds of the plan's balanced
// partition (at least ceil(64 NC / threads)).  kGather: the row-sharded gather is fused
// (each output row also goes to every other rank's gather region; the last
// CTA exchanges the arrivals and copies the other ranks' rows into y).
template <bool kSplit, bool kNative, int kOut, int kW, int kR, bool kGather, bool kSlab>
__global__ void __launch_bounds__(kW * 32, 1) b1_kernel(const B1Args a) {
    constexpr int kT = kW * 32;
    extern __shared__ __align__(128) char smem[];
    const int G = a.d_in / kGroup;
    const int n8 = a.d_in >> 3;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int c = blockIdx.x;
    // Column slabs (kSlab, long rows): CTAs [cs0, cs0 + P) work on slab sl,
    // the NCs chunks sl NCs .. (sl + 1) NCs - 1 of every row block.  The unit
    // indices below are the slab's, (row block, chunk of the slab), and a
    // row's slab sums meet in the CTA of slab 0 that stores it.
    const int nslab = kSlab ? a.nslab : 1;
    const int grid = static_cast<int>(gridDim.x);
    const int sl = nslab > 1 ? ((c + 1) * nslab - 1) / grid : 0;
    const int cs0 = sl * grid / nslab;
    const int P = (sl + 1) * grid / nslab - cs0;
    const int cl = c - cs0;         // this CTA's index within its slab
    const int NC = a.NCs;           // chunks per row block in this CTA's unit sequence
    const int chunk0 = sl * a.NCs;  // first chunk of the slab
    const long long U = a.U;        // units of the slab: row blocks x NC
    auto gunit = [&](int u) -> long long {  // a unit of the slab as a unit of the weights
        if (nslab == 1) return u;
        const int rb = u / NC;
        return static_cast<long long>(rb) * a.NC + chunk0 + (u - rb * NC);
    };

    // This CTA's units [cu0, cu1) in (row block, chunk) order.  Warp w takes
    // cu0 + w, cu0 + w + kW, ..., so all warps work through the first row block
    // together at the start and through the last one at the end.
    const int cu0 = unit_start(U, cl, P), cu1 = unit_start(U, cl + 1, P);
    const int rbf = cu0 / NC;                 // first row block touched by this CTA
    const int rbz = (cu1 - 1) / NC;           // last
    const int nrb = rbz - rbf + 1;
    // A row block split between CTAs is finished by the CTA holding its chunk 0
    // (the "finaliser", for which it is the last row block); every later CTA
    // touching it (a "contributor", for which it is the first row block)
    // publishes its partial row sums early, without the outlier columns, which
    // the finaliser adds for the whole block.
    const bool contrib = cu0 > rbf * NC;
    const bool finaliser = cu1 < (rbz + 1) * NC && !(rbf == rbz && contrib);
    const int n_pub = min(kW, min(cu1, (rbf + 1) * NC) - cu0);  // warps holding units of rbf
    const int wn = (cu1 - cu0 > warp) ? (cu1 - cu0 - warp + kW - 1) / kW : 0;  // units of this warp
    const int orb0 = contrib ? rbf + 1 : rbf;  // outlier rows of this CTA: row blocks orb0 .. rbz
    const size_t row_stride = static_cast<size_t>(a.d_in) / 2;

    // Ring: this warp's i-th unit goes to slot warp + kW (i % D), D stages per
    // warp (as many as fit next to the plan, at least kB1Stages).
    const int D = kNative ? a.depth : kStages;
    const uint32_t ring = smem_u32(smem + a.S.ring);
    const uint32_t bars = smem_u32(smem + a.S.bars);
    auto slot_of = [&](int k) -> int { return warp + kW * k; };
    float* part = reinterpret_cast<float*>(smem + a.S.part);    // [row block][warp][16]
    float* opart = reinterpret_cast<float*>(smem + a.S.opart);  // [warp][row block][16]
    uint4* xb = reinterpret_cast<uint4*>(smem + a.S.bsm);
    float4* xp4 = reinterpret_cast<float4*>(smem + a.S.xp);
    uint8_t* mask = reinterpret_cast<uint8_t*>(smem + a.S.mask);
    float* red = reinterpret_cast<float*>(smem + a.S.red);
    uint32_t* list = reinterpret_cast<uint32_t*>(smem + a.S.list);

    if (lane == 0) {
        for (int k = 0; k < D && k < wn; ++k) mbar_init(bars + 8 * slot_of(k), 1);
        fence_mbar_init();
    }
    for (int i = tid; i < nrb * kW * 16; i += kT) part[i] = 0.f;
    if (kSplit && kOut != kOutNone)
        for (int i = tid; i < kW * a.nrb_max * 16; i += kT) opart[i] = 0.f;
    for (int i = tid; i < kB1ChunkB / 16; i += kT) reinterpret_cast<uint4*>(smem + a.S.zero)[i] = make_uint4(0, 0, 0, 0);
    __syncthreads();

    uint32_t szr0[kStages], szr8[kStages];  // reference layout: (scale, zero) of lane t's group, rows g, g+8

    // Weight bytes of unit u into stage s (s < D; compile-time for the
    // reference layout, whose scale/zero go to registers).
    auto issue = [&](int s, int u) {
        const int rb = u / NC, cc = u - rb * NC;
        const uint32_t bar = bars + 8 * slot_of(s);
        const uint32_t dst = ring + slot_of(s) * kStageBytes;
        if (kNative) {
            if (lane == 0) {
                mbar_arrive_expect_tx(bar, kB1UnitBytes);
                bulk_g2s(dst, a.native + static_cast<size_t>(gunit(u)) * kB1UnitBytes, kB1UnitBytes, bar);
            }
        } else {
            const int rbase = rb * kRowBlock;
            const int ng = min(kCG, G - kCG * cc);
            const int vrows = min(kRowBlock, a.d_out - rbase);
            const uint32_t rbytes = static_cast<uint32_t>(ng) * 64u;
            if (lane == 0) mbar_arrive_expect_tx(bar, vrows * rbytes);
            __syncwarp();
            if (lane < vrows)
                bulk_g2s(dst + lane * kB1RowPitch,
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

    // The weights do not depend on the preceding kernel: each warp's first
    // kB1Stages units are pulled into L2 before griddepcontrol.wait (native
    // layout).  After the wait x is requested first (cp.async into shared
    // memory), then the ring's first fill, which so does not hold x up.  (Copying the
    // units into shared memory before the wait, or all of a CTA's share at
    // once, puts the weight stream in front of x on the SM's return path and
    // made chains of GEMVs slower.)
    const int fill = min(wn, D);
    uint32_t armed = 0;  // stages with a copy in flight
    if (kNative && lane == 0)
        for (int k = 0; k < fill && k < kB1Stages; ++k)
            prefetch_l2_bulk(a.native + static_cast<size_t>(gunit(cu0 + warp + kW * k)) * kB1UnitBytes, kB1UnitBytes);
    pdl_launch_dependents();
    pdl_wait();  // x, y and the workspace may belong to the preceding kernel until here
    // This call's tag: one more than the last completed call's (never zero).
    // Every CTA reads it before it finishes, and the last CTA to finish
    // advances it, so all CTAs of a call see the same tag.
    uint32_t& s_tag = *reinterpret_cast<uint32_t*>(smem + a.S.misc);
    // Gather: misc[1] this call's number (calls this rank completed + 1; its
    // parity picks the copy written in the ranks' regions, its low 16 bits
    // tag the words), misc[2] last CTA.
    uint32_t* gmisc = reinterpret_cast<uint32_t*>(smem + a.S.misc);
    if (tid == 0) {
        const uint32_t e = ldcg_u32(a.hdr) + 1u;
        s_tag = e == 0u ? 1u : e;
        if (kGather) gmisc[1] = ldcg_u32(a.g_region[a.g_rank] + a.g_lay.hdr) + 1u;
    }
    // Output row `row` (< d_out) of this call: y, and with the gather also
    // every other rank's copy (peer stores over NVLink).
    auto store_row = [&](int row, float v) {
        const uint16_t h = __half_as_ushort(__float2half_rn(v));
        if (!kGather) {
            a.y[row] = h;
            return;
        }
        const int grow = a.g_rank * a.g_rows_per + row;
        if (grow >= a.g_total) return;
        a.y[grow] = h;
        const uint32_t call = gmisc[1];
        const size_t off = a.g_lay.yfull + static_cast<size_t>(call & 1u) * a.g_lay.ybytes + 4 * static_cast<size_t>(grow);
        const uint32_t word = static_cast<uint32_t>(h) | ((call & 0xFFFFu) << 16);
        for (int q = 0; q < a.g_world; ++q)
            if (q != a.g_rank) st_relaxed_sys_u32(reinterpret_cast<uint32_t*>(a.g_region[q] + off), word);
    };
    // Output row `row` of this call with this CTA's sum v: with column slabs
    // a CTA of slab sl > 0 publishes v as a tagged word (this call's tag in the
    // high half) for the row's slab-0 CTA, which waits for the nslab - 1
    // words (bounded), adds them in slab order and stores the row.
    bool slab_ok = true;
    auto emit_row = [&](int row, float v) {
        if (nslab == 1) {
            store_row(row, v);
            return;
        }
        unsigned long long* w = a.xsl + static_cast<size_t>(row >> 4) * (nslab - 1) * 16 + (row & 15);
        const uint32_t tag = s_tag;
        if (sl > 0) {
            st_relaxed_gpu_u64(w + (sl - 1) * 16, (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(v));
            return;
        }
        const long long t0 = clock64();
        for (int q = 1; q < nslab; ++q) {
            unsigned long long u = ld_relaxed_gpu_u64(w + (q - 1) * 16);
            while (static_cast<uint32_t>(u >> 32) != tag && clock64() - t0 < (1ll << 31))
                u = ld_relaxed_gpu_u64(w + (q - 1) * 16);
            slab_ok = slab_ok && static_cast<uint32_t>(u >> 32) == tag;
            v += __uint_as_float(static_cast<uint32_t>(u));
        }
        store_row(row, v);
    };
    // x into xb in natural order (requested before the weight copies, so that
    // it does not queue behind them on the SM's return path): with column
    // slabs only the slab's pieces, and for the split GEMV all of x once more
    // into the staging area (the statistics and the outlier count are over
    // all of x).  The staging area is the row sums, the outlier list and the
    // outlier buffers, none of which is used before the plan ends.
    const int piece0 = 64 * chunk0;
    const int n8s = nslab > 1 ? min(64 * NC, n8 - piece0) : n8;
    const bool stage_x = kSplit && nslab > 1;
    uint4* xstage = reinterpret_cast<uint4*>(smem + a.S.part);
    load_x_async<kT>(a.x + 8 * static_cast<size_t>(piece0), n8s, xb);
    if (stage_x) load_x_async<kT>(a.x, n8, xstage);
    if (kNative) {
        for (int k = 0; k < fill; ++k) {
            issue(k, cu0 + warp + kW * k);
            armed |= 1u << k;
        }
    } else {
#pragma unroll
        for (int s = 0; s < kStages; ++s) {
            if (s < wn) {
                issue(s, cu0 + warp + kW * s);
                armed |= 1u << s;
            }
        }
    }
    cp_async_wait_all();
    __syncthreads();

    // ---- activation plan: statistics, mask, MMA B fragments of x', outlier list ----
    int n_out = 0;
    int* pscratch = reinterpret_cast<int*>(red) + 32;  // after the statistics' 32 floats
    if (kSplit) {
        const uint4* xs = stage_x ? xstage : xb;  // all of x
        const XStats st = x_stats<kT>(xs, n8, a.d_in, a.k, a.inv_n, a.inv_n1, red);
        int total_all = 0;
        if (stage_x) {
            int cnt = 0;
            for (int p = tid; p < n8; p += kT) cnt += __popc(piece_bits(xs[p], st.mean, st.thresh));
            total_all = block_count<kT>(cnt, pscratch + 128);
        }
        n_out = plan_balanced<kT, kR, true, kSlab>(xb, n8s, NC, a.d_in, st.mean, st.thresh, xp4, list,
                                                   reinterpret_cast<uint32_t*>(mask), pscratch, xs, piece0, total_all);
        if (stage_x) {  // the staging area becomes the row sums again
            for (int i = tid; i < nrb * kW * 16; i += kT) part[i] = 0.f;
            if (kOut != kOutNone)
                for (int i = tid; i < kW * a.nrb_max * 16; i += kT) opart[i] = 0.f;
            __syncthreads();
        }
    } else {
        plan_balanced<kT, kR, false>(xb, n8s, NC, a.d_in, 0.f, 0.f, xp4, nullptr, nullptr, pscratch);
    }

    // ---- outlier columns: y[r] += W16[r][c] * x[c] for the rows of row blocks orb0 .. rbz ----
    // A small tensor-core GEMM.  Tasks (row block, 16 outlier columns), in
    // row-block-major order, are split contiguously over the warps and run
    // between the warps' units.  A task's 16 column segments (16 rows of FP16
    // each, column-major) come into one of the warp's kB1OutBufs buffers, one
    // 16-byte piece per lane; ldmatrix.trans turns them into the MMA A fragment
    // (rows x outlier columns) and B holds the outliers' x.  A warp accumulates
    // in registers while it stays in one row block and then writes its opart row.
    constexpr bool kOutl = kSplit && kOut != kOutNone;
    const int n_orb = (kOutl && n_out > 0 && orb0 <= rbz) ? rbz - orb0 + 1 : 0;
    const int nbat = (n_out + kB1OutBatch - 1) / kB1OutBatch;
    const int ntask = n_orb * nbat;
    const int tk0 = static_cast<int>(static_cast<long long>(ntask) * warp / kW);
    const int ntk = static_cast<int>(static_cast<long long>(ntask) * (warp + 1) / kW) - tk0;
    const uint32_t wbuf = smem_u32(smem + a.S.obuf) + warp * kB1OutBufs * kB1OutBufBytes;
    float od[4] = {0.f, 0.f, 0.f, 0.f};
    auto o_issue = [&](int k) {  // task tk0 + k into buffer k % kB1OutBufs
        const int task = tk0 + k;
        const int rb = orb0 + task / nbat;
        const int kc = (task % nbat) * kB1OutBatch + (lane >> 1);  // outlier (list index) of this lane's piece
        const int row0 = rb * kRowBlock + 8 * (lane & 1);
        const uint32_t dst = wbuf + (k % kB1OutBufs) * kB1OutBufBytes + 16 * lane;
        const bool valid = kc < n_out && row0 < a.d_out;
        const int col = valid ? static_cast<int>(list[kc] & 0xFFFFu) : 0;
        if (kOut == kOutStaged) {
            if (valid) cp_async16(dst, a.w16_cm + static_cast<size_t>(col) * a.d_out + row0);
            else sts_v4(dst, make_uint4(0, 0, 0, 0));
            cp_async_commit();
        } else {
            uint16_t h[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int r = row0 + i;
                h[i] = (valid && r < a.d_out)
                           ? (kOut == kOutColDirect ? ldg_u16(a.w16_cm + static_cast<size_t>(col) * a.d_out + r)
                                                    : ldg_u16(a.w16 + static_cast<size_t>(r) * a.d_in + col))
                           : static_cast<uint16_t>(0);
            }
            sts_v4(dst, make_uint4(pack_h2(h[0], h[1]), pack_h2(h[2], h[3]), pack_h2(h[4], h[5]),
                                   pack_h2(h[6], h[7])));
        }
    };
    auto o_step = [&](int k) {  // run task tk0 + k
        const int task = tk0 + k;
        const int rb = orb0 + task / nbat;
        const int k0 = (task % nbat) * kB1OutBatch;
        if (kOut == kOutStaged) {
            if (k + 2 < ntk) cp_async_wait_group<2>();
            else if (k + 1 < ntk) cp_async_wait_group<1>();
            else cp_async_wait_group<0>();
        }
        __syncwarp();
        const uint32_t buf = wbuf + (k % kB1OutBufs) * kB1OutBufBytes;
        uint32_t a0, a1, a2, a3;
        // matrix j = (column half j >> 1, row half j & 1); lane 8j + i gives column (j >> 1) * 8 + i
        ldmatrix_x4_trans(buf + (((lane >> 4) * 8 + (lane & 7)) * 32) + ((lane >> 3) & 1) * 16, a0, a1, a2, a3);
        auto xo = [&](int kk) -> uint32_t { return kk < n_out ? (list[kk] >> 16) : 0u; };
        const uint32_t b0 = xo(k0 + 2 * t) | (xo(k0 + 2 * t + 1) << 16);
        const uint32_t b1 = xo(k0 + 2 * t + 8) | (xo(k0 + 2 * t + 9) << 16);
        mma_16816(od, a0, a1, a2, a3, b0, b1);
        __syncwarp();  // every lane is done with the buffer before it is refilled
        if (k + kB1OutBufs < ntk) o_issue(k + kB1OutBufs);
        if (k == ntk - 1 || (task + 1) % nbat == 0) {  // leaving row block rb
            if (t == 0) {
                float* op = opart + (warp * a.nrb_max + (rb - rbf)) * 16;
                op[g] = od[0];
                op[g + 8] = od[2];
            }
            od[0] = od[1] = od[2] = od[3] = 0.f;
        }
    };
    int o_done = 0;  // outlier tasks run by this warp
    for (int k = 0; k < kB1OutBufs && k < ntk; ++k) o_issue(k);

    // Partial row sums of rbf (shared with earlier CTAs) go to the workspace as
    // soon as the warps holding its units are done with it: those warps meet on
    // named barrier 1 and the last of them publishes.  Each sum is one 64-bit
    // word (this call's tag << 32 | FP32 bits), written in one piece, so the
    // finaliser needs no fence or flag: the tag marks a value published by
    // this call.  Called exactly once by each of warps 0 .. n_pub-1 (also on
    // the error path, so that the barrier fills).
    bool pub_pending = contrib && warp < n_pub;
    auto publish_first = [&]() {
        if (warp == n_pub - 1) {
            if (n_pub > 1) named_bar_sync(1, n_pub * 32);
            if (lane < 16) {
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < kW; ++w) v += part[w * 16 + lane];
                st_relaxed_gpu_u64(a.fix + c * 16 + lane,
                                   (static_cast<unsigned long long>(s_tag) << 32) | __float_as_uint(v));
            }
        } else {
            named_bar_arrive(1, n_pub * 32);
        }
    };
    // The finaliser's warp 0 (lanes 0-15 = rows of rbz) adds the contributors'
    // sums in CTA order.  With one contributor its word is loaded in the middle
    // of the unit loop and only inspected at the end.
    const int c_hi = finaliser ? cs0 + unit_owner(static_cast<long long>(rbz + 1) * NC - 1, P, U) : c;
    unsigned long long early = 0ull;

    // ---- units ----
    const uint32_t zero_a = smem_u32(smem + a.S.zero);
    const uint32_t bsm_a = smem_u32(xb);
    const uint32_t xp_a = smem_u32(xp4);
    const bool b_owner = (g >> 1) == t;  // lane supplies B column 2t (g even) or 2t+1 (g odd)
    const uint32_t b_lane = t * 16 + (g & 1) * 8;
    float acc0 = 0.f, acc8 = 0.f;
    bool ok = true;
    uint32_t phase = 0;  // per stage: parity of the next completion
    // Unit i of this warp, in stage s, whose copy has landed.  sz0 / sz8: the
    // reference layout's (scale, zero) registers of the stage.
    auto consume = [&](int i, int s, uint32_t sz0, uint32_t sz8) {
        const uint32_t st = ring + slot_of(s) * kStageBytes;
        const int u = cu0 + warp + kW * i;
        const int rb = u / NC, cc = u - rb * NC;
        uint4 aw[4][2];  // [slice][row g / g+8]: 32 columns of group t
#pragma unroll
        for (int sl = 0; sl < 4; ++sl)
#pragma unroll
            for (int h = 0; h < 2; ++h)
                aw[sl][h] = kNative ? lds_v4(st + native_piece(sl, h, g, t) * 16)
                                    : lds_v4(st + (g + 8 * h) * kB1RowPitch + 64 * t + 16 * sl);
        const uint32_t bb = (b_owner ? bsm_a + cc * kB1ChunkB : zero_a) + b_lane;
        float dl[4][4], dh[4][4];
#pragma unroll
        for (int sl = 0; sl < 4; ++sl)
#pragma unroll
            for (int q = 0; q < 4; ++q) dl[sl][q] = dh[sl][q] = 0.f;
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
#pragma unroll
            for (int sl = 0; sl < 4; ++sl) {
                const Biased4 qa = biased_word(word_of(aw[sl][0], wi));
                const Biased4 qb = biased_word(word_of(aw[sl][1], wi));
                const uint2 b = lds_v2(bb + (wi * 4 + sl) * 64);
                mma_16816(dl[sl], qa.lo0, qb.lo0, qa.lo1, qb.lo1, b.x, b.y);
                mma_16816(dh[sl], qa.hi0, qb.hi0, qa.hi1, qb.hi1, b.x, b.y);
            }
        }
        const float lo0 = (dl[0][0] + dl[1][0]) + (dl[2][0] + dl[3][0]);
        const float hi0 = (dh[0][1] + dh[1][1]) + (dh[2][1] + dh[3][1]);
        const float lo8 = (dl[0][2] + dl[1][2]) + (dl[2][2] + dl[3][2]);
        const float hi8 = (dh[0][3] + dh[1][3]) + (dh[2][3] + dh[3][3]);
        if (kNative) {
            sz0 = lds_u32(st + kB1UnitPacked + 16 * g + 4 * t);
            sz8 = lds_u32(st + kB1UnitPacked + 16 * (g + 8) + 4 * t);
        }
        const uint4 xqb = lds_v4(xp_a + (kCG * cc + t) * 16);
        const float xe = __uint_as_float(xqb.x), xo = __uint_as_float(xqb.y), xs = __uint_as_float(xqb.z);
        const float S0 = fmaf(hi0 - xo, 0.0625f, lo0 - xe);
        const float S8 = fmaf(hi8 - xo, 0.0625f, lo8 - xe);
        acc0 = fmaf(h2f_bits(lo16(sz0)), fmaf(-h2f_bits(hi16(sz0)), xs, S0), acc0);
        acc8 = fmaf(h2f_bits(lo16(sz8)), fmaf(-h2f_bits(hi16(sz8)), xs, S8), acc8);
        const bool last_in_rb = i == wn - 1 || u + kW >= (rb + 1) * NC;
        if (last_in_rb) {
            // This warp is done with row block rb: publish its row sums.
            acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
            acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
            acc8 += __shfl_xor_sync(0xffffffffu, acc8, 1);
            acc8 += __shfl_xor_sync(0xffffffffu, acc8, 2);
            if (t == 0) {
                float* pp = part + ((rb - rbf) * kW + warp) * 16;
                pp[g] = acc0;
                pp[g + 8] = acc8;
            }
            acc0 = acc8 = 0.f;
        }
        __syncwarp();
        if (i + D < wn) {
            issue(s, u + kW * D);
            armed |= 1u << s;
        }
        if (last_in_rb && rb == rbf && pub_pending) {
            publish_first();
            pub_pending = false;
        }
        if (finaliser && c_hi == c + 1 && warp == 0 && i == wn / 2)
            early = ld_relaxed_gpu_u64(a.fix + (c + 1) * 16 + (lane & 15));
        // outlier tasks, spread evenly over this warp's units
        const int target = min(ntk, (ntk * (i + 1) + wn - 1) / wn);
        for (; o_done < target; ++o_done) o_step(o_done);
    };
    if (kNative) {
        for (int i = 0, s = 0; i < wn && ok; ++i, s = (s + 1 == D) ? 0 : s + 1) {
            const bool got = mbar_wait_bounded(bars + 8 * slot_of(s), (phase >> s) & 1u);
            if (!__all_sync(0xffffffffu, got)) {
                ok = false;
                if (lane == 0) atomicOr(&g_error_word, 1u);
            } else {
                phase ^= 1u << s;
                armed &= ~(1u << s);
                consume(i, s, 0u, 0u);
            }
        }
    } else {
        for (int ib = 0; ib < wn && ok; ib += kStages) {
#pragma unroll
            for (int s = 0; s < kStages; ++s) {
                const int i = ib + s;
                if (i < wn && ok) {
                    const bool got = mbar_wait_bounded(bars + 8 * slot_of(s), (phase >> s) & 1u);
                    if (!__all_sync(0xffffffffu, got)) {
                        ok = false;
                        if (lane == 0) atomicOr(&g_error_word, 1u);
                    } else {
                        phase ^= 1u << s;
                        armed &= ~(1u << s);
                        consume(i, s, szr0[s], szr8[s]);
                    }
                }
            }
        }
    }
    if (!ok) {
        // Do not leave copies in flight into shared memory this CTA is about to release.
        for (int k = 0; k < D; ++k)
            if (armed & (1u << k)) mbar_wait_bounded(bars + 8 * slot_of(k), (phase >> k) & 1u);
    }
    if (pub_pending) publish_first();  // error path: keep named barrier 1 balanced
    for (; o_done < ntk; ++o_done) o_step(o_done);  // warps without units, error path
    __syncthreads();

    // Row sums: the warps' INT4 sums in order, then the warps' outlier sums in
    // order.  rbf of a contributor was published above; rbz of a finaliser adds
    // the contributors' sums (in CTA order).
    const bool with_out = kOutl && n_orb > 0;
    for (int r = tid; r < nrb * 16; r += kT) {
        const int rbl = r >> 4, rr = r & 15;
        const int rb = rbf + rbl;
        if ((rbl == 0 && contrib) || (rb == rbz && finaliser)) continue;
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < kW; ++w) sum += part[(rbl * kW + w) * 16 + rr];
        if (with_out && rb >= orb0)
#pragma unroll
            for (int w = 0; w < kW; ++w) sum += opart[(w * a.nrb_max + rbl) * 16 + rr];
        const int row = rb * kRowBlock + rr;
        if (row < a.d_out) emit_row(row, sum);
    }
    if (finaliser && warp == 0) {
        const int rbl = rbz - rbf;
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < kW; ++w) sum += part[(rbl * kW + w) * 16 + (lane & 15)];
        if (with_out)
#pragma unroll
            for (int w = 0; w < kW; ++w) sum += opart[(w * a.nrb_max + rbl) * 16 + (lane & 15)];
        const int row = rbz * kRowBlock + (lane & 15);
        const uint32_t tag = s_tag;
        bool ok_all = true;
        for (int cc = c + 1; cc <= c_hi; ++cc) {
            unsigned long long* slot = a.fix + cc * 16 + (lane & 15);
            unsigned long long v = (cc == c + 1) ? early : 0ull;
            if (static_cast<uint32_t>(v >> 32) != tag) {
                v = ld_relaxed_gpu_u64(slot);
                const long long t0 = clock64();
                while (static_cast<uint32_t>(v >> 32) != tag && clock64() - t0 < (1ll << 31))
                    v = ld_relaxed_gpu_u64(slot);
            }
            ok_all = ok_all && static_cast<uint32_t>(v >> 32) == tag;
            sum += __uint_as_float(static_cast<uint32_t>(v));
        }
        if (!__all_sync(0xffffffffu, ok_all) && lane == 0) atomicOr(&g_error_word, 2u);
        if (lane < 16 && row < a.d_out) emit_row(row, sum);
    }
    if (!slab_ok) atomicOr(&g_error_word, 2u);

    // This CTA is done with the workspace (its tag read, its words published,
    // its finaliser wait over): the last CTA of the call advances the tag.
    if constexpr (kGather) {
        // The rows this CTA stores: its row blocks from rbf (rbf + 1 when a
        // contributor) to rbz, below d_out.
        const int rs = (contrib ? rbf + 1 : rbf) * kRowBlock;
        const int re = sl > 0 ? rs : min((rbz + 1) * kRowBlock, a.d_out);  // slab 0 stores the rows
        __syncthreads();  // (every thread has the call number)
        if (re > rs) gather_rows<kT>(a, gmisc[1], rs, re);
    }
    __syncthreads();
    if (tid == 0) {
        const bool last = atomicAdd(a.hdr + 1, 1u) == gridDim.x - 1u;
        if (last) {
            a.hdr[1] = 0u;
            a.hdr[0] = s_tag;
            // every CTA has read this call's number: count the call completed
            if (kGather) reinterpret_cast<unsigned int*>(a.g_region[a.g_rank] + a.g_lay.hdr)[0] = gmisc[1];
        }
    }
}

// Native unit layout: per (row-block rb, 4-group chunk c) one block of
// kB1UnitBytes = 4096 bytes of packed codes, 256 pieces of 16 bytes (piece
// native_piece(sl, h, g, t): row rb*16 + g + 8h, group 4c + t, columns
// 32 sl .. 32 sl + 31 of that group) followed by 256 bytes of
// (scale | zero << 16) for [16 rows][4 groups].  Rows past d_out and groups
// past G are zero.
__global__ void build_native_kernel(const uint8_t* __restrict__ packed, const uint16_t* __restrict__ scales,
                                    const uint16_t* __restrict__ zeros, int d_out, int d_in,
                                    uint8_t* __restrict__ out, long long n_chunks) {
    const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= n_chunks) return;
    constexpr int kChunks = kB1UnitBytes / 16;  // 272 sixteen-byte pieces per unit
    const int G = d_in / kGroup;
    const int NC = (G + kCG - 1) / kCG;
    const long long unit = idx / kChunks;
    const int i = static_cast<int>(idx % kChunks);
    const int rb = static_cast<int>(unit / NC), c = static_cast<int>(unit % NC);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (i < kB1UnitPacked / 16) {
        const int sl = i >> 6, h = (i >> 5) & 1, pos = i & 31;
        const int t = pos >> 3, g = (pos & 7) ^ (2 * t);  // inverse of native_piece
        const int row = rb * kRowBlock + g + 8 * h;
        const int grp = kCG * c + t;
        if (row < d_out && grp < G)
            v = *reinterpret_cast<const uint4*>(packed + static_cast<size_t>(row) * (d_in / 2) + 64 * grp + 16 * sl);
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
// Standalone outlier detector (one CTA of the GEMV's thread count): the same
// mask, list and statistics as the GEMV's plan, written out.
// ---------------------------------------------------------------------------
struct DetectSmem {
    int xs, mask, list, red, total;
};
__host__ __device__ inline DetectSmem detect_smem(int d_in) {
    DetectSmem S;
    int off = 0;
    S.xs = off;   off += 2 * d_in;
    S.mask = off; off += align16(d_in / 8);
    S.list = off; off += align16(d_in);
    S.red = off;  off += 2048;  // statistics and scan scratch; the exact sum of x at +1024
    S.total = off;
    return S;
}

__global__ void __launch_bounds__(kStatThreads, 1)
    detect_kernel(const uint16_t* __restrict__ x, int d_in, float k, float inv_n, float inv_n1,
                  uint32_t* mask_words, int32_t* indices, int32_t* count, float* stats) {
    extern __shared__ __align__(128) char smem[];
    const DetectSmem S = detect_smem(d_in);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int n8 = d_in / 8;
    uint4* xs = reinterpret_cast<uint4*>(smem + S.xs);
    uint8_t* mask = reinterpret_cast<uint8_t*>(smem + S.mask);
    uint32_t* list = reinterpret_cast<uint32_t*>(smem + S.list);
    float* red = reinterpret_cast<float*>(smem + S.red);
    load_x_async<kStatThreads>(x, n8, xs);
    cp_async_wait_all();
    __syncthreads();
    const XStats st = x_stats<kStatThreads>(xs, n8, d_in, k, inv_n, inv_n1, red);
    const int n = x_mask_list<kStatThreads>(xs, d_in, st.mean, st.thresh, reinterpret_cast<uint32_t*>(mask), list,
                                            reinterpret_cast<int*>(red) + 2 * (kStatThreads / 32));
    __syncthreads();
    const uint32_t* words = reinterpret_cast<const uint32_t*>(mask);
    if (mask_words)
        for (int i = tid; i < d_in / 32; i += kStatThreads) mask_words[i] = words[i];
    if (tid == 0) {
        if (count) *count = n;
        if (stats) {
            stats[0] = st.mean;
            stats[1] = st.thresh;
            stats[2] = st.var;
            stats[3] = st.m2;
        }
    }
    if (indices && warp < 4) {
        // The reference's list order: stripe class 0 ascending, then 1, 2, 3.
        int before = 0;
        for (int i = lane; i < n; i += 32)
            before += ((static_cast<int>(list[i] & 0xFFFFu) >> 5) & 3) < warp ? 1 : 0;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) before += __shfl_xor_sync(0xffffffffu, before, o);
        int pos = before;
        for (int base = 0; base < n; base += 32) {
            const int i = base + lane;
            const int c = (i < n) ? static_cast<int>(list[i] & 0xFFFFu) : 0;
            const bool mine = i < n && ((c >> 5) & 3) == warp;
            const unsigned bal = __ballot_sync(0xffffffffu, mine);
            if (mine) indices[pos + __popc(bal & ((1u << lane) - 1u))] = c;
            pos += __popc(bal);
        }
    }
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
constexpr int kNumKernels = 528;
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
    // all of the unified L1 / shared memory as shared memory (two 113 KB CTAs per SM)
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
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


template <bool kSplit, bool kNative, int kOut, int kW, int kR, bool kGather = false, bool kSlab = false>
dq_status_t launch_b1(const B1Args& a, int grid, cudaStream_t stream) {
    constexpr int wi = kW == kB1Warps ? 0 : 1;
    constexpr int ri = kR == 1 ? 0 : kR == 2 ? 1 : kR == 4 ? 2 : 3;
    constexpr int id = 4 + 16 * (4 * wi + ri) + (kSplit ? 8 : 0) + (kNative ? 4 : 0) + kOut + (kGather ? 128 : 0) +
                       (kSlab ? 256 : 0);
    static_assert(id < kNumKernels, "kernel attribute slot");
    const dq_status_t st = ensure_smem(b1_kernel<kSplit, kNative, kOut, kW, kR, kGather, kSlab>, id, a.S.total);
    if (st != DQ_OK) return st;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kW * 32);
    cfg.dynamicSmemBytes = a.S.total;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, b1_kernel<kSplit, kNative, kOut, kW, kR, kGather, kSlab>, a);
    if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
    return check_launch();
}

template <bool kNative, int kW, int kR, bool kSlab = false>
dq_status_t launch_b1_out(const B1Args& a, int out_mode, int grid, cudaStream_t stream) {
    switch (out_mode) {
        case kOutStaged: return launch_b1<true, kNative, kOutStaged, kW, kR, false, kSlab>(a, grid, stream);
        case kOutColDirect: return launch_b1<true, kNative, kOutColDirect, kW, kR, false, kSlab>(a, grid, stream);
        case kOutRowDirect: return launch_b1<true, kNative, kOutRowDirect, kW, kR, false, kSlab>(a, grid, stream);
        default: return launch_b1<false, kNative, kOutNone, kW, kR, false, kSlab>(a, grid, stream);
    }
}

template <int kW>
dq_status_t launch_b1_native(const B1Args& a, int out_mode, int rounds, int grid, cudaStream_t stream) {
    if (a.nslab > 1)  // column slabs: at most 4 rounds (b1_setup)
        return rounds <= 2 ? launch_b1_out<true, kW, 2, true>(a, out_mode, grid, stream)
                           : launch_b1_out<true, kW, 4, true>(a, out_mode, grid, stream);
    if (rounds <= 1) return launch_b1_out<true, kW, 1>(a, out_mode, grid, stream);
    if (rounds <= 2) return launch_b1_out<true, kW, 2>(a, out_mode, grid, stream);
    if (rounds <= 4) return launch_b1_out<true, kW, 4>(a, out_mode, grid, stream);
    return launch_b1_out<true, kW, plan_rounds_max<kW>()>(a, out_mode, grid, stream);
}

// The gathering split GEMV: native layout, staged outlier columns (the
// slices are whole row blocks, so d_out is a multiple of 16).
template <int kW>
dq_status_t launch_b1_gather(const B1Args& a, int rounds, int grid, cudaStream_t stream) {
    if (a.nslab > 1)
        return rounds <= 2 ? launch_b1<true, true, kOutStaged, kW, 2, true, true>(a, grid, stream)
                           : launch_b1<true, true, kOutStaged, kW, 4, true, true>(a, grid, stream);
    if (rounds <= 1) return launch_b1<true, true, kOutStaged, kW, 1, true>(a, grid, stream);
    if (rounds <= 2) return launch_b1<true, true, kOutStaged, kW, 2, true>(a, grid, stream);
    if (rounds <= 4) return launch_b1<true, true, kOutStaged, kW, 4, true>(a, grid, stream);
    return launch_b1<true, true, kOutStaged, kW, plan_rounds_max<kW>(), true>(a, grid, stream);
}

dq_status_t launch_b1_warps(const B1Args& a, int warps, int out_mode, int rounds, int grid, cudaStream_t stream) {
    if (!a.native)
        return warps == kB1Warps
                   ? launch_b1_out<false, kB1Warps, plan_rounds_max<kB1Warps>()>(a, out_mode, grid, stream)
                   : launch_b1_out<false, kB1WarpsSmall, plan_rounds_max<kB1WarpsSmall>()>(a, out_mode, grid, stream);
    return warps == kB1Warps ? launch_b1_native<kB1Warps>(a, out_mode, rounds, grid, stream)
                             : launch_b1_native<kB1WarpsSmall>(a, out_mode, rounds, grid, stream);
}

// Launch geometry of one batch-1 call.
struct B1Plan {
    int grid, warps, out_mode, rounds;
};

dq_status_t b1_setup(const dq_weights_t& w, const uint16_t* x, uint16_t* y, float k, bool split, void* workspace,
                     size_t workspace_bytes, B1Args& a, B1Plan& p) {
    DeviceInfo di;
    const dq_status_t st = device_info(&di);
    if (st != DQ_OK) return st;
    const int G = w.d_in / kGroup;
    const long long n_rb = (static_cast<long long>(w.d_out) + kRowBlock - 1) / kRowBlock;
    const int NC = (G + kCG - 1) / kCG;
    if (n_rb * NC > INT_MAX) return DQ_ERR_UNSUPPORTED;
    a = B1Args{};
    a.packed = w.packed;
    a.scales = w.scales;
    a.zeros = w.zeros;
    a.native = w.native;
    a.w16 = w.fp16;
    a.w16_cm = w.fp16_cm;
    a.x = x;
    a.y = y;
    a.k = k;
    a.inv_n = 1.0f / static_cast<float>(w.d_in);
    a.inv_n1 = w.d_in > 1 ? 1.0f / static_cast<float>(w.d_in - 1) : 0.f;
    a.d_out = w.d_out;
    a.d_in = w.d_in;
    a.NC = NC;
    const WsLayout W = ws_layout(w.d_out, w.d_in);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    a.hdr = reinterpret_cast<unsigned int*>(ws + W.hdr);
    a.fix = reinterpret_cast<unsigned long long*>(ws + W.fix);
    a.xsl = reinterpret_cast<unsigned long long*>(ws + ws_slab_offset());
    int grid = di.sm_count < n_rb * NC ? di.sm_count : static_cast<int>(n_rb * NC);
    if (grid > kMaxCtas) grid = kMaxCtas;
    // Column slabs for long rows (native layout): every slab's CTAs then
    // cover all row blocks over fewer chunks, so a CTA's plan converts only
    // its slab of x.  Not when the workspace has no room for the slab words,
    // a slab would get fewer than two CTAs, a slab's plan would take more
    // than 4 rounds, or a CTA's share is long (the plan is then a small part
    // of it).
    int nslab = w.native ? b1_slabs(NC) : 1;
    if (nslab > 1) {
        const int ncs = NC / nslab;
        const long long per_cta = (n_rb * NC + grid - 1) / grid;
        if (grid < 2 * nslab || 64 * ncs > 4 * 32 * kB1WarpsSmall || per_cta > kB1SlabMaxUnits ||
            workspace_bytes < ws_slab_offset() + b1_slab_bytes(w.d_out, nslab))
            nslab = 1;
    }
    a.nslab = nslab;
    a.NCs = NC / nslab;
    a.U = static_cast<int>(n_rb * a.NCs);
    int nrb_max = 1;
    for (int sl = 0; sl < nslab; ++sl) {
        const int c0 = sl * grid / nslab, P = (sl + 1) * grid / nslab - c0;
        for (int c = 0; c < P; ++c) {
            const int u0 = unit_start(a.U, c, P), u1 = unit_start(a.U, c + 1, P);
            if (u1 <= u0) continue;
            const int n = (u1 - 1) / a.NCs - u0 / a.NCs + 1;
            if (n > nrb_max) nrb_max = n;
        }
    }
    a.nrb_max = nrb_max;
    const int slab_nc = nslab > 1 ? a.NCs : 0;
    p.grid = grid;
    p.out_mode = kOutNone;
    if (split) p.out_mode = w.fp16_cm ? ((w.d_out % 8) == 0 ? kOutStaged : kOutColDirect) : kOutRowDirect;
    if (w.native) {
        // A ring of as many stages per warp as fit (at least kB1Stages, no more
        // than a warp has units), 16 warps or 12.
        const int per_cta = nslab > 1 ? (a.U + grid / nslab - 1) / (grid / nslab) : (a.U + grid - 1) / grid;
        const int u_warp = (per_cta + kB1WarpsSmall - 1) / kB1WarpsSmall;
        const int ring_warps[2] = {kB1Warps, kB1WarpsSmall};
        for (int warps : ring_warps) {
            for (int depth = kB1MaxDepth; depth >= kB1Stages; --depth) {
                if (depth > kB1Stages && depth > u_warp) continue;
                a.S = b1_smem(w.d_in, nrb_max, split, warps, warps * depth, slab_nc);
                if (a.S.total > di.smem_optin) continue;
                a.depth = depth;
                p.warps = warps;
                p.rounds = (64 * a.NCs + 32 * warps - 1) / (32 * warps);  // plan rounds: pieces per thread
                return DQ_OK;
            }
        }
        return DQ_ERR_UNSUPPORTED;
    }
    // Reference layout: kB1Stages per warp, 16 warps where their rings fit next
    // to x and the plan, else 12.
    a.depth = kB1Stages;
    p.warps = kB1Warps;
    a.S = b1_smem(w.d_in, nrb_max, split, p.warps, p.warps * kB1Stages);
    if (a.S.total > di.smem_optin) {
        p.warps = kB1WarpsSmall;
        a.S = b1_smem(w.d_in, nrb_max, split, p.warps, p.warps * kB1Stages);
    }
    if (a.S.total > di.smem_optin) return DQ_ERR_UNSUPPORTED;
    p.rounds = (64 * NC + 32 * p.warps - 1) / (32 * p.warps);
    return DQ_OK;
}

}  // namespace

size_t b1_workspace_bytes(int d_out, int d_in) {
    const int NC = (d_in / kGroup + kCG - 1) / kCG;
    const int S = b1_slabs(NC);
    return S > 1 ? ws_slab_offset() + b1_slab_bytes(d_out, S) : ws_layout(d_out, d_in).total;
}

dq_status_t launch_gemv_b1(const dq_weights_t& w, const uint16_t* x, uint16_t* y, float k,
                           bool split, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
    B1Args a;
    B1Plan p;
    const dq_status_t st = b1_setup(w, x, y, k, split, workspace, workspace_bytes, a, p);
    if (st != DQ_OK) return st;
    return launch_b1_warps(a, p.warps, p.out_mode, p.rounds, p.grid, stream);
}

dq_status_t launch_gemv_b1_gather(const dq_weights_t& w, const uint16_t* x, uint16_t* y, float k, void* workspace,
                                  size_t workspace_bytes, const dq_gather_t& g, cudaStream_t stream) {
    B1Args a;
    B1Plan p;
    const dq_status_t st = b1_setup(w, x, y, k, true, workspace, workspace_bytes, a, p);
    if (st != DQ_OK) return st;
    if (!a.native || p.out_mode != kOutStaged) return DQ_ERR_UNSUPPORTED;
    a.g_rank = g.rank;
    a.g_world = g.world;
    a.g_rows_per = g.rows_per;
    a.g_total = g.d_total;
    for (int q = 0; q < kMaxGatherRanks; ++q)
        a.g_region[q] = q < g.world ? static_cast<uint8_t*>(g.region[q]) : nullptr;
    a.g_lay = gather_layout(g.rows_per);
    return p.warps == kB1Warps ? launch_b1_gather<kB1Warps>(a, p.rounds, p.grid, stream)
                               : launch_b1_gather<kB1WarpsSmall>(a, p.rounds, p.grid, stream);
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
    const int smem = detect_smem(d_in).total;
    if (smem > di.smem_optin) return DQ_ERR_UNSUPPORTED;
    const dq_status_t s2 = ensure_smem(detect_kernel, 1, smem);
    if (s2 != DQ_OK) return s2;
    detect_kernel<<<1, kStatThreads, smem, stream>>>(x, d_in, k, 1.0f / static_cast<float>(d_in),
                                            d_in > 1 ? 1.0f / static_cast<float>(d_in - 1) : 0.f, mask_words,
                                            indices, count, stats);
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
    const dim3 grid(d_in / 64, (d_out + 63) / 64);
    colmajor_kernel<<<grid, 256, 0, stream>>>(w16, d_out, d_in, cm);
    return check_launch();
}

}  // namespace dq
