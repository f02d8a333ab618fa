// dq_batched.cu -- the split GEMV for a batch of 1 <= M <= 16 activation
// vectors on sm_100a: y[m] = split_gemv(W, x[m], k) for every m, i.e. the
// reference's batch-1 split GEMV (src/split_gemv.cu:25-198 of dyn-quant)
// applied to each vector with its own statistics and outlier mask, while the
// weights stream from HBM once for all vectors.
//
// Three kernels, chained on the stream by programmatic dependent launch:
//  1. bplan_kernel, one CTA per vector: the statistics and the outlier mask
//     of x[m], with the code and the fixed partition of the batch-1 kernel
//     (dq_plan.cuh), so each vector gets exactly the batch-1 mask; the CTA
//     writes its vector's outlier-only row (x[m][c] where c is an outlier of
//     m, else 0) and its share of the x' tables (the MMA B operands of every
//     chunk, outliers zeroed, and the per-group sums).
//  2. bdense_kernel: the INT4 part over x', split over K: CTA (cx, slab)
//     copies its slab's x' tables in with two bulk copies and streams chunks
//     [slab S, slab S + S) of the row blocks [rb0, rb1) through per-warp
//     cp.async.bulk rings.  Each warp owns whole row blocks and writes its
//     slab's partial sums.  While the tables arrive, every CTA derives the
//     union of the M masks (ascending columns) and gathers its share of the
//     union's columns of the outlier-only rows into x_o[u][m], one union
//     column's vectors contiguous.
//  3. bout_kernel, one CTA per 16-row block: the FP16 part,
//     Y_o = W16[:, union] x_o, on the tensor cores, then y = the slabs'
//     partial sums + Y_o, in a fixed order (results do not depend on timing).
//     Each warp takes every eighth 16-column batch of the union; the A
//     segments (16 rows of a column, contiguous in the column-major mirror)
//     and the B segments (the column's x_o values) come in by 16-byte cp.async
//     and ldmatrix.trans; the eight warps' sums are added in a fixed order.
//     Its CTAs start as the dense kernel's CTAs drain (those hold all of an
//     SM's registers), after the dense kernel has completed.
//
// Tensor-core formulation of the INT4 part (mma.sync.m16n8k16, f16 x f16 ->
// f32; 16 weight rows x 8 vectors x 16 columns of one 128-column group).
// ldmatrix over the native unit layout gives lane (g, t) word t of the pieces
// of group j at slices 0..3 for rows g and g + 8 (columns 32 sl + 8 t ..
// 32 sl + 8 t + 7 of the group).  A holds the codes as exact FP16 integers
// (q for even columns, 16 q for odd columns: the exponent-bias trick, then the
// bias subtracted); B is x' of vector g in the same column order, from a
// per-CTA table.  Per group and vector:
//   D_lo = sum_even q x'        D_hi = 16 sum_odd q x'
//   y += s (D_hi / 16 + D_lo - z X)
// which is the reference's sum over the group of s (q - z) x'.
#include <algorithm>

#include "dq_common.cuh"
#include "dq_internal.h"
#include "dq_plan.cuh"

namespace dq {

namespace {

// Set by a batched kernel whose bounded wait on its own copies gave up.
__device__ unsigned int g_berror_word;

constexpr int kUnit = kB1UnitBytes;

// The arguments of NG problems of one launch (NG = 1: a plain batched call;
// NG > 1: a grouped call, problem g in blockIdx.y (plan, FP16 part) or
// blockIdx.z (INT4 part)).
template <class A, int NG>
struct Group {
    A p[NG];
};

// The codes of a word as exact FP16 integers: q for the even columns, 16 q for
// the odd ones (the exponent-biased values with the bias 1024 taken off, one
// exact HSUB2 per register).  Without the bias the MMA sums q x' directly:
// with large activations (the gated activations of an MoE expert run into
// the hundreds) a sum that carries 1024 X loses low bits in the tensor core's
// accumulation.
__device__ __forceinline__ Biased4 exact_word(uint32_t w) {
    constexpr uint32_t kMagic = 0x64006400u;
    Biased4 r = biased_word(w);
    r.lo0 = hsub2_u32(r.lo0, kMagic);
    r.lo1 = hsub2_u32(r.lo1, kMagic);
    r.hi0 = hsub2_u32(r.hi0, kMagic);
    r.hi1 = hsub2_u32(r.hi1, kMagic);
    return r;
}

__device__ __forceinline__ float4 lds_f4(uint32_t addr) {
    const uint4 v = lds_v4(addr);
    return make_float4(__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z), __uint_as_float(v.w));
}

// ---------------------------------------------------------------------------
// 1. Plan: statistics, masks, x' tables
// ---------------------------------------------------------------------------
struct BPSmem {
    int xs, mask, red, total;
};

inline BPSmem bp_smem(int d_in) {
    BPSmem S;
    int off = 0;
    S.xs = off;   off += align16(2 * d_in);
    S.mask = off; off += align16(d_in / 8);
    S.red = off;  off += kB1RedBytes;
    S.total = off;
    return S;
}

struct BPArgs {
    const uint16_t* x;   // [M][d_in]
    uint32_t* masks;     // [kBgMaxM][W]
    uint16_t* xrow;      // [MP][d_in] outlier-only rows (rows m < M)
    uint4* xtab;         // [NC][4 groups][4 slices][MP][4] the INT4 part's B operands
    float4* xsum;        // [NC][4 groups][MP] per-group sums of x'
    float k, inv_n, inv_n1;
    int M, MP, d_in, W, NC;
    BPSmem S;
};

// One CTA per vector slot m < MP.  For m < M: the statistics and the outlier
// mask of x[m] with the code and the fixed partition of the batch-1 kernel
// (dq_plan.cuh), so each vector gets exactly the batch-1 mask; the vector's
// outlier-only row (x[m][c] where c is an outlier of m, else 0); and the
// vector's share of the x' tables that every INT4-part CTA copies in whole:
// piece p (8 columns) of chunk cc goes to xtab[cc][group][slice][m][p & 3] as
// the f16 pairs (x0,x4), (x2,x6), (x1,x5), (x3,x7) of x' (x with m's outliers
// zeroed), and xsum[cc][group][m] = (1024 sum x' even columns, 1024 sum x' odd
// columns, sum x', 0).  For M <= m < MP (padding of the last 8-vector tile):
// zeros in the tables.
template <int NG>
__global__ void __launch_bounds__(kStatThreads, 1) bplan_kernel(const Group<BPArgs, NG> grp) {
    const BPArgs& a = grp.p[NG == 1 ? 0 : blockIdx.y];
    constexpr int NT = kStatThreads;
    extern __shared__ __align__(128) char smem[];
    uint4* xs = reinterpret_cast<uint4*>(smem + a.S.xs);
    uint32_t* mask32 = reinterpret_cast<uint32_t*>(smem + a.S.mask);
    float* red = reinterpret_cast<float*>(smem + a.S.red);
    const int m = blockIdx.x, tid = threadIdx.x;
    const int n8 = a.d_in >> 3;
    const int npc = a.NC * 64;  // pieces of the tables: whole 512-column chunks
    auto tab = [&](int p) -> uint4* {
        const int cc = p >> 6, q = p & 63;
        return a.xtab + ((((cc * 4 + (q >> 4)) * 4 + ((q >> 2) & 3)) * a.MP + m) * 4 + (q & 3));
    };
    auto sum_of = [&](int p) -> float4* { return a.xsum + ((p >> 4) * a.MP + m); };

    pdl_launch_dependents();
    pdl_wait();  // x and the workspace may belong to the preceding kernel until here
    if (m >= a.M) {
        for (int p = tid; p < npc; p += NT) {
            *tab(p) = make_uint4(0, 0, 0, 0);
            if ((p & 15) == 0) *sum_of(p) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        return;
    }
    load_x_async<NT>(a.x + static_cast<size_t>(m) * a.d_in, n8, xs);
    cp_async_wait_all();
    __syncthreads();
    const XStats st = x_stats<NT>(xs, n8, a.d_in, a.k, a.inv_n, a.inv_n1, red);
    x_mask_list<NT>(xs, a.d_in, st.mean, st.thresh, mask32, nullptr,
                    reinterpret_cast<int*>(red) + 2 * (kStatThreads / 32));
    __syncthreads();
    for (int i = tid; i < a.W; i += NT) a.masks[static_cast<size_t>(m) * a.W + i] = mask32[i];
    // npc is a multiple of 64 and NT of 32: a warp's 32 pieces are all below
    // npc or all above, and a half-warp holds the 16 pieces of one group.
    const uint8_t* mb = reinterpret_cast<const uint8_t*>(mask32);
    for (int p = tid; p < npc; p += NT) {
        const uint4 w = p < n8 ? xs[p] : make_uint4(0, 0, 0, 0);
        const uint32_t b = p < n8 ? mb[p] : 0u;
        uint32_t keep[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
            keep[i] = ((b >> (2 * i)) & 1u ? 0x0000FFFFu : 0u) | ((b >> (2 * i + 1)) & 1u ? 0xFFFF0000u : 0u);
        if (p < n8)
            *reinterpret_cast<uint4*>(a.xrow + static_cast<size_t>(m) * a.d_in + 8 * p) =
                make_uint4(w.x & keep[0], w.y & keep[1], w.z & keep[2], w.w & keep[3]);
        const uint4 v = make_uint4(w.x & ~keep[0], w.y & ~keep[1], w.z & ~keep[2], w.w & ~keep[3]);
        float pe = add_f16_f32(lo16(v.w), add_f16_f32(lo16(v.z), add_f16_f32(lo16(v.y), add_f16_f32(lo16(v.x), 0.f))));
        float po = add_f16_f32(hi16(v.w), add_f16_f32(hi16(v.z), add_f16_f32(hi16(v.y), add_f16_f32(hi16(v.x), 0.f))));
        *tab(p) = make_uint4((v.x & 0xFFFFu) | (v.z << 16), (v.y & 0xFFFFu) | (v.w << 16),
                             (v.x >> 16) | (v.z & 0xFFFF0000u), (v.y >> 16) | (v.w & 0xFFFF0000u));
#pragma unroll
        for (int o = 8; o >= 1; o >>= 1) {
            pe += __shfl_xor_sync(0xffffffffu, pe, o);
            po += __shfl_xor_sync(0xffffffffu, po, o);
        }
        if ((p & 15) == 0) *sum_of(p) = make_float4(1024.f * pe, 1024.f * po, pe + po, 0.f);
    }
}

// ---------------------------------------------------------------------------
// 1b. Union of the masks and the outlier columns' x (run by the INT4-part CTAs)
// ---------------------------------------------------------------------------
struct BUArgs {
    const uint32_t* masks;  // [kBgMaxM][W]
    const uint16_t* xrow;   // [MP][d_in] outlier-only rows (rows m < M)
    uint16_t* ulist;        // [d_in] union columns, ascending
    uint16_t* xo;           // [d_in rounded up to 16][MP] by union position
    unsigned int* ctr;      // [1] union size
    int M, MP, d_in, W;
};

// CTA b of G: derives the union of the M masks and its prefix (ascending
// columns) itself, then takes the union positions [U b / G, U (b + 1) / G):
// their columns into ulist and xo[u][m] = xrow[m][column] (zero for the
// padding vectors m >= M); CTA G - 1 also zeroes the positions
// U .. (U rounded up to 16) - 1, and CTA 0 stores U.  NT threads, all of them
// calling; barrier-synchronised.  scratch: NT / 32 ints; pcol: kBuMaxPos u16.
template <int NT>
__device__ void union_share(const BUArgs& a, int b, int G, int* scratch, uint16_t* pcol) {
    constexpr int kWq = (kMaxDIn / 32 + NT - 1) / NT;  // mask words per thread at most
    const int tid = threadIdx.x;
    const int w0 = static_cast<int>(static_cast<long long>(tid) * a.W / NT);
    const int w1 = static_cast<int>(static_cast<long long>(tid + 1) * a.W / NT);
    uint32_t u[kWq];
    int cnt[1] = {0};
#pragma unroll
    for (int q = 0; q < kWq; ++q) {
        const int wj = w0 + q;
        u[q] = 0u;
        if (wj < w1) {
            uint32_t v[kBgMaxM];  // every vector's word in flight at once
#pragma unroll
            for (int mm = 0; mm < kBgMaxM; ++mm)
                v[mm] = mm < a.M ? ldcg_u32(a.masks + static_cast<size_t>(mm) * a.W + wj) : 0u;
#pragma unroll
            for (int mm = 0; mm < kBgMaxM; ++mm) u[q] |= v[mm];
            cnt[0] += __popc(u[q]);
        }
    }
    int pre[1], tot[1];
    block_scan<NT, 1>(cnt, pre, tot, scratch);
    const int U = tot[0];
    const int lo = static_cast<int>(static_cast<long long>(U) * b / G);
    const int hi = static_cast<int>(static_cast<long long>(U) * (b + 1) / G);
    if (b == 0 && tid == 0) a.ctr[1] = static_cast<unsigned>(U);
    // The share in windows of kBuMaxPos positions: their columns into pcol
    // (by the threads owning their mask words), then the gather by all.
    for (int wlo = lo; wlo < hi; wlo += kBuMaxPos) {
        const int whi = min(hi, wlo + kBuMaxPos);
        int pos = pre[0];
#pragma unroll
        for (int q = 0; q < kWq; ++q) {
            uint32_t rest = u[q];
            while (rest && pos < whi) {
                const int col = 32 * (w0 + q) + __ffs(rest) - 1;
                if (pos >= wlo) {
                    pcol[pos - wlo] = static_cast<uint16_t>(col);
                    a.ulist[pos] = static_cast<uint16_t>(col);
                }
                ++pos;
                rest &= rest - 1u;
            }
        }
        __syncthreads();
        const int n = whi - wlo;
        for (int i = tid; i < n * a.MP; i += NT) {
            const int p = i / a.MP, mm = i - p * a.MP;
            const uint16_t v = mm < a.M ? ldcg_u16(a.xrow + static_cast<size_t>(mm) * a.d_in + pcol[p]) : uint16_t{0};
            a.xo[static_cast<size_t>(wlo + p) * a.MP + mm] = v;
        }
        __syncthreads();  // pcol is rewritten by the next window
    }
    if (b == G - 1) {
        const int upad = (U + 15) & ~15;
        for (int i = tid; i < (upad - U) * a.MP; i += NT) a.xo[static_cast<size_t>(U) * a.MP + i] = 0;
    }
}

// ---------------------------------------------------------------------------
// 2. FP16 part over the union's columns
// ---------------------------------------------------------------------------
// How the FP16 weights of the union's columns are read (as in the batch-1 kernel).
enum : int {
    kBoStaged = 0,     // column-major mirror, d_out % 8 == 0: 16-byte cp.async per lane
    kBoColDirect = 1,  // column-major mirror, other d_out: plain loads
    kBoRowDirect = 2,  // row-major FP16 only: plain loads
};

struct BOArgs {
    const uint16_t* w16;     // row-major FP16 [d_out][d_in]
    const uint16_t* w16_cm;  // column-major mirror [d_in][d_out]
    const uint16_t* ulist;   // [d_in] union columns, ascending
    const uint16_t* xo;      // [d_in][MP] by union position
    const unsigned int* ctr;
    const float* dpart;      // [nslab][MP][d_out] the INT4 part's partial sums
    uint16_t* y;             // [M][d_out]
    int d_out, d_in, MP, M, nslab;
};

// One CTA per RB consecutive 16-row blocks (RB = 1, 2 or 4: column segments
// of 32 RB contiguous bytes in the column-major mirror).  Dynamic shared
// memory: per warp kBgOutBufs buffers of [16 columns x 16 RB rows of W16 |
// 16 columns x 16 vectors of x_o], then the union's columns (2 bytes each,
// room for d_in), copied in at the start, so that no copy of a column segment
// waits on a load of its column index.  After the loop the buffers hold the
// warps' sums.
template <int RB>
__host__ __device__ constexpr int bout_buf_bytes() { return RB * 512 + 512; }
template <int RB>
inline int bout_smem(int d_in) { return kBgOutWarps * kBgOutBufs * bout_buf_bytes<RB>() + align16(2 * d_in) + 16; }

template <int kOut, int NT, int RB, int NG>
__global__ void __launch_bounds__(kBgOutWarps * 32) bout_kernel(const Group<BOArgs, NG> grp) {
    const BOArgs& a = grp.p[NG == 1 ? 0 : blockIdx.y];
    constexpr int MP = 8 * NT;
    constexpr int kBuf = bout_buf_bytes<RB>();
    constexpr int kA = RB * 512;  // A part of a buffer: column ci's RB * 16 rows at ci * 32 RB
    static_assert(kBgOutWarps * RB * NT * 4 * 32 * 4 <= kBgOutWarps * kBgOutBufs * kBuf, "warp sums in the buffers");
    extern __shared__ __align__(128) unsigned char osm[];
    uint16_t* ucol = reinterpret_cast<uint16_t*>(osm + kBgOutWarps * kBgOutBufs * kBuf);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int rb0 = blockIdx.x * RB;

    // The union and x_o come from the INT4-part kernel's CTAs (which hold all
    // of the SMs' registers, so this grid's CTAs start as they drain).
    pdl_launch_dependents();
    pdl_wait();
    const int U = static_cast<int>(ldcg_u32(a.ctr + 1));
    for (int i = threadIdx.x; 8 * i < U; i += kBgOutWarps * 32)
        reinterpret_cast<uint4*>(ucol)[i] = ldcg_v4(a.ulist + 8 * i);
    __syncthreads();
    const int nbat = (U + 15) / 16;
    const int nb = warp < nbat ? (nbat - warp + kBgOutWarps - 1) / kBgOutWarps : 0;  // batches warp, warp + 8, ...
    const uint32_t wbase = smem_u32(osm) + warp * kBgOutBufs * kBuf;

    // Batch k of this warp into buffer k % kBgOutBufs.  A: 16 columns x 2 RB
    // pieces of 8 rows, piece i = lane + 32 j -> column i / (2 RB), rows
    // 8 (i % (2 RB)) ..; B: lane = (column lane >> 1, half lane & 1), 8
    // vectors of x_o.
    auto issue = [&](int k) {
        const int kb = 16 * (warp + kBgOutWarps * k);
        const uint32_t buf = wbase + (k % kBgOutBufs) * kBuf;
#pragma unroll
        for (int j = 0; j < RB; ++j) {
            const int i = lane + 32 * j;
            const int ci = i / (2 * RB), pi = i % (2 * RB);
            const int kc = kb + ci;
            const int row0 = rb0 * kRowBlock + 8 * pi;
            const uint32_t da = buf + ci * (32 * RB) + 16 * pi;
            const bool valid = kc < U;
            const int col = valid ? static_cast<int>(ucol[kc]) : 0;
            if (kOut == kBoStaged) {
                if (valid && row0 < a.d_out) cp_async16(da, a.w16_cm + static_cast<size_t>(col) * a.d_out + row0);
                else sts_v4(da, make_uint4(0, 0, 0, 0));
            } else {
                uint16_t h[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const int r = row0 + e;
                    h[e] = (valid && r < a.d_out)
                               ? (kOut == kBoColDirect ? ldg_u16(a.w16_cm + static_cast<size_t>(col) * a.d_out + r)
                                                       : ldg_u16(a.w16 + static_cast<size_t>(r) * a.d_in + col))
                               : static_cast<uint16_t>(0);
                }
                sts_v4(da, make_uint4(pack_h2(h[0], h[1]), pack_h2(h[2], h[3]), pack_h2(h[4], h[5]),
                                      pack_h2(h[6], h[7])));
            }
        }
        {
            const int kc = kb + (lane >> 1), half = lane & 1;
            const uint32_t db = buf + kA + 16 * lane;
            if (kc < ((U + 15) & ~15) && (MP == 16 || half == 0))
                cp_async16(db, a.xo + static_cast<size_t>(kc) * MP + 8 * half);
            else sts_v4(db, make_uint4(0, 0, 0, 0));
        }
        cp_async_commit();
    };
    float d[RB][NT][4];
#pragma unroll
    for (int r = 0; r < RB; ++r)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) d[r][nt][0] = d[r][nt][1] = d[r][nt][2] = d[r][nt][3] = 0.f;
    for (int k = 0; k < kBgOutBufs && k < nb; ++k) issue(k);
    for (int k = 0; k < nb; ++k) {
        if (k + 2 < nb) cp_async_wait_group<2>();
        else if (k + 1 < nb) cp_async_wait_group<1>();
        else cp_async_wait_group<0>();
        __syncwarp();
        const uint32_t ab = wbase + (k % kBgOutBufs) * kBuf, bb = ab + kA;
        // B: matrix j = (column half j & 1, vector half j >> 1); rows are columns (32 bytes each)
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(bb + ((((lane >> 3) & 1) * 8 + (lane & 7)) * 32) + (lane >> 4) * 16, b0, b1, b2, b3);
#pragma unroll
        for (int r = 0; r < RB; ++r) {
            // A of row block r: matrix j = (column half j >> 1, row half j & 1);
            // lane 8j + i gives column (j >> 1) * 8 + i
            uint32_t a0, a1, a2, a3;
            ldmatrix_x4_trans(ab + ((lane >> 4) * 8 + (lane & 7)) * (32 * RB) + 32 * r + ((lane >> 3) & 1) * 16,
                              a0, a1, a2, a3);
            mma_16816(d[r][0], a0, a1, a2, a3, b0, b1);
            if (NT == 2) mma_16816(d[r][NT - 1], a0, a1, a2, a3, b2, b3);
        }
        __syncwarp();  // every lane is done with the buffers before they are refilled
        if (k + kBgOutBufs < nb) issue(k + kBgOutBufs);
    }
    cp_async_wait_group<0>();
    __syncthreads();  // every warp is done with its buffers: they take the warps' sums
    float* red = reinterpret_cast<float*>(osm);  // [warp][r][nt][4][32]
#pragma unroll
    for (int r = 0; r < RB; ++r)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) red[(((warp * RB + r) * NT + nt) * 4 + e) * 32 + lane] = d[r][nt][e];
    __syncthreads();
    // The warps' sums in warp order, then the INT4 part's slabs in order.
    for (int i = threadIdx.x; i < RB * NT * 4 * 32; i += kBgOutWarps * 32) {
        const int r = i / (NT * 128), nt = (i >> 7) % NT, e = (i >> 5) & 3, ln = i & 31;
        const int row = (rb0 + r) * kRowBlock + (ln >> 2) + 8 * (e >> 1);
        const int tok = nt * 8 + 2 * (ln & 3) + (e & 1);
        if (row >= a.d_out || tok >= a.M) continue;
        float v = 0.f;
        for (int s0 = 0; s0 < a.nslab; s0 += 4) {
            float q[4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
                q[j] = s0 + j < a.nslab
                           ? ldcg_f32(a.dpart + (static_cast<size_t>(s0 + j) * MP + tok) * a.d_out + row) : 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) v += q[j];
        }
        float o = 0.f;
#pragma unroll
        for (int w = 0; w < kBgOutWarps; ++w) o += red[(((w * RB + r) * NT + nt) * 4 + e) * 32 + ln];
        a.y[static_cast<size_t>(tok) * a.d_out + row] = __half_as_ushort(__float2half_rn(v + o));
    }
}

// ---------------------------------------------------------------------------
// 3. INT4 part, split over K, and the final sums
// ---------------------------------------------------------------------------
struct BDArgs {
    const uint8_t* native;   // unit layout
    const uint4* xtab;       // [NC][4][4][MP][4] x' tables of the plan kernel
    const float4* xsum;      // [NC][4][MP]
    float* dpart;            // [nslab][MP][d_out]
    BUArgs un;               // the union and x_o, a share per CTA
    int M, d_out, d_in, NC, NRB, S, nslab, cps;
    int pf_rb;               // row blocks per warp (from its first) pulled into L2 before the plan is ready
    int sm_ring, sm_bars, sm_xtab, sm_xsum;
};

struct BDSmem {
    int ring, bars, xtab, xsum, total;
};

inline BDSmem bd_smem(int S, int MP) {
    BDSmem L;
    int off = 0;
    L.ring = off; off += kBgWarps * kBgStages * kUnit;
    L.bars = off; off += (kBgWarps * kBgStages * 8 + 8 + 127) / 128 * 128;  // + the tables' mbarrier
    L.xtab = off; off += S * MP * 1024;
    L.xsum = off; off += S * kB1ChunkGroups * MP * 16;
    L.total = off;
    return L;
}

template <int NT, int NG>
__global__ void __launch_bounds__(kBgWarps * 32, 1) bdense_kernel(const Group<BDArgs, NG> grp) {
    const BDArgs& a = grp.p[NG == 1 ? 0 : blockIdx.z];
    constexpr int MP = 8 * NT;
    extern __shared__ __align__(128) char smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int sb = blockIdx.y;
    const int c0 = sb * a.S, nch = min(a.S, a.NC - c0);
    const int rb0 = static_cast<int>(static_cast<long long>(a.NRB) * blockIdx.x / a.cps);
    const int rb1 = static_cast<int>(static_cast<long long>(a.NRB) * (blockIdx.x + 1) / a.cps);
    // Warp w owns the row blocks rb0 + w, rb0 + w + kBgWarps, ...; its units
    // are their nch chunks of this slab, row block by row block.
    const int nrw = (rb1 - rb0 > warp) ? (rb1 - rb0 - warp + kBgWarps - 1) / kBgWarps : 0;
    const int wn = nrw * nch;
    const uint32_t ring = smem_u32(smem + a.sm_ring) + warp * kBgStages * kUnit;
    const uint32_t bars = smem_u32(smem + a.sm_bars) + warp * kBgStages * 8;
    uint4* xtab = reinterpret_cast<uint4*>(smem + a.sm_xtab);
    float4* xsum = reinterpret_cast<float4*>(smem + a.sm_xsum);

    auto unit_of = [&](int j) -> long long {
        const int r = j / nch;
        return static_cast<long long>(rb0 + warp + kBgWarps * r) * a.NC + c0 + (j - r * nch);
    };
    auto issue = [&](int s, int j) {  // lane 0 only
        const uint32_t bar = bars + 8 * s;
        mbar_arrive_expect_tx(bar, kUnit);
        bulk_g2s(ring + s * kUnit, a.native + unit_of(j) * kUnit, kUnit, bar);
    };
    const uint32_t xbar = smem_u32(smem + a.sm_bars) + kBgWarps * kBgStages * 8;  // the x' tables

    // The weights do not depend on the preceding kernels: the first stages go
    // out before griddepcontrol.wait, and the warp's first pf_rb row blocks
    // (each one contiguous run of nch units) are pulled into L2 meanwhile, so
    // the stream runs while the plan kernels work.
    uint32_t armed = 0;
    if (tid == 0) mbar_init(xbar, 1);
    if (lane == 0) {
#pragma unroll
        for (int s = 0; s < kBgStages; ++s) mbar_init(bars + 8 * s, 1);
        fence_mbar_init();
#pragma unroll
        for (int s = 0; s < kBgStages; ++s)
            if (s < wn) issue(s, s);
        for (int r = 0; r < nrw && r < a.pf_rb; ++r)
            prefetch_l2_bulk(a.native + unit_of(r * nch) * kUnit, static_cast<uint32_t>(nch) * kUnit);
    }
#pragma unroll
    for (int s = 0; s < kBgStages; ++s)
        if (s < wn) armed |= 1u << s;
    __syncthreads();  // the tables' mbarrier is initialised

    pdl_wait();  // the x' tables, masks and rows come from the plan kernel
    pdl_launch_dependents();

    // This slab's x' tables (chunks c0 .. c0 + nch - 1 of every vector), built
    // once by the plan kernel: two bulk copies, in flight while the CTA does
    // its share of the union and x_o for the FP16-part kernel.
    if (tid == 0 && rb1 > rb0) {
        const uint32_t tb = static_cast<uint32_t>(nch) * MP * 1024, sb2 = static_cast<uint32_t>(nch) * 4 * MP * 16;
        mbar_arrive_expect_tx(xbar, tb + sb2);
        bulk_g2s(smem_u32(xtab), a.xtab + static_cast<size_t>(c0) * MP * 64, tb, xbar);
        bulk_g2s(smem_u32(xsum), a.xsum + static_cast<size_t>(c0) * 4 * MP, sb2, xbar);
    }
    {
        __shared__ int uscratch[kBgWarps];
        __shared__ uint16_t pcol[kBuMaxPos];
        union_share<kBgWarps * 32>(a.un, blockIdx.y * gridDim.x + blockIdx.x, gridDim.x * gridDim.y, uscratch, pcol);
    }
    if (rb1 <= rb0) return;  // no row blocks (no copies were issued)
    const bool xok = mbar_wait_bounded(xbar, 0u);

    const uint32_t xtab_a = smem_u32(xtab);
    const uint32_t xsum_a = smem_u32(xsum);
    const int lm = lane >> 3, lr = lane & 7;  // ldmatrix: this lane addresses row lr of matrix (slice) lm

    float yacc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) yacc[nt][0] = yacc[nt][1] = yacc[nt][2] = yacc[nt][3] = 0.f;

    // Row block rb done by this warp: its partial sums for this slab.
    auto finish_rb = [&](int rb) {
        float* dp = a.dpart + static_cast<size_t>(sb) * MP * a.d_out;
        const int row0 = rb * kRowBlock + g;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int row = row0 + 8 * (e >> 1);
                const int tok = nt * 8 + 2 * t + (e & 1);
                if (row < a.d_out) dp[static_cast<size_t>(tok) * a.d_out + row] = yacc[nt][e];
            }
    };

    bool ok = __all_sync(0xffffffffu, xok);
    if (!ok && lane == 0) atomicOr(&g_berror_word, 1u);
    uint32_t phase = 0;
    for (int j = 0; ok && j < wn; ++j) {
        const int s = j % kBgStages;
        const bool got = mbar_wait_bounded(bars + 8 * s, (phase >> s) & 1u);
        if (!__all_sync(0xffffffffu, got)) {
            ok = false;
            if (lane == 0) atomicOr(&g_berror_word, 1u);
            break;
        }
        phase ^= 1u << s;
        armed &= ~(1u << s);
        const int r = j / nch, cc = j - r * nch;
        const uint32_t st = ring + s * kUnit;
#pragma unroll
        for (int jg = 0; jg < kB1ChunkGroups; ++jg) {
            uint32_t w0[4], w1[4];  // [slice]: word t of the pieces of group jg, rows g and g + 8
            ldmatrix_x4(st + native_piece(lm, 0, lr, jg) * 16, w0[0], w0[1], w0[2], w0[3]);
            ldmatrix_x4(st + native_piece(lm, 1, lr, jg) * 16, w1[0], w1[1], w1[2], w1[3]);
            float dlo[NT][4], dhi[NT][4];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) dlo[nt][e] = dhi[nt][e] = 0.f;
#pragma unroll
            for (int sl = 0; sl < 4; ++sl) {
                const Biased4 qa = exact_word(w0[sl]);
                const Biased4 qb = exact_word(w1[sl]);
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    const uint4 b = lds_v4(xtab_a + ((((cc * 4 + jg) * 4 + sl) * MP + nt * 8 + g) * 4 + t) * 16);
                    mma_16816(dlo[nt], qa.lo0, qb.lo0, qa.lo1, qb.lo1, b.x, b.y);
                    mma_16816(dhi[nt], qa.hi0, qb.hi0, qa.hi1, qb.hi1, b.z, b.w);
                }
            }
            // (scale | zero << 16) of group jg, rows g and g + 8
            const uint32_t e0 = lds_u32(st + kB1UnitPacked + 16 * g + 4 * jg);
            const uint32_t e8 = lds_u32(st + kB1UnitPacked + 16 * (g + 8) + 4 * jg);
            const float s0 = h2f_bits(lo16(e0)), z0 = h2f_bits(hi16(e0));
            const float s8 = h2f_bits(lo16(e8)), z8 = h2f_bits(hi16(e8));
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const uint32_t xa_addr = xsum_a + ((cc * 4 + jg) * MP + nt * 8 + 2 * t) * 16;
                const float4 xa = lds_f4(xa_addr);       // vector nt*8 + 2t
                const float4 xb = lds_f4(xa_addr + 16);  // vector nt*8 + 2t + 1
                yacc[nt][0] = fmaf(s0, fmaf(-z0, xa.z, fmaf(dhi[nt][0], 0.0625f, dlo[nt][0])), yacc[nt][0]);
                yacc[nt][1] = fmaf(s0, fmaf(-z0, xb.z, fmaf(dhi[nt][1], 0.0625f, dlo[nt][1])), yacc[nt][1]);
                yacc[nt][2] = fmaf(s8, fmaf(-z8, xa.z, fmaf(dhi[nt][2], 0.0625f, dlo[nt][2])), yacc[nt][2]);
                yacc[nt][3] = fmaf(s8, fmaf(-z8, xb.z, fmaf(dhi[nt][3], 0.0625f, dlo[nt][3])), yacc[nt][3]);
            }
        }
        __syncwarp();  // every lane is done with the stage before it is refilled
        if (j + kBgStages < wn) {
            if (lane == 0) issue(s, j + kBgStages);
            armed |= 1u << s;
        }
        if (cc == nch - 1) {
            finish_rb(rb0 + warp + kBgWarps * r);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) yacc[nt][0] = yacc[nt][1] = yacc[nt][2] = yacc[nt][3] = 0.f;
        }
    }
    if (!ok) {
        // Do not leave copies in flight into shared memory this CTA is about to release.
        if (!xok) mbar_wait_bounded(xbar, 0u);
#pragma unroll
        for (int s = 0; s < kBgStages; ++s)
            if (armed & (1u << s)) mbar_wait_bounded(bars + 8 * s, (phase >> s) & 1u);
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
constexpr int kMaxDevices = 64;
constexpr int kNumKernels = 48;
int g_smem_set[kMaxDevices][kNumKernels];

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

// Every batched kernel is a programmatic dependent of its predecessor on the stream.
template <class K, class A>
dq_status_t launch_pdl(K kernel, dim3 grid, int threads, int smem, cudaStream_t stream, const A& args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
    return DQ_OK;
}

template <int kOut, int NT, int RB, int NG>
dq_status_t launch_bout_rb(const Group<BOArgs, NG>& g, int ng, cudaStream_t stream) {
    constexpr int rbi = RB == 1 ? 0 : RB == 2 ? 1 : 2;
    constexpr int id = 6 + ((2 * kOut + NT - 1) * 3 + rbi) * 2 + (NG == 1 ? 0 : 1);
    static_assert(id < kNumKernels, "kernel attribute slot");
    const BOArgs& a = g.p[0];
    const int smem = bout_smem<RB>(a.d_in);
    const dq_status_t st = ensure_smem(bout_kernel<kOut, NT, RB, NG>, id, smem);
    if (st != DQ_OK) return st;
    const int nrb = (a.d_out + kRowBlock - 1) / kRowBlock;
    return launch_pdl(bout_kernel<kOut, NT, RB, NG>, dim3((nrb + RB - 1) / RB, ng), kBgOutWarps * 32, smem, stream,
                      g);
}

// Row blocks per FP16-part CTA.  One 8-vector tile: as many as keep at least
// one CTA per SM (8192 x 8192 at M = 8: 35.8 -> 33.9 us per call with two;
// the MoE step 0.80 -> 0.72 ms).  Two tiles: one (at M = 16 two row blocks
// per CTA took the call from 36 to 45 us in back-to-back calls, though the
// kernel alone ran as fast).
template <int kOut, int NT, int NG>
dq_status_t launch_bout(const Group<BOArgs, NG>& g, int ng, int sm_count, cudaStream_t stream) {
    const long long ctas = static_cast<long long>((g.p[0].d_out + kRowBlock - 1) / kRowBlock) * ng;
    if constexpr (NT == 1) {
        if (ctas >= 4LL * sm_count) return launch_bout_rb<kOut, NT, 4, NG>(g, ng, stream);
        if (ctas >= 2LL * sm_count) return launch_bout_rb<kOut, NT, 2, NG>(g, ng, stream);
    }
    return launch_bout_rb<kOut, NT, 1, NG>(g, ng, stream);
}

template <int NT, int NG>
dq_status_t launch_batched_group(const BgGeom& G, int ng, const Group<BPArgs, NG>& pg, const Group<BDArgs, NG>& dg,
                                 const Group<BOArgs, NG>& og, int out_mode, int sm_count, int dsmem,
                                 cudaStream_t stream) {
    dq_status_t st = ensure_smem(bplan_kernel<NG>, NG == 1 ? 0 : 1, pg.p[0].S.total);
    if (st != DQ_OK) return st;
    st = ensure_smem(bdense_kernel<NT, NG>, 2 + (NT - 1) * 2 + (NG == 1 ? 0 : 1), dsmem);
    if (st != DQ_OK) return st;
    st = launch_pdl(bplan_kernel<NG>, dim3(G.MP, ng), kStatThreads, pg.p[0].S.total, stream, pg);
    if (st != DQ_OK) return st;
    st = launch_pdl(bdense_kernel<NT, NG>, dim3(dg.p[0].cps, G.nslab, ng), kBgWarps * 32, dsmem, stream, dg);
    if (st != DQ_OK) return st;
    switch (out_mode) {
        case kBoStaged: return launch_bout<kBoStaged, NT, NG>(og, ng, sm_count, stream);
        case kBoColDirect: return launch_bout<kBoColDirect, NT, NG>(og, ng, sm_count, stream);
        default: return launch_bout<kBoRowDirect, NT, NG>(og, ng, sm_count, stream);
    }
}

// The kernels' arguments for one problem (weights w, M vectors x, outputs y)
// with its workspace region ws, in the call's geometry G; cps CTAs per slab,
// and the share pf_share of each warp's row blocks that the INT4 part pulls
// into L2 before its dependency wait (1 or more: all).
void problem_args(const dq_weights_t& w, const uint16_t* x, uint16_t* y, int M, float k, char* ws, const BgGeom& G,
                  int cps, double pf_share, BPArgs& pa, BDArgs& da, BOArgs& oa) {
    const BgWs L = bg_ws(G, w.d_out, w.d_in);
    const BDSmem DS = bd_smem(G.S, G.MP);
    pa.x = x;
    pa.masks = reinterpret_cast<uint32_t*>(ws + L.masks);
    pa.xrow = reinterpret_cast<uint16_t*>(ws + L.xrow);
    pa.xtab = reinterpret_cast<uint4*>(ws + L.xtab);
    pa.xsum = reinterpret_cast<float4*>(ws + L.xsum);
    pa.k = k;
    pa.inv_n = 1.0f / static_cast<float>(w.d_in);
    pa.inv_n1 = w.d_in > 1 ? 1.0f / static_cast<float>(w.d_in - 1) : 0.f;
    pa.M = M;
    pa.MP = G.MP;
    pa.d_in = w.d_in;
    pa.W = G.W;
    pa.NC = G.NC;
    pa.S = bp_smem(w.d_in);

    BUArgs ua;
    ua.masks = pa.masks;
    ua.xrow = pa.xrow;
    ua.ulist = reinterpret_cast<uint16_t*>(ws + L.ulist);
    ua.xo = reinterpret_cast<uint16_t*>(ws + L.xo);
    ua.ctr = reinterpret_cast<unsigned int*>(ws + L.ctr);
    ua.M = M;
    ua.MP = G.MP;
    ua.d_in = w.d_in;
    ua.W = G.W;

    oa.w16 = w.fp16;
    oa.w16_cm = w.fp16_cm;
    oa.ulist = ua.ulist;
    oa.xo = ua.xo;
    oa.ctr = ua.ctr;
    oa.dpart = reinterpret_cast<float*>(ws + L.dpart);
    oa.y = y;
    oa.d_out = w.d_out;
    oa.d_in = w.d_in;
    oa.MP = G.MP;
    oa.M = M;
    oa.nslab = G.nslab;

    da.native = w.native;
    da.xtab = pa.xtab;
    da.xsum = pa.xsum;
    da.un = ua;
    da.dpart = reinterpret_cast<float*>(ws + L.dpart);
    da.M = M;
    da.d_out = w.d_out;
    da.d_in = w.d_in;
    da.NC = G.NC;
    da.NRB = G.NRB;
    da.S = G.S;
    da.nslab = G.nslab;
    da.cps = cps;
    {
        // L2 prefetch of the weights during the plan: each warp's first row
        // blocks, pf_share of them (1: all).
        const int nrw_max = (G.NRB / cps + 1 + kBgWarps - 1) / kBgWarps + 1;
        da.pf_rb = pf_share >= 1.0 ? nrw_max : static_cast<int>(nrw_max * pf_share);
    }
    da.sm_ring = DS.ring;
    da.sm_bars = DS.bars;
    da.sm_xtab = DS.xtab;
    da.sm_xsum = DS.xsum;
}

int out_mode_of(const dq_weights_t& w) {
    return w.fp16_cm ? ((w.d_out % 8) == 0 ? kBoStaged : kBoColDirect) : kBoRowDirect;
}

}  // namespace

dq_status_t launch_gemv_batched(const dq_weights_t& w, const uint16_t* x, uint16_t* y, int M, float k,
                                void* workspace, cudaStream_t stream) {
    DeviceInfo di;
    dq_status_t st = device_info(&di);
    if (st != DQ_OK) return st;
    const BgGeom G = bg_geom(w.d_out, w.d_in, M);
    const BDSmem DS = bd_smem(G.S, G.MP);
    if (DS.total > di.smem_optin || bp_smem(w.d_in).total > di.smem_optin) return DQ_ERR_UNSUPPORTED;
    const int cps = std::max(1, std::min(G.NRB, di.sm_count / G.nslab));
    const double total = static_cast<double>(G.NRB) * G.NC * kUnit;
    Group<BPArgs, 1> pg;
    Group<BDArgs, 1> dg;
    Group<BOArgs, 1> og;
    problem_args(w, x, y, M, k, static_cast<char*>(workspace), G, cps, kBgPrefetchBytes / total, pg.p[0], dg.p[0],
                 og.p[0]);
    const int om = out_mode_of(w);
    return G.NT == 1 ? launch_batched_group<1, 1>(G, 1, pg, dg, og, om, di.sm_count, DS.total, stream)
                     : launch_batched_group<2, 1>(G, 1, pg, dg, og, om, di.sm_count, DS.total, stream);
}

size_t batched_grouped_region(int d_out, int d_in, int m_max) {
    return align256(bg_ws(bg_geom(d_out, d_in, m_max), d_out, d_in).total);
}

dq_status_t launch_gemv_batched_grouped(const dq_weights_t* w, const uint16_t* const* x, uint16_t* const* y,
                                        const int32_t* m, int ng, float k, void* workspace, cudaStream_t stream) {
    DeviceInfo di;
    dq_status_t st = device_info(&di);
    if (st != DQ_OK) return st;
    int m_max = 1;
    for (int e = 0; e < ng; ++e) m_max = std::max(m_max, static_cast<int>(m[e]));
    const int d_out = w[0].d_out, d_in = w[0].d_in;
    const BgGeom G = bg_geom(d_out, d_in, m_max);
    const BDSmem DS = bd_smem(G.S, G.MP);
    if (DS.total > di.smem_optin || bp_smem(d_in).total > di.smem_optin) return DQ_ERR_UNSUPPORTED;
    const size_t region = batched_grouped_region(d_out, d_in, m_max);
    // The INT4 part's CTAs: about one per SM over all problems.
    const int cps = std::max(1, std::min(G.NRB, di.sm_count / (G.nslab * ng)));
    const double total = static_cast<double>(G.NRB) * G.NC * kUnit * ng;
    Group<BPArgs, kBgMaxGroups> pg;
    Group<BDArgs, kBgMaxGroups> dg;
    Group<BOArgs, kBgMaxGroups> og;
    for (int e = 0; e < ng; ++e)
        problem_args(w[e], x[e], y[e], m[e], k, static_cast<char*>(workspace) + e * region, G, cps,
                     kBgPrefetchBytes / total, pg.p[e], dg.p[e], og.p[e]);
    const int om = out_mode_of(w[0]);
    return G.NT == 1 ? launch_batched_group<1, kBgMaxGroups>(G, ng, pg, dg, og, om, di.sm_count, DS.total, stream)
                     : launch_batched_group<2, kBgMaxGroups>(G, ng, pg, dg, og, om, di.sm_count, DS.total, stream);
}

dq_status_t read_batched_error(uint32_t* word, bool clear) {
    cudaError_t e = cudaMemcpyFromSymbol(word, g_berror_word, sizeof(uint32_t));
    if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
    if (clear) {
        const uint32_t z = 0;
        e = cudaMemcpyToSymbol(g_berror_word, &z, sizeof(uint32_t));
        if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
    }
    return DQ_OK;
}

}  // namespace dq
