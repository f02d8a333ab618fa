// dq_stream.cu -- the batch-1 split / INT4 GEMV with a device-side task queue.
//
// Reference path (dyn-quant): src/split_gemv.cu:25-198 (split), src/int4_gemv.cu:12-100
// (INT4 only), src/outlier_detect.cuh:104-205 (the detector, here the plan).
//
// One call is one kernel: a persistent grid of one 16-warp CTA per SM.  The
// weights are cut into tasks of at most kTaskUnits units (a unit is 16 rows x
// 512 columns of the native layout, 4352 bytes): a task is a range of one row
// block's chunks when a row block has 8 chunks or more, else a run of whole
// row blocks.  CTA c starts with task c; every further task comes from an
// atomic counter in the workspace, so a CTA that starts late (its SM was still
// busy with the previous kernel) simply takes fewer tasks, and all CTAs finish
// within about one task of each other.
//
// Inside a CTA:
//   warp 15      the producer: takes tasks, streams their units into a ring of
//                R shared-memory slots with cp.async.bulk (one mbarrier per
//                slot; the consumers free the slots on a second set), and
//                stages the FP16 outlier-column segments of the row blocks a
//                task starts (bulk copies from the column-major mirror).
//   warps 0..14  the plan (statistics, mask, MMA fragments of x', per-group
//                sums, outlier list; dq_gplan.cuh), then the units: the
//                consumer of ring position p is warp p % 15.  A unit's 16 row
//                sums go to a per-unit slot in shared memory; the warp that
//                finishes a task's last unit runs its epilogue: the row sums
//                in unit order, plus the outlier columns on the tensor cores
//                for the row blocks whose chunk 0 is in the task, then either
//                y (the task holds whole row blocks) or the task's partial
//                sums in the workspace, where the last of a row block's tasks
//                to arrive adds them in task order and writes y.  Results do
//                not depend on which CTA or warp ran what: bit-reproducible.
//
// The unit arithmetic is the tensor-core formulation of dq_gemv.cu (biased
// INT4 codes in A, x' of group t in MMA columns 2t / 2t+1, the bias removed
// per group in FP32).  No wait depends on another CTA: counters in the
// workspace are reset by the CTA or task that takes them last.  Every wait on
// this CTA's own copies is bounded (about a second); on timeout the kernel
// sets bit 5 of the device error word and carries on (its output is then not
// valid), so that every counter still completes.
#include <cfloat>
#include <climits>
#include <cstdlib>

#include "dq_common.cuh"
#include "dq_gplan.cuh"
#include "dq_plan.cuh"
#include "dq_internal.h"

namespace dq {

namespace {

constexpr int kSW = 16;               // warps per CTA
constexpr int kSCons = kStreamConsumers;  // consumer warps; warp kSCons produces
constexpr int kST = kSW * 32;
constexpr int kTU = kStreamTaskUnits; // units per task, at most
constexpr int kTS = 8;                // tasks in flight per CTA, at most
constexpr int kObSegs = 512;          // outlier segments (32 B) per staging buffer
constexpr int kObBytes = kObSegs * 32;
constexpr int kOTile = 512;           // per-warp tile of 16 outlier columns x 16 rows
constexpr long long kWaitCycles = 1ll << 31;

__device__ unsigned int g_stream_error;  // bit 5 of the device error word

struct STask {
    int t;       // task index
    int ub, ue;  // units [ub, ue)
    int ob;      // outlier staging sequence number, -1: none
    int nseg;    // outlier segments of the task (row blocks x outliers)
    int staged;  // segments staged in shared memory (the rest: loads from the mirror)
    int pad0, pad1;
};

struct SArgs {
    const uint8_t* native;
    const uint16_t* w16_cm;
    const uint16_t* x;
    uint16_t* y;
    unsigned int* ctr;    // [0] tasks taken from the queue, [1] CTAs done
    unsigned int* rbcnt;  // [n_rb] tasks of the row block done (tpr > 1)
    float* part;          // [n_rb][tpr][16] partial row sums (tpr > 1)
    float k, inv_n, inv_n1;
    int d_out, d_in, G, NC, n_rb, tpr, m, n_tasks, n_static, R;
    SSmem S;
};

__device__ __forceinline__ void task_range(const SArgs& a, int t, int& ub, int& ue) {
    if (a.tpr > 1 || a.NC >= kTU) {
        const int rb = t / a.tpr, kk = t - rb * a.tpr;
        ub = rb * a.NC + kk * a.NC / a.tpr;
        ue = rb * a.NC + (kk + 1) * a.NC / a.tpr;
    } else {
        ub = t * a.m * a.NC;
        ue = min((t + 1) * a.m, a.n_rb) * a.NC;
    }
}

// Bounded wait on this CTA's mbarrier; once a wait of this thread has given
// up (ok false) the later ones do not wait at all, so that a failed call ends
// quickly (its output is then not valid and the error word says so).
__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity, bool ok = true) {
    if (!ok) return false;
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > kWaitCycles) return false;
    }
    return true;
}

template <bool kSplit, int kPPT>
__global__ void __launch_bounds__(kST, 1) stream_kernel(const SArgs a) {
    extern __shared__ __align__(128) char smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int NC = a.NC, R = a.R;
    const int P = gridDim.x, c = blockIdx.x;

    const uint32_t ring = smem_u32(smem + a.S.ring);
    const uint32_t fullb = smem_u32(smem + a.S.full);
    const uint32_t emptyb = smem_u32(smem + a.S.empty);
    const uint32_t obfull = smem_u32(smem + a.S.obbar);
    const uint32_t obempty = obfull + 16;
    int4* desc = reinterpret_cast<int4*>(smem + a.S.desc);
    STask* ttab = reinterpret_cast<STask*>(smem + a.S.ttab);
    float* upart = reinterpret_cast<float*>(smem + a.S.upart);  // [kTS][kTU][16]
    int* tdone = reinterpret_cast<int*>(smem + a.S.misc);       // [kTS]
    int* tgen = tdone + kTS;                                     // [kTS]
    volatile int* plan_ready = tgen + kTS;                       // [1]: 1 + number of outliers
    int* obgen = tgen + kTS + 4;                                 // [2]: epilogues done per staging buffer
    float* red = reinterpret_cast<float*>(smem + a.S.red);       // 32 floats + scan scratch
    int* scratch = reinterpret_cast<int*>(red + 32);
    uint4* xb = reinterpret_cast<uint4*>(smem + a.S.xb);
    float4* xp4 = reinterpret_cast<float4*>(smem + a.S.xp);
    uint32_t* mask32 = reinterpret_cast<uint32_t*>(smem + a.S.mask);
    uint32_t* list = reinterpret_cast<uint32_t*>(smem + a.S.list);

    if (tid == 0) {
        for (int s = 0; s < R; ++s) {
            mbar_init(fullb + 8 * s, 1);
            mbar_init(emptyb + 8 * s, 1);
        }
        mbar_init(obfull, 1);
        mbar_init(obfull + 8, 1);
        mbar_init(obempty, 1);
        mbar_init(obempty + 8, 1);
        fence_mbar_init();
    }
    for (int i = tid; i < 2 * kTS + 8; i += kST) tdone[i] = 0;
    for (int i = tid; i < R; i += kST) desc[i] = make_int4(-1, 0, 0, 0);  // a slot never filled reads as the end
    for (int i = tid; i < 32; i += kST) red[i] = 0.f;
    for (int i = tid; i < kB1ChunkB / 16; i += kST) reinterpret_cast<uint4*>(smem + a.S.zero)[i] = make_uint4(0, 0, 0, 0);
    // The groups past d_in in the last chunk stay zero: their fragment pieces
    // (interleaved with the real groups' in the chunk's block: piece (wi, sl)
    // of group jj at 4 (4 wi + sl) + jj) and their per-group sums.
    const int jj_pad = a.G - 4 * (NC - 1);  // first padding group of the last chunk
    auto zero_pad = [&](int t0, int nt) {
        for (int i = t0; i < 64; i += nt)
            if ((i & 3) >= jj_pad) xb[64 * (NC - 1) + i] = make_uint4(0, 0, 0, 0);
    };
    zero_pad(tid, kST);
    for (int i = tid + a.G; i < 4 * NC; i += kST) xp4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    __syncthreads();

    // The weights do not depend on the preceding kernel; they may have been
    // written by it, though, so only an L2 prefetch of this CTA's likely first
    // tasks runs before griddepcontrol.wait.
    if (warp == kSCons && lane == 0) {
        for (int q = 0; q < 2; ++q) {
            const int tq = c + q * P;
            if (tq < a.n_tasks) {
                int ub, ue;
                task_range(a, tq, ub, ue);
                for (int u = ub; u < ue; ++u)
                    prefetch_l2_bulk(a.native + static_cast<size_t>(u) * kB1UnitBytes, kB1UnitBytes);
            }
        }
    }
    pdl_launch_dependents();
    pdl_wait();  // x, y and the workspace may belong to the preceding kernel until here

    bool ok = true;
    if (warp == kSCons) {
        // ------------------------------------------------------------ producer
        int p = 0;        // ring position
        int ts = 0;       // tasks of this CTA so far
        int ob_seq = 0;   // outlier stagings so far
        // Tasks j < J0 of this CTA are static (task c + P j); the rest come
        // from the queue, each index taken two tasks ahead of its use so that
        // the atomic's latency stays off the issue path.
        const int J0 = a.n_static / P;
        int j = 0;  // tasks of this CTA so far (= ts)
        int t_cur = J0 > 0 ? c : INT_MAX;
        unsigned int g0 = 0, g1 = 0;  // queue indices taken ahead
        if (lane == 0) {
            if (J0 == 0) {
                const unsigned int q = atomicAdd(a.ctr, 1u);
                t_cur = static_cast<int>(min(q, static_cast<unsigned int>(INT_MAX / 2))) + a.n_static;
            }
            // (with J0 >= 3 both are taken in the loop, at tasks J0 - 2 and J0 - 1)
            if (J0 <= 2) g0 = atomicAdd(a.ctr, 1u);
            if (J0 <= 1) g1 = atomicAdd(a.ctr, 1u);
        }
        int n_out = -1;
        while (true) {
            t_cur = __shfl_sync(0xffffffffu, t_cur, 0);
            if (t_cur >= a.n_tasks) break;
            int ub, ue;
            task_range(a, t_cur, ub, ue);
            const int slot_t = ts % kTS;
            // the task slot is free once task ts - kTS has run its epilogue
            if (lane == 0 && ts >= kTS && ok) {
                const long long t0 = clock64();
                while (*reinterpret_cast<volatile int*>(tgen + slot_t) < ts / kTS) {
                    if (clock64() - t0 > kWaitCycles) { ok = false; break; }
                }
            }
            // row blocks whose chunk 0 is in the task carry its outlier columns
            const int rbA = (ub + NC - 1) / NC, rbB = (ue + NC - 1) / NC;
            STask T;
            T.t = t_cur;
            T.ub = ub;
            T.ue = ue;
            T.ob = -1;
            T.nseg = 0;
            T.staged = 0;
            if (kSplit && rbB > rbA) {
                if (n_out < 0) {  // the plan's outlier count
                    if (lane == 0) {
                        const long long t0 = clock64();
                        int v;
                        while ((v = *plan_ready) == 0) {
                            if (clock64() - t0 > kWaitCycles) { ok = false; v = 1; break; }
                        }
                        n_out = v - 1;
                    }
                    n_out = __shfl_sync(0xffffffffu, n_out, 0);
                    __threadfence_block();  // the plan's list, published with the flag
                }
                if (n_out > 0) {
                    T.nseg = (rbB - rbA) * n_out;
                    T.staged = min(T.nseg, kObSegs);
                    T.ob = ob_seq++;
                }
            }
            if (lane == 0) ttab[slot_t] = T;
            __syncwarp();
            // The units: lane i issues the task's unit i (ring position p + i).
            // One thread's bulk copies are processed one after another, so the
            // lanes issue in parallel.  A slot is refilled only after its
            // consumer freed it; if that wait gives up, nothing more is issued.
            {
                const int nu = ue - ub;
                ok = __shfl_sync(0xffffffffu, ok, 0);
                bool fail = false;
                if (lane < nu && ok) {
                    const int pp = p + lane, s = pp % R, use = pp / R;
                    if (use > 0 && !wait_bounded(emptyb + 8 * s, (use - 1) & 1)) fail = true;
                    if (!fail) {
                        desc[s] = make_int4(ub + lane, ts, lane, nu);
                        mbar_arrive_expect_tx(fullb + 8 * s, kB1UnitBytes);
                        bulk_g2s(ring + s * kB1UnitBytes, a.native + static_cast<size_t>(ub + lane) * kB1UnitBytes,
                                 kB1UnitBytes, fullb + 8 * s);
                    }
                }
                if (__any_sync(0xffffffffu, fail)) ok = false;
                p += nu;
            }
            // the outlier segments (the whole warp issues the copies)
            if (kSplit && T.ob >= 0) {
                const int b = T.ob & 1;
                const uint32_t buf = smem_u32(smem + a.S.obuf) + b * kObBytes;
                if (lane == 0 && T.ob >= 2 && !wait_bounded(obempty + 8 * b, ((T.ob >> 1) - 1) & 1, ok)) ok = false;
                if (!__shfl_sync(0xffffffffu, ok, 0)) T.staged = 0;  // failed: no copies, no arming
                const int last_rows = a.d_out - (a.n_rb - 1) * kRowBlock;
                // 16-byte cp.async pieces (rows 0-7 and 8-15 of a segment), spread over
                // the lanes; each lane's copies join the buffer's barrier phase, and
                // lane 0's arrive closes it.
                for (int pc = lane; pc < 2 * T.staged; pc += 32) {
                    const int sg = pc >> 1, hh = pc & 1;
                    const int rb = rbA + sg / n_out, kk = sg % n_out;
                    const int rows = rb == a.n_rb - 1 ? last_rows : kRowBlock;
                    const int col = static_cast<int>(list[kk] & 0xFFFFu);
                    if (8 * hh < rows && col < a.d_in)
                        cp_async16(buf + sg * 32 + 16 * hh,
                                   a.w16_cm + static_cast<size_t>(col) * a.d_out + rb * kRowBlock + 8 * hh);
                }
                if (T.staged > 0) cp_async_mbar_arrive(obfull + 8 * b);
                __syncwarp();
                if (lane == 0 && T.staged > 0) mbar_arrive(obfull + 8 * b);
            }
            ++ts;
            ++j;
            if (lane == 0) {
                if (j < J0) {
                    t_cur = c + P * j;
                    if (j + 2 == J0) g0 = atomicAdd(a.ctr, 1u);  // the first two queue tasks, ahead
                    if (j + 1 == J0) g1 = atomicAdd(a.ctr, 1u);
                } else {
                    t_cur = static_cast<int>(min(g0, static_cast<unsigned int>(INT_MAX / 2))) + a.n_static;
                    g0 = g1;
                    if (t_cur < a.n_tasks) g1 = atomicAdd(a.ctr, 1u);
                }
                if (!ok) t_cur = INT_MAX;  // a wait gave up: issue nothing more
            }
        }
        // one end marker per consumer warp (lane e for warp (p + e) % 15)
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (lane < kSCons && ok) {
            const int pp = p + lane, s = pp % R, use = pp / R;
            bool got = use == 0 || wait_bounded(emptyb + 8 * s, (use - 1) & 1);
            if (got) {
                desc[s] = make_int4(-1, 0, 0, 0);
                mbar_arrive(fullb + 8 * s);
            } else {
                ok = false;
            }
        }
    } else {
        // ------------------------------------------------------------ plan
        auto bar = []() { named_bar_sync(1, kSCons * 32); };
        GpRegs<kPPT> xr;
        gp_load<kPPT>(a.x, a.G, tid, xr);
        int n_out = 0;
        if (kSplit) {
            // The statistics in the partition of dq_plan.cuh (that of the block
            // kernel, the detector and the batched plan: the same bits), from
            // x in natural order in xb (overwritten by the fragments below).
            {
                const int TPG = 16 / kPPT;
                if (tid < a.G * TPG) {
                    const int j = tid / TPG, h = tid % TPG;
#pragma unroll
                    for (int i = 0; i < kPPT; ++i) xb[16 * j + kPPT * h + i] = xr.v[i];
                }
            }
            bar();
            const XStats st = x_stats_bar<kSCons * 32>(xb, a.d_in / 8, a.d_in, a.k, a.inv_n, a.inv_n1, red, bar);
            bar();  // every thread is done with xb
            zero_pad(tid, kSCons * 32);
            const int cap = a.d_in / 16;  // no stripe class can exceed its capacity below this total
            n_out = gp_frags<kPPT, kSCons, true>(xr, a.G, st.mean, st.thresh, nullptr, cap, xb, xp4, list, scratch, bar);
            if (n_out > cap) {
                // The reference's capacity rule may drop outliers: the mask from x
                // in natural order (written over xb), then fragments and list again.
                bar();
                const int TPG = 16 / kPPT;
                if (tid < a.G * TPG) {
                    const int j = tid / TPG, h = tid % TPG;
#pragma unroll
                    for (int i = 0; i < kPPT; ++i) xb[16 * j + kPPT * h + i] = xr.v[i];
                }
                bar();
                gp_capacity_mask<kSCons>(xb, a.d_in, st.mean, st.thresh, mask32, scratch, bar);
                zero_pad(tid, kSCons * 32);  // the copy of x covered some padding pieces
                n_out = gp_frags<kPPT, kSCons, true>(xr, a.G, st.mean, st.thresh, mask32, INT_MAX, xb, xp4, list,
                                                     scratch + 64, bar);
            }
        } else {
            gp_frags<kPPT, kSCons, false>(xr, a.G, 0.f, 0.f, nullptr, 0, xb, xp4, nullptr, scratch, bar);
        }
        bar();  // fragments, sums and list complete
        // for the producer's outlier staging; set only now, when every
        // thread's list entries are in (the consumers use their own n_out)
        if (tid == 0) *plan_ready = 1 + n_out;

        // ------------------------------------------------------------ units
        const uint32_t zero_a = smem_u32(smem + a.S.zero);
        const uint32_t bsm_a = smem_u32(xb);
        const uint32_t xp_a = smem_u32(xp4);
        const bool b_owner = (g >> 1) == t;  // lane supplies B column 2t (g even) or 2t+1 (g odd)
        const uint32_t b_lane = t * 16 + (g & 1) * 8;
        const uint32_t otile = smem_u32(smem + a.S.otile) + warp * kOTile;
        // positions of this warp: at most every unit of the call plus the end marker
        const int p_max = a.n_rb * NC + kSCons;
        for (int p = warp;; p += kSCons) {
            const int s = p % R;
            if (!wait_bounded(fullb + 8 * s, (p / R) & 1, ok)) ok = false;
            const int4 d = desc[s];
            // (a descriptor is valid unless a wait gave up; checked all the same,
            // so that nothing below can index out of range)
            const bool valid = d.x >= 0 && d.x < a.n_rb * NC && d.y >= 0 && d.z >= 0 && d.z < d.w && d.w <= kTU;
            if (!valid || p > p_max) {
                if (d.x >= 0) ok = false;
                break;
            }
            const int u = d.x, ts = d.y, ui = d.z, nu = d.w;
            const uint32_t st = ring + s * kB1UnitBytes;
            const int cc = u % NC;
            uint4 aw[4][2];  // [slice][row g / g+8]: 32 columns of group t
#pragma unroll
            for (int sl = 0; sl < 4; ++sl)
#pragma unroll
                for (int h = 0; h < 2; ++h) aw[sl][h] = lds_v4(st + native_piece(sl, h, g, t) * 16);
            const uint32_t sz0 = lds_u32(st + kB1UnitPacked + 16 * g + 4 * t);
            const uint32_t sz8 = lds_u32(st + kB1UnitPacked + 16 * (g + 8) + 4 * t);
            __syncwarp();
            if (lane == 0) mbar_arrive(emptyb + 8 * s);  // the unit is in registers: free the slot
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
                    const Biased4 qa = biased_word(gp_word(aw[sl][0], wi));
                    const Biased4 qb = biased_word(gp_word(aw[sl][1], wi));
                    const uint2 b = lds_v2(bb + (wi * 4 + sl) * 64);
                    mma_16816(dl[sl], qa.lo0, qb.lo0, qa.lo1, qb.lo1, b.x, b.y);
                    mma_16816(dh[sl], qa.hi0, qb.hi0, qa.hi1, qb.hi1, b.x, b.y);
                }
            }
            const float lo0 = (dl[0][0] + dl[1][0]) + (dl[2][0] + dl[3][0]);
            const float hi0 = (dh[0][1] + dh[1][1]) + (dh[2][1] + dh[3][1]);
            const float lo8 = (dl[0][2] + dl[1][2]) + (dl[2][2] + dl[3][2]);
            const float hi8 = (dh[0][3] + dh[1][3]) + (dh[2][3] + dh[3][3]);
            const uint4 xqb = lds_v4(xp_a + (kB1ChunkGroups * cc + t) * 16);
            const float xe = __uint_as_float(xqb.x), xo = __uint_as_float(xqb.y), xs = __uint_as_float(xqb.z);
            const float S0 = fmaf(hi0 - xo, 0.0625f, lo0 - xe);
            const float S8 = fmaf(hi8 - xo, 0.0625f, lo8 - xe);
            float acc0 = h2f_bits(lo16(sz0)) * fmaf(-h2f_bits(hi16(sz0)), xs, S0);
            float acc8 = h2f_bits(lo16(sz8)) * fmaf(-h2f_bits(hi16(sz8)), xs, S8);
            acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
            acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
            acc8 += __shfl_xor_sync(0xffffffffu, acc8, 1);
            acc8 += __shfl_xor_sync(0xffffffffu, acc8, 2);
            float* up = upart + ((ts % kTS) * kTU + ui) * 16;
            if (t == 0) {
                up[g] = acc0;
                up[g + 8] = acc8;
            }
            __threadfence_block();
            __syncwarp();
            int last = 0;
            if (lane == 0) last = atomicAdd(tdone + ts % kTS, 1) == nu - 1;
            last = __shfl_sync(0xffffffffu, last, 0);
            if (!last) continue;

            // ---------------------------------------------------- task epilogue
            __threadfence_block();
            STask T = ttab[ts % kTS];
            if (T.ub < 0 || T.ue > a.n_rb * NC || T.ue - T.ub != nu || T.t < 0 || T.t >= a.n_tasks) {
                ok = false;  // only after a wait gave up: no epilogue
                continue;
            }
            const int rbA = (T.ub + NC - 1) / NC;
            // The staging buffer's previous task (T.ob - 2) must be done with it
            // first: then the buffer's barrier is at most one phase behind this
            // task's, and the parity wait below is exact.
            if (kSplit && T.ob >= 0 && lane == 0 && ok) {
                const long long t0 = clock64();
                while (*reinterpret_cast<volatile int*>(obgen + (T.ob & 1)) < (T.ob >> 1)) {
                    if (clock64() - t0 > kWaitCycles) { ok = false; break; }
                }
            }
            if (kSplit && T.ob >= 0) ok = __shfl_sync(0xffffffffu, ok, 0) && ok;
            if (kSplit && T.ob >= 0 && !wait_bounded(obfull + 8 * (T.ob & 1), (T.ob >> 1) & 1, ok)) ok = false;
            const uint32_t obuf = smem_u32(smem + a.S.obuf) + (T.ob & 1) * kObBytes;
            for (int rb = T.ub / NC; rb <= (T.ue - 1) / NC; ++rb) {
                // INT4 part of the row block's units in this task, in unit order
                const int u0 = max(T.ub, rb * NC), u1 = min(T.ue, (rb + 1) * NC);
                float v = 0.f;
                if (lane < 16)
                    for (int uu = u0; uu < u1; ++uu) v += upart[((ts % kTS) * kTU + (uu - T.ub)) * 16 + lane];
                // outlier columns: W16[rows][U] x_U on the tensor cores, 16 columns at a time
                if (kSplit && T.ob >= 0 && rb >= rbA) {
                    const int rbl = rb - rbA;
                    float od[4] = {0.f, 0.f, 0.f, 0.f};
                    for (int k0 = 0; k0 < n_out; k0 += kB1OutBatch) {
                        // lane (i, hh): column k0 + i, rows 8 hh .. 8 hh + 7 of the row block
                        const int kk = k0 + (lane >> 1), hh = lane & 1;
                        const int sg = rbl * n_out + kk;
                        uint4 seg = make_uint4(0, 0, 0, 0);
                        if (kk < n_out) {
                            const int row0 = rb * kRowBlock + 8 * hh;
                            if (sg < T.staged) {
                                seg = lds_v4(obuf + sg * 32 + 16 * hh);
                            } else {
                                const int col = static_cast<int>(list[kk] & 0xFFFFu);
                                if (row0 < a.d_out && col < a.d_in)
                                    seg = ldg_v4(a.w16_cm + static_cast<size_t>(col) * a.d_out + row0);
                            }
                        }
                        sts_v4(otile + 16 * lane, seg);
                        __syncwarp();
                        uint32_t a0, a1, a2, a3;
                        ldmatrix_x4_trans(otile + (((lane >> 4) * 8 + (lane & 7)) * 32) + ((lane >> 3) & 1) * 16, a0,
                                          a1, a2, a3);
                        auto xo_ = [&](int q) -> uint32_t { return q < n_out ? (list[q] >> 16) : 0u; };
                        const uint32_t b0 = xo_(k0 + 2 * t) | (xo_(k0 + 2 * t + 1) << 16);
                        const uint32_t b1 = xo_(k0 + 2 * t + 8) | (xo_(k0 + 2 * t + 9) << 16);
                        mma_16816(od, a0, a1, a2, a3, b0, b1);
                        __syncwarp();
                    }
                    // lane r (< 16) takes row r: from lane 4 (r & 7), od[0] (r < 8) or od[2]
                    const float o0 = __shfl_sync(0xffffffffu, od[0], 4 * (lane & 7));
                    const float o2 = __shfl_sync(0xffffffffu, od[2], 4 * (lane & 7));
                    v += (lane & 8) ? o2 : o0;
                }
                const int row = rb * kRowBlock + lane;
                auto store_row = [&](float value) { a.y[row] = __half_as_ushort(__float2half_rn(value)); };
                if (a.tpr == 1) {
                    if (lane < 16 && row < a.d_out) store_row(v);
                } else {
                    // this task's share of the row block; the last of its tasks adds them up
                    const int kk = T.t - rb * a.tpr;
                    if (lane < 16) a.part[(static_cast<size_t>(rb) * a.tpr + kk) * 16 + lane] = v;
                    __threadfence();
                    __syncwarp();
                    int lst = 0;
                    if (lane == 0) lst = atomicAdd(a.rbcnt + rb, 1u) == static_cast<unsigned>(a.tpr - 1);
                    lst = __shfl_sync(0xffffffffu, lst, 0);
                    if (lst) {
                        __threadfence();
                        float sum = 0.f;
                        if (lane < 16)
                            for (int q = 0; q < a.tpr; ++q)
                                sum += q == kk ? v : ldcg_f32(a.part + (static_cast<size_t>(rb) * a.tpr + q) * 16 + lane);
                        if (lane < 16 && row < a.d_out) store_row(sum);
                        if (lane == 0) a.rbcnt[rb] = 0u;
                    }
                }
            }
            __syncwarp();
            if (lane == 0) {
                if (kSplit && T.ob >= 0) {
                    *reinterpret_cast<volatile int*>(obgen + (T.ob & 1)) = (T.ob >> 1) + 1;
                    mbar_arrive(obempty + 8 * (T.ob & 1));
                }
                tdone[ts % kTS] = 0;
                __threadfence_block();
                *reinterpret_cast<volatile int*>(tgen + ts % kTS) = ts / kTS + 1;
            }
        }
    }
    if (!ok) atomicOr(&g_stream_error, 1u);

    // Every CTA done: the last one resets the queue for the next call.
    __syncthreads();
    if (tid == 0 && atomicAdd(a.ctr + 1, 1u) == gridDim.x - 1u) {
        a.ctr[0] = 0u;
        a.ctr[1] = 0u;
    }
}

// Per-device, per-kernel "max dynamic shared memory" opt-in, done once.
constexpr int kMaxDevices = 64;
constexpr int kNumKernels = 8;  // (split, plan pieces per thread)
int g_smem_set[kMaxDevices][kNumKernels];

template <class K>
dq_status_t ensure_smem_s(K kernel, int id, int bytes) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
    if (dev >= 0 && dev < kMaxDevices && __atomic_load_n(&g_smem_set[dev][id], __ATOMIC_ACQUIRE) >= bytes)
        return DQ_OK;
    const int want = bytes < 48 * 1024 ? 48 * 1024 : bytes;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, want);
    if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
    if (dev >= 0 && dev < kMaxDevices) {
        int cur = __atomic_load_n(&g_smem_set[dev][id], __ATOMIC_ACQUIRE);
        while (cur < want && !__atomic_compare_exchange_n(&g_smem_set[dev][id], &cur, want, false, __ATOMIC_ACQ_REL,
                                                          __ATOMIC_ACQUIRE)) {
        }
    }
    return DQ_OK;
}

template <bool kSplit, int kPPT>
dq_status_t launch_stream_t(const SArgs& a, int grid, cudaStream_t stream) {
    constexpr int id = (kSplit ? 4 : 0) + (kPPT == 1 ? 0 : kPPT == 2 ? 1 : kPPT == 4 ? 2 : 3);
    const dq_status_t st = ensure_smem_s(stream_kernel<kSplit, kPPT>, id, a.S.total);
    if (st != DQ_OK) return st;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kST);
    cfg.dynamicSmemBytes = a.S.total;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, stream_kernel<kSplit, kPPT>, a);
    if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
    e = cudaGetLastError();
    if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
    return DQ_OK;
}

template <bool kSplit>
dq_status_t launch_stream_p(const SArgs& a, int ppt, int grid, cudaStream_t stream) {
    switch (ppt) {
        case 1: return launch_stream_t<kSplit, 1>(a, grid, stream);
        case 2: return launch_stream_t<kSplit, 2>(a, grid, stream);
        case 4: return launch_stream_t<kSplit, 4>(a, grid, stream);
        default: return launch_stream_t<kSplit, 8>(a, grid, stream);
    }
}

// Ring slots: an optional cap from the environment (DQ_STREAM_SLOTS), read once.
int slot_cap() {
    static const int cap = [] {
        const char* s = std::getenv("DQ_STREAM_SLOTS");
        const int v = s ? std::atoi(s) : 0;
        return v > 0 ? v : kStreamMaxSlots;
    }();
    return cap;
}

}  // namespace

bool stream_supported(const dq_weights_t& w, bool split) {
    return w.native != nullptr && (!split || (w.fp16_cm != nullptr && w.d_out % 8 == 0)) && w.d_out > 0 &&
           w.d_in <= kMaxDIn;
}

dq_status_t launch_gemv_stream(const dq_weights_t& w, const uint16_t* x, uint16_t* y, float k, bool split,
                               void* workspace, cudaStream_t stream) {
    DeviceInfo di;
    const dq_status_t st = device_info(&di);
    if (st != DQ_OK) return st;
    const StreamGeom sg = stream_geom(w.d_out, w.d_in);
    SArgs a{};
    a.native = w.native;
    a.w16_cm = w.fp16_cm;
    a.x = x;
    a.y = y;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const StreamWs L = stream_ws(w.d_out, w.d_in);
    a.ctr = reinterpret_cast<unsigned int*>(ws + L.ctr);
    a.rbcnt = reinterpret_cast<unsigned int*>(ws + L.rbcnt);
    a.part = reinterpret_cast<float*>(ws + L.part);
    a.k = k;
    a.inv_n = 1.0f / static_cast<float>(w.d_in);
    a.inv_n1 = w.d_in > 1 ? 1.0f / static_cast<float>(w.d_in - 1) : 0.f;
    a.d_out = w.d_out;
    a.d_in = w.d_in;
    a.G = w.d_in / kGroup;
    a.NC = sg.NC;
    a.n_rb = sg.n_rb;
    a.tpr = sg.tpr;
    a.m = sg.m;
    a.n_tasks = sg.n_tasks;
    const int grid = di.sm_count < sg.n_tasks ? di.sm_count : sg.n_tasks;
    // All but about the last two tasks of every CTA are assigned round robin;
    // the rest are taken from the queue by whichever CTAs are free.
    const int per = sg.n_tasks / grid;
    a.n_static = (per > 2 ? per - 2 : 0) * grid;
    // As many ring slots as fit next to the plan, a multiple of the consumer
    // warps: ring position p is consumed by warp p % 15 and its slot p % R
    // was last used by position p - R, so with R a multiple of 15 the same
    // warp consumed that use first (in order), and the parity waits on the
    // slot's barriers never see a phase two uses old.  At least 15 slots (a
    // task's units and the consumers' end markers go out in one step each).
    int R = slot_cap() / kSCons * kSCons;
    if (R < kSCons) R = kSCons;
    for (; R >= kSCons; R -= kSCons) {
        a.S = stream_smem(w.d_in, split, R);
        if (a.S.total <= di.smem_optin) break;
    }
    if (R < kSCons) return DQ_ERR_UNSUPPORTED;
    a.R = R;
    const int ppt = 16 / gp_tpg(a.G);
    return split ? launch_stream_p<true>(a, ppt, grid, stream) : launch_stream_p<false>(a, ppt, grid, stream);
}

dq_status_t read_stream_error(uint32_t* word, bool clear) {
    unsigned int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_stream_error, sizeof(v));
    if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
    if (clear && v) {
        const unsigned int zero = 0;
        e = cudaMemcpyToSymbol(g_stream_error, &zero, sizeof(zero));
        if (e != cudaSuccess) { set_cuda_error(e); return DQ_ERR_CUDA; }
    }
    *word = v;
    return DQ_OK;
}

}  // namespace dq
