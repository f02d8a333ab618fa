// dq_internal.h -- host-side interface between the C ABI (dq_abi.cu) and the
// kernel translation units.  Not installed; include/dq_abi.h is the public API.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/dq_abi.h"

namespace dq {

// Geometry of the batch-1 split / INT4 kernel (shared by host sizing and
// device carving).
constexpr int kB1Warps = 16;                         // warps per CTA (one CTA per SM), at most
constexpr int kB1WarpsSmall = 12;                    // when 16 warps' rings do not fit next to x
constexpr int kB1MaxDepth = 8;                       // ring stages per warp, at most
constexpr int kB1Stages = 2;                         // ring stages per warp, reference layout (native: at least)
constexpr int kB1ChunkGroups = 4;                    // 128-column groups per unit
constexpr int kB1UnitPacked = 4096;                  // packed INT4 of one unit (16 rows x 512 columns)
constexpr int kB1StageSZ = 256;                      // 16 rows x 4 groups x (scale, zero)
constexpr int kB1UnitBytes = kB1UnitPacked + kB1StageSZ;  // one unit of the native layout
constexpr int kB1RowPitch = 272;                     // reference layout: smem bytes per weight row
constexpr int kB1StageBytes = kB1UnitBytes;          // 16 rows x 272 bytes is the same size
constexpr int kB1ChunkB = 1024;                      // MMA B fragments of one 512-column chunk
constexpr int kB1RedBytes = 2048;                    // reduction / scan scratch
constexpr int kB1OutBatch = 16;                      // outlier columns per tensor-core task
constexpr int kB1OutBufs = 3;                        // per-warp task buffers in flight
constexpr int kB1OutBufBytes = kB1OutBatch * 32;     // 16 columns x 16 rows of FP16
constexpr int kStatThreads = 512;                    // fixed partition of the statistics of x
constexpr int kMaxCtas = 1024;                       // bound on the GEMV grid (workspace sizing)

__host__ __device__ inline int align16(int v) { return (v + 15) & ~15; }

// Shared memory of one batch-1 GEMV CTA with `warps` warps.  Every CTA derives
// the activation plan itself (x is at most 60 KB and stays in L2):
//   ring  slots of weight units (a warp's i-th unit in slot warp + warps (i % depth))
//   bars  one mbarrier per slot
//   misc  this call's tag (workspace protocol)
//   zero  1 KB of zeros (B operand of lanes outside their column pair)
//   bsm   x, then in place the MMA B fragments of x' (outliers zeroed), NC chunks
//   xp    per group float4 (1024 sum x' even cols, 1024 sum x' odd cols, sum x', 0)
//   mask  outlier bits (split only)
//   red   reduction and scan scratch
//   part  per row block and warp: partial row sums of the INT4 part
//   opart per warp and row block: partial row sums of the outlier columns (split only)
//   list  outliers, column | FP16 bits of x << 16, capacity d_in/4 (split only)
//   obuf  per warp, kB1OutBufs buffers of 16 outlier columns x 16 rows (split only)
struct B1Smem {
    int ring, bars, misc, zero, bsm, xp, mask, red, part, opart, list, obuf, total;
};

// slots: ring slots of kB1StageBytes, each with its mbarrier.  slab_nc: the
// chunks of a column slab (0: no slabs); bsm and xp then hold the slab's
// fragments only, while the mask and the list stay sized for all of x, and
// part .. obuf (unused until the plan is done) first hold all of x for the
// statistics.
inline B1Smem b1_smem(int d_in, int nrb_max, bool split, int warps, int slots, int slab_nc = 0) {
    const int NCall = (d_in / 128 + kB1ChunkGroups - 1) / kB1ChunkGroups;
    const int NC = slab_nc > 0 ? slab_nc : NCall;
    B1Smem S;
    int off = 0;
    S.ring = off;  off += slots * kB1StageBytes;
    S.bars = off;  off += (slots * 8 + 127) / 128 * 128;
    S.misc = off;  off += 128;  // this call's tag
    S.zero = off;  off += kB1ChunkB;
    S.bsm = off;   off += NC * kB1ChunkB;
    S.xp = off;    off += NC * kB1ChunkGroups * 16;
    S.mask = off;  off += split ? NCall * 64 : 0;
    S.red = off;   off += kB1RedBytes;
    S.part = off;  off += nrb_max * warps * 16 * 4;
    S.opart = off; off += split ? warps * nrb_max * 16 * 4 : 0;
    S.list = off;  off += split ? align16(d_in) : 0;
    S.obuf = off;  off += split ? warps * kB1OutBufs * kB1OutBufBytes : 0;
    // Column slabs of the split GEMV stage all of x from part on while the
    // plan runs (the statistics are over all of x).
    if (slab_nc > 0 && split && off < S.part + align16(2 * d_in)) off = S.part + align16(2 * d_in);
    S.total = off;
    return S;
}

// Workspace of a batch-1 GEMV call:
//   hdr  [0] the number of the last completed call (its tag), [1] CTAs of the
//        running call that have finished (the last one resets it to zero and
//        advances [0])
//   fix  per CTA, the 16 partial row sums of its first row block when that
//        block is shared with the preceding CTA, each a 64-bit word
//        (tag << 32 | FP32 bits): a word is this call's only if it carries
//        this call's tag, so words left by an earlier call are never taken.
// Zero before first use; every call leaves it ready for the next one (also a
// call whose bounded waits gave up).  Long rows cut into column slabs also
// use the slab region after the fixed header (ws_slab_offset).
struct WsLayout {
    size_t hdr, fix, total;
};

inline size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

constexpr int kB1SlabMinNC = 48;          // chunks per row (d_in / 512) from which rows are cut into slabs
constexpr int kB1SlabMaxUnits = 128;      // ... when a CTA's share is at most this many units
// Column slabs of a batch-1 call with NC chunks per row: the largest divisor
// of NC not above ceil(NC / 16) (so a slab holds about 16 chunks), or 1.
inline int b1_slabs(int NC) {
    if (NC < kB1SlabMinNC) return 1;
    for (int S = (NC + 15) / 16; S > 1; --S)
        if (NC % S == 0) return S;
    return 1;
}
// Slab region: per row block and slab 1 .. S-1, 16 tagged partial row sums
// (tag << 32 | FP32 bits), 8 bytes each.
inline size_t b1_slab_bytes(int d_out, int S) {
    const size_t n_rb = (static_cast<size_t>(d_out) + 15) / 16;
    return align256(n_rb * static_cast<size_t>(S - 1) * 16 * sizeof(unsigned long long));
}

// Gather region of one rank (row-sharded split GEMV with the gather fused):
//   hdr    u32 [0] calls this rank has completed (the running call's number
//          is that + 1)
//   yfull  two copies of the full output (kMaxGatherRanks x rows_per rows),
//          for calls of parity 0 and 1, one 32-bit word per row: the FP16
//          value in the low half, the low 16 bits of the call's number in
//          the high half.  Rank q stores its rows of a call straight into
//          every other rank's copy of that parity; a word is this call's
//          once it carries this call's tag (one 32-bit store: value and tag
//          arrive together), so no fence or flag is needed.
// Zero-filled once; every rank makes the same calls in the same order.  A
// rank is at most one call ahead of another (it waits for every other
// rank's rows of each call), so the copy it writes is never the one read.
constexpr int kMaxGatherRanks = DQ_MAX_GATHER_RANKS;
struct GatherLayout {
    size_t hdr, yfull, ybytes, total;
};
inline GatherLayout gather_layout(int rows_per) {
    GatherLayout L;
    L.hdr = 0;
    L.yfull = 256;
    L.ybytes = align256(static_cast<size_t>(kMaxGatherRanks) * rows_per * 4);
    L.total = L.yfull + 2 * L.ybytes;
    return L;
}

inline WsLayout ws_layout(int d_out, int d_in) {
    (void)d_out;
    (void)d_in;
    WsLayout W;
    W.hdr = 0;
    W.fix = 256;
    W.total = W.fix + align256(static_cast<size_t>(kMaxCtas) * 16 * sizeof(unsigned long long));
    return W;
}

// ---------------------------------------------------------------------------
// The streaming batch-1 GEMV (dq_stream.cu): tasks of at most
// kStreamTaskUnits units from a queue in the workspace.
// ---------------------------------------------------------------------------
constexpr int kStreamTaskUnits = 8;   // units per task, at most
constexpr int kStreamMaxSlots = 45;   // ring slots per CTA, at most
constexpr int kStreamConsumers = 15;  // consumer warps of a streaming CTA; ring slots are a multiple of it
constexpr int kStreamMaxRb = 16384;   // row blocks the arrival counters cover (262144 rows)

// Tasks of one shape: a row block of NC >= kStreamTaskUnits chunks is cut into
// tpr chunk ranges (one task each); shorter row blocks go m to a task.
struct StreamGeom {
    int NC, n_rb, tpr, m, n_tasks;
};
inline StreamGeom stream_geom(int d_out, int d_in) {
    StreamGeom g;
    g.NC = (d_in / 128 + kB1ChunkGroups - 1) / kB1ChunkGroups;
    g.n_rb = (d_out + 15) / 16;
    if (g.NC >= kStreamTaskUnits) {
        g.tpr = (g.NC + kStreamTaskUnits - 1) / kStreamTaskUnits;
        g.m = 1;
        g.n_tasks = g.n_rb * g.tpr;
    } else {
        g.tpr = 1;
        g.m = kStreamTaskUnits / g.NC;
        g.n_tasks = (g.n_rb + g.m - 1) / g.m;
    }
    return g;
}

// The workspace of every batch-1 and batched call starts with a fixed header
// of counters that must be zero on entry and that every call leaves zero (or,
// for the b1 kernel, tagged with the call's number); no kernel uses the
// header as scratch, so calls of any shapes can share one workspace.
//   [0, ws_layout().total)   the b1 kernel's tag, arrivals and tagged partial sums
//   stream_ctr               [0] tasks taken from the queue, [1] CTAs done
//   stream_rbcnt             [kStreamMaxRb] tasks of each row block done
//   batched_ctr              [1] the batched call's union size (written every call)
// After the header, per-shape scratch that each call overwrites.
struct WsHeader {
    size_t stream_ctr, stream_rbcnt, batched_ctr, total;
};
inline WsHeader ws_header() {
    WsHeader H;
    size_t off = ws_layout(0, 128).total;
    H.stream_ctr = off;   off += 256;
    H.stream_rbcnt = off; off += align256(static_cast<size_t>(kStreamMaxRb) * 4);
    H.batched_ctr = off;  off += 256;
    H.total = off;
    return H;
}
// The slab region of the batch-1 kernel follows the fixed header; per-shape
// scratch of the other kernels follows the slab region of the shape.
inline size_t ws_slab_offset() { return ws_header().total; }
inline size_t ws_scratch_base(int d_out, int d_in) {
    const int NC = (d_in / 128 + kB1ChunkGroups - 1) / kB1ChunkGroups;
    const int S = b1_slabs(NC);
    return ws_header().total + (S > 1 ? b1_slab_bytes(d_out, S) : 0);
}

struct StreamWs {
    size_t ctr, rbcnt, part, total;
};
inline StreamWs stream_ws(int d_out, int d_in) {
    const StreamGeom g = stream_geom(d_out, d_in);
    const WsHeader H = ws_header();
    StreamWs L;
    L.ctr = H.stream_ctr;
    L.rbcnt = H.stream_rbcnt;
    const size_t base = ws_scratch_base(d_out, d_in);
    L.part = base;
    L.total = base + (g.tpr > 1 ? align256(static_cast<size_t>(g.n_rb) * g.tpr * 64) : 0);
    return L;
}

// Shared memory of one streaming CTA (R ring slots):
//   ring   R slots of kB1UnitBytes
//   full   R mbarriers (copy landed), empty R mbarriers (slot free)
//   obbar  2 full + 2 empty mbarriers of the outlier staging buffers
//   desc   R x int4 (unit, task number, unit in task, units of the task)
//   ttab   the tasks in flight (8 x 32 bytes)
//   upart  per task in flight and unit, 16 row sums
//   misc   task counters and generations, plan flag
//   red    statistics and scan scratch
//   zero   1 KB of zeros (B operand of lanes outside their column pair)
//   xb     MMA B fragments of x' (NC chunks)
//   xp     per group (1024 sum x' even, 1024 sum x' odd, sum x', 0)
//   mask   capacity-rule mask words (split)
//   list   outliers: column | FP16 bits of x << 16 (split)
//   obuf   2 staging buffers of 512 outlier segments of 32 bytes (split)
//   otile  per consumer warp, a 16-column x 16-row tile (split)
struct SSmem {
    int ring, full, empty, obbar, desc, ttab, upart, misc, red, zero, xb, xp, mask, list, obuf, otile, total;
};
inline SSmem stream_smem(int d_in, bool split, int R) {
    const int NC = (d_in / 128 + kB1ChunkGroups - 1) / kB1ChunkGroups;
    SSmem S;
    int off = 0;
    S.ring = off;  off += R * kB1UnitBytes;
    S.full = off;  off += align16(R * 8);
    S.empty = off; off += align16(R * 8);
    S.obbar = off; off += 32;
    S.desc = off;  off += R * 16;
    S.ttab = off;  off += 8 * 32;
    S.upart = off; off += 8 * kStreamTaskUnits * 16 * 4;
    S.misc = off;  off += 128;
    S.red = off;   off += 1024;
    S.zero = off;  off += kB1ChunkB;
    S.xb = off;    off += NC * kB1ChunkB;
    S.xp = off;    off += NC * kB1ChunkGroups * 16;
    S.mask = off;  off += split ? NC * 64 : 0;
    S.list = off;  off += split ? align16(d_in) : 0;
    S.obuf = off;  off += split ? 2 * 512 * 32 : 0;
    S.otile = off; off += split ? 15 * 512 : 0;
    S.total = off;
    return S;
}

// Position of the 16-byte piece (slice sl, half h; row g + 8h of the row
// block, group t of the chunk) among the 256 pieces of a unit's packed codes.
// Within each (sl, h) block of 32 pieces, (g, t) sits at 8 t + (g ^ 2t): the
// batch-1 kernel (lane 4g + t loads its own piece) and the batched kernel
// (ldmatrix rows g = 0..7 of one group t) both touch 8 distinct 16-byte bank
// groups per shared-memory wavefront.
__host__ __device__ inline int native_piece(int sl, int h, int g, int t) {
    return (sl * 2 + h) * 32 + 8 * t + (g ^ (2 * t));
}

// Bytes of the native unit layout the GEMV kernels stream with one bulk copy
// per unit: [row-block][4-group chunk] blocks of kB1UnitBytes.
inline size_t native_bytes(int d_out, int d_in) {
    const size_t n_rb = (static_cast<size_t>(d_out) + 15) / 16;
    const size_t nc = (static_cast<size_t>(d_in / 128) + kB1ChunkGroups - 1) / kB1ChunkGroups;
    return n_rb * nc * kB1UnitBytes;
}

// ---------------------------------------------------------------------------
// Batched split GEMV (1 <= M <= 16 activation vectors, dq_batched.cu)
// ---------------------------------------------------------------------------
constexpr int kBgMaxM = 16;       // vectors per call
constexpr int kBgMaxGroups = 16;  // problems of one grouped batched call
constexpr int kBgWarps = 16;      // warps of a dense CTA (one CTA per SM)
constexpr int kBgStages = 2;      // bulk-copy ring stages per warp
constexpr int kBgOutWarps = 8;    // warps of an FP16-part CTA
constexpr int kBgOutBufs = 3;     // per-warp outlier segment buffers in flight
constexpr int kBuMaxPos = 256;    // union positions an INT4-part CTA gathers per window
constexpr double kBgPrefetchBytes = 64.0 * 1024 * 1024;  // L2 the batched INT4 part claims ahead of the plan
constexpr int kBgRefSMs = 148;    // SM count the slab width is chosen for (keeps the workspace device-independent)

// Split of one batched call.  NT tiles of 8 vectors (MP = 8 NT columns of the
// MMA); S chunks (512 columns) per slab, nslab slabs.
struct BgGeom {
    int M, NT, MP, NC, NRB, S, nslab, W;
};

inline BgGeom bg_geom(int d_out, int d_in, int M) {
    BgGeom g;
    g.M = M;
    g.NT = (M + 7) / 8;
    g.MP = 8 * g.NT;
    g.NC = (d_in / 128 + kB1ChunkGroups - 1) / kB1ChunkGroups;
    g.NRB = (d_out + 15) / 16;
    g.W = d_in / 32;
    // The x' table of a slab (S chunks x MP vectors x 1 KB) sits next to the
    // weight rings; narrower slabs when there are too few (row block, slab)
    // tasks to keep every warp of every SM streaming.
    g.S = g.NT == 1 ? 8 : 4;
    while (g.S > 1 && static_cast<long long>((g.NC + g.S - 1) / g.S) * g.NRB < kBgRefSMs * kBgWarps * 3 / 4) g.S /= 2;
    g.nslab = (g.NC + g.S - 1) / g.S;
    return g;
}

// Workspace of a batched call, after the batch-1 region (ws_layout): byte
// offsets from the start of the workspace.  All of it is scratch that a call
// writes before it reads it.
//   ctr    [0] unused (zero), [1] union size
//   masks  [kBgMaxM][W] outlier bits of each vector
//   ulist  [d_in] u16: the union of the masks, ascending columns
//   xrow   [MP][d_in] FP16: x[m][c] where column c is an outlier of vector m, else 0
//   xo     [d_in][MP] FP16: xrow[m][ulist[u]] at [u][m], u < U rounded up to 16
//   xtab   [NC][4][4][MP][4] 16-byte MMA B pieces of x' (each vector's outliers zeroed)
//   xsum   [NC][4][MP] float4 per-group sums of x'
//   dpart  [nslab][MP][d_out] FP32 per-slab partial sums of the INT4 part
struct BgWs {
    size_t ctr, masks, ulist, xrow, xo, xtab, xsum, dpart, total;
};

inline BgWs bg_ws(const BgGeom& g, int d_out, int d_in);

// Device facts cached per ordinal.
struct DeviceInfo {
    int sm_count;
    int smem_optin;
};
dq_status_t device_info(DeviceInfo* out);

void set_cuda_error(cudaError_t e);

// Kernel launchers (arguments already validated by the C ABI layer).
dq_status_t launch_gemv_b1(const dq_weights_t& w, const uint16_t* x, uint16_t* y, float k,
                           bool split, void* workspace, size_t workspace_bytes, cudaStream_t stream);
// Workspace bytes the batch-1 kernel uses for a shape (its slab region included).
size_t b1_workspace_bytes(int d_out, int d_in);
// The split GEMV with the row-sharded gather fused (native layout and mirror,
// d_out a multiple of 16): y holds g.d_total rows.
dq_status_t launch_gemv_b1_gather(const dq_weights_t& w, const uint16_t* x, uint16_t* y, float k, void* workspace,
                                  size_t workspace_bytes, const dq_gather_t& g, cudaStream_t stream);
dq_status_t launch_build_native(const uint8_t* packed, const uint16_t* scales, const uint16_t* zeros,
                                int d_out, int d_in, uint8_t* out, cudaStream_t stream);
dq_status_t read_device_error(uint32_t* word, bool clear);
dq_status_t launch_reference_gemv(const uint16_t* w16, const uint16_t* x, uint16_t* y, int d_out,
                                  int d_in, cudaStream_t stream);
dq_status_t launch_detect(const uint16_t* x, int d_in, float k, uint32_t* mask_words,
                          int32_t* indices, int32_t* count, float* stats, cudaStream_t stream);
dq_status_t launch_quantize(const uint16_t* w16, int d_out, int d_in, uint8_t* packed,
                            uint16_t* scales, uint16_t* zeros, cudaStream_t stream);
dq_status_t launch_colmajor(const uint16_t* w16, int d_out, int d_in, uint16_t* cm,
                            cudaStream_t stream);

inline BgWs bg_ws(const BgGeom& g, int d_out, int d_in) {
    BgWs L;
    const WsHeader H = ws_header();
    L.ctr = H.batched_ctr;
    size_t off = ws_scratch_base(d_out, d_in);
    L.masks = off; off += align256(static_cast<size_t>(kBgMaxM) * g.W * 4);
    L.ulist = off; off += align256(static_cast<size_t>(d_in) * 4);
    L.xrow = off;  off += align256(static_cast<size_t>(d_in) * g.MP * 2);
    L.xo = off;    off += align256(static_cast<size_t>(d_in + 16) * g.MP * 2);
    L.xtab = off;  off += align256(static_cast<size_t>(g.NC) * g.MP * 1024);
    L.xsum = off;  off += align256(static_cast<size_t>(g.NC) * 4 * g.MP * 16);
    L.dpart = off; off += align256(static_cast<size_t>(g.nslab) * g.MP * d_out * 4);
    L.total = off;
    return L;
}

bool stream_supported(const dq_weights_t& w, bool split);
dq_status_t launch_gemv_stream(const dq_weights_t& w, const uint16_t* x, uint16_t* y, float k, bool split,
                               void* workspace, cudaStream_t stream);
dq_status_t read_stream_error(uint32_t* word, bool clear);

dq_status_t launch_gemv_batched(const dq_weights_t& w, const uint16_t* x, uint16_t* y, int M, float k,
                                void* workspace, cudaStream_t stream);
// Grouped batched call: ng problems of one shape (weights w[e], m[e] vectors
// x[e] -> y[e]), problem e in the workspace region e of
// batched_grouped_region(d_out, d_in, max m) bytes.
dq_status_t launch_gemv_batched_grouped(const dq_weights_t* w, const uint16_t* const* x, uint16_t* const* y,
                                        const int32_t* m, int ng, float k, void* workspace, cudaStream_t stream);
size_t batched_grouped_region(int d_out, int d_in, int m_max);
dq_status_t read_batched_error(uint32_t* word, bool clear);
// h[r][:d] = fp16(silu(a[r][:d]) * b[r][:d]) for r < rows, a and b rows ld apart (d, ld multiples of 8).
dq_status_t launch_silu_mul(const uint16_t* a, const uint16_t* b, uint16_t* h, long long rows, long long d,
                            long long ld, cudaStream_t stream);
dq_status_t launch_combine(const uint16_t* y, const int32_t* rows, const float* weight, float* out, int m, int d,
                           cudaStream_t stream);

// Largest d_in the single-pass kernels accept (x, its B fragments and the
// outlier list live in shared memory next to the weight rings).
constexpr int kMaxDIn = 30720;

}  // namespace dq
