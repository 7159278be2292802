// Tile scheduling shared by the device kernels and the host planner/tests.
//
// A persistent CTA (or CTA pair) walks the linear tile index space
// t = cluster_id, cluster_id + num_clusters, ... and maps every t to a tile
// (tile_m, tile_n) with a grouped raster: `group_m` consecutive M tiles are swept
// together along N, so the ~#SM tiles in flight at any moment share a band of A
// row-blocks and a band of B column-blocks that fits in L2. The same role as the
// grouped `Schedule` of the H100 family (csrc/h100/gemm_8192x8192_v18.cuh:207-260),
// written as a closed-form bijection so that no tile is dropped or repeated for any
// (num_m, num_n, group_m), including ragged last groups.
#pragma once

#ifndef VG_HD
#if defined(__CUDACC__)
#define VG_HD __host__ __device__ __forceinline__
#else
#define VG_HD inline
#endif
#endif

namespace vg {

VG_HD int ceil_div_i(int a, int b) { return (a + b - 1) / b; }

// t in [0, num_m*num_n) -> (tile_m, tile_n). Bijective for group_m >= 1.
VG_HD void raster_tile(int t, int num_m, int num_n, int group_m, int &tile_m, int &tile_n) {
    const int per_group = group_m * num_n;
    const int g = t / per_group;
    const int first_m = g * group_m;
    const int rem_m = num_m - first_m;
    const int gsize = rem_m < group_m ? rem_m : group_m;
    const int r = t - g * per_group;
    tile_m = first_m + r % gsize;
    tile_n = r / gsize;
}

// ── work units of the persistent workers ──────────────────────────────────────
// A unit is tile (tile_m, tile_n) restricted to k-blocks [kb0, kb1).
//   data-parallel: worker w takes whole tiles w, w+P, w+2P, ... (grouped raster).
//   split-K:       the same walk over T·S units, T tiles times S splits of the K range:
//                  unit u is tile u % T (raster) over k-blocks [s·KB/S, (s+1)·KB/S) with
//                  s = u / T, whose fp32 partial goes to split s of a workspace.
//   stream-K:      the T·KB (tile, k-block) iterations are cut into P equal contiguous
//                  ranges, [w·W/P, (w+1)·W/P) with W = T·KB, walked in order. A unit that
//                  starts inside a tile (kb0 > 0) is PARTIAL: its fp32 accumulator goes to
//                  workspace slot w. A unit that holds a split tile's k-block 0 is the
//                  OWNER: it adds the partials of workers first_contrib..last_contrib and
//                  stores C. A worker's partial unit can only be its first unit and its
//                  owner unit only its last, so an owner waits only on later workers'
//                  first units: no cycle.
//   contiguous:    worker w takes the whole tiles [w·T/P, (w+1)·T/P) in row-major order
//                  (tile_n fastest), so consecutive tiles of a worker share their A
//                  row-block (the A-resident kernel keeps it in shared memory).
enum UnitMode : int { kModeRaster = 0, kModeStreamK = 1, kModeContiguous = 2 };
enum UnitKind : int { kUnitFull = 0, kUnitPartial = 1, kUnitOwner = 2 };

struct WorkUnit {
    int tile_m, tile_n, kb0, kb1, kind;
    int first_contrib, last_contrib; // owner units: workers holding the other k-blocks
    int split;                       // split-K: which K split (0 otherwise)
};

struct UnitIter {
    int mode;
    bool sk;
    int w, P, num_m, num_n, group_m, KB, S;
    long long i, end, W; // stream-K position
    int t;               // data-parallel position
    int t_end;           // contiguous: one past this worker's last tile

    VG_HD void init(int unit_mode, int worker, int workers, int nm, int nn, int gm, int kb,
                    int splits = 1) {
        mode = unit_mode;
        sk = unit_mode == kModeStreamK;
        w = worker;
        P = workers;
        num_m = nm;
        num_n = nn;
        group_m = gm;
        KB = kb;
        S = splits < 1 ? 1 : splits;
        W = (long long)nm * nn * kb;
        i = begin_of(w);
        end = begin_of(w + 1);
        t = w;
        if (mode == kModeContiguous) {
            const long long T = (long long)nm * nn;
            t = (int)(T * w / P);
            t_end = (int)(T * (w + 1) / P);
        }
    }
    // Contiguous mode: whether the tile `next` returns after the current one (if any) is in
    // a different M row-block, i.e. the current tile is the last user of its A row-block.
    VG_HD bool last_of_row(int tile_m) const { return t >= t_end || t / num_n != tile_m; }
    VG_HD long long begin_of(int worker) const { return (long long)worker * W / P; }
    // Worker whose range contains iteration index `idx`.
    VG_HD int worker_of(long long idx) const { return (int)(((idx + 1) * P + W - 1) / W) - 1; }

    VG_HD bool next(WorkUnit &u) {
        if (mode == kModeContiguous) {
            if (t >= t_end)
                return false;
            u.tile_m = t / num_n;
            u.tile_n = t - u.tile_m * num_n;
            u.kb0 = 0;
            u.kb1 = KB;
            u.kind = kUnitFull;
            u.first_contrib = u.last_contrib = -1;
            u.split = 0;
            ++t;
            return true;
        }
        if (!sk) {
            const int T = num_m * num_n;
            if (t >= T * S)
                return false;
            const int s = t / T;
            raster_tile(t - s * T, num_m, num_n, group_m, u.tile_m, u.tile_n);
            u.kb0 = (int)((long long)s * KB / S);
            u.kb1 = (int)((long long)(s + 1) * KB / S);
            u.kind = kUnitFull;
            u.first_contrib = u.last_contrib = -1;
            u.split = s;
            t += P;
            return true;
        }
        if (i >= end)
            return false;
        const int tile = (int)(i / KB);
        const int k0 = (int)(i % KB);
        const long long left = end - i;
        const int k1 = (k0 + left < KB) ? (int)(k0 + left) : KB;
        raster_tile(tile, num_m, num_n, group_m, u.tile_m, u.tile_n);
        u.kb0 = k0;
        u.kb1 = k1;
        u.split = 0;
        u.first_contrib = u.last_contrib = -1;
        if (k0 == 0 && k1 == KB) {
            u.kind = kUnitFull;
        } else if (k0 == 0) {
            u.kind = kUnitOwner;
            u.first_contrib = w + 1;
            u.last_contrib = worker_of((long long)(tile + 1) * KB - 1);
        } else {
            u.kind = kUnitPartial;
        }
        i += k1 - k0;
        return true;
    }
};

// Contiguous row-block shard of M rows over `world` ranks: rank r owns rows
// [r*ceil(M/world), min(M, (r+1)*ceil(M/world))). Ranks past the end own 0 rows.
VG_HD void shard_rows(long long M, int world, int rank, long long &row0, long long &rows) {
    const long long per = (M + world - 1) / world;
    long long lo = per * rank;
    long long hi = lo + per;
    if (lo > M) lo = M;
    if (hi > M) hi = M;
    row0 = lo;
    rows = hi - lo;
}

} // namespace vg
