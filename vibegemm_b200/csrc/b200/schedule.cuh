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
