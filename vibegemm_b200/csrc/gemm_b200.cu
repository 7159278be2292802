// Host side of the B200 FP16 GEMM: launch planning, TMA descriptors, the kernel
// version ladder and the C ABI declared in include/vibegemm_b200.h.
//
// Version ladder (each rung is a registered backend, following the reference's own
// methodology of keeping every kernel version in the registry,
// csrc/gemm_h100_backends.cu:56-117):
//   v0  1 CTA, 128×256 tile, one tile per CTA, direct global stores.
//   v1  1 CTA, persistent grid (one CTA per SM), grouped raster, TMEM double buffer,
//       TMA-store epilogue.
//   v2  CTA pair (tcgen05 cta_group::2), 256×256 tile, 6-stage ring, persistent
//       clusters, grouped raster, TMEM double buffer, TMA-store epilogue.
//   v3  CTA pair, 256×512 tile (one 128×512 fp32 accumulator per CTA = all of TMEM),
//       4-stage ring of 48 KB, per-half TMEM hand-back with half-0 run-ahead: 3/4 of
//       v2's L2→SMEM bytes and half its TMA loads per FLOP. Under the 1 kW power cap
//       the lower data movement keeps the SM clock ~15 % higher than v2's.
//   v4  v2's CTA-pair kernel with stream-K scheduling: the (tile, k-block) iterations
//       are split evenly over the co-resident pairs; split tiles are finished by the
//       pair holding k-block 0 from fp32 partials in a workspace. For grids with fewer
//       tiles than pair slots.
//   v5  v1 with 128×192 tiles (UMMA N=192): for grids too small to fill the GPU with
//       128×256 tiles, a third more tiles of three quarters the work.
//   v6  v3 launched with one CTA pair per tile, placed by the hardware as pairs free up
//       (no epilogue overlap, but no static tile-to-SM assignment): for very long K,
//       where the static schedule's slowest pairs set the end of the launch.
//   v7  v5 with a fifth pipeline stage (long K over under-filled grids).
//   v8  v2's 256×256 pair tile with chunked accumulation: each 4096-long K chunk is summed
//       by the tensor cores from zero and added in fp32 into a running sum in TMEM buffer 1;
//       tiles claimed at run time as in v9.
//   v9  v3's 256×512 pair tile, persistent, with tiles claimed at run time (atomic
//       counter; pairs that finish early take more tiles) and, for K >= 16384, chunked
//       accumulation whose fp32 running sum lives in a per-CTA slot in global memory.
//   v10 v9 without the chunking: one accumulation chain per output, as cuBLAS (the
//       fastest long-K kernel; bit-identical to v3/v6).
//   v11 split-K over v2's pair tile for grids with few tiles and long K: tile × K-split
//       units fill the pairs, each writes an fp32 partial, and a reduction kernel adds the
//       splits in order and stores C (deterministic; every output's chain is K / splits).
//   auto (the default entry point) picks one of them per shape (select_version).
//
// Shapes are unrestricted (M, N, K >= 0). TMA needs 16-B aligned bases and row
// strides: when A or B (K % 8 != 0 or a misaligned pointer) cannot be described,
// a pre-pass copies it into a K-padded workspace from the stream-ordered pool;
// when C cannot be (N % 8 != 0 or misaligned), the epilogue stages each box in shared
// memory and writes it row by row with coalesced 2-B stores. Partial tiles use TMA out-of-bounds zero fill and store clipping.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "b200/gemm_kernel.cuh"
#include "b200/schedule.cuh"
#include "vibegemm_b200.h"

namespace vg {
namespace {

struct VersionDesc {
    const char *name;
    int cta_group;
    int bn; // tile columns
    int stages;
    bool persistent;
    bool tma_store;
    int group_m;
    bool stream_k = false;
    bool promote = false; // chunked accumulation with an fp32 running sum (accurate long K)
    bool dyn = false;     // tiles claimed at run time (atomic counter) by the persistent pairs
    bool split_k = false; // K range split over several units, fp32 partials + reduction kernel
    bool a_resident = false; // K <= 256: A row-block kept in shared memory over contiguous tile runs
};

constexpr VersionDesc kVersions[] = {
    {"VibeGEMM B200 v0", 1, 256, 4, false, false, 8},
    {"VibeGEMM B200 v1", 1, 256, 4, true, true, 8},
    {"VibeGEMM B200 v2", 2, 256, 6, true, true, 8},
    {"VibeGEMM B200 v3", 2, 512, 4, true, true, 16},
    {"VibeGEMM B200 v4", 2, 256, 6, true, true, 8, true},
    {"VibeGEMM B200 v5", 1, 192, 4, true, true, 8},
    {"VibeGEMM B200 v6", 2, 512, 4, false, true, 16},
    {"VibeGEMM B200 v7", 1, 192, 5, true, true, 8},
    // Raster groups of the chunked kernels measured at 32768³, sustained (TFLOP/s): v8 group 4
    // 1183 vs 8 1105; v9 group 8 1303–1307 vs 16 1272–1291 vs 4 1274.
    {"VibeGEMM B200 v8", 2, 256, 6, true, true, 4, false, true, true},
    {"VibeGEMM B200 v9", 2, 512, 4, true, true, 8, false, true, true},
    {"VibeGEMM B200 v10", 2, 512, 4, true, true, 16, false, false, true},
    {"VibeGEMM B200 v11", 2, 256, 6, true, true, 8, false, false, false, true},
    // v12: v2's tile and double-buffered TMEM with A resident in shared memory for K <= 256
    // (6 B stages); above that it runs as v2.
    {"VibeGEMM B200 v12", 2, 256, 6, true, true, 8, false, false, false, false, true},
};
constexpr int kNumVersions = sizeof(kVersions) / sizeof(kVersions[0]);
constexpr int kAutoVersion = -1; // per-shape choice, the default entry point's policy

// Chunked accumulation: k-blocks (of 64) per tensor-core chunk, K = 4096. The tensor cores'
// fp32 accumulation rounds toward zero, and the error of one chain grows about linearly with
// its length: the bounded relative error |c - r| / max(|r|, 2e-2·sqrt(K/1024)) of one chain,
// on uniform[-1,1] inputs (16 sampled rows of M = N = K), is 0.82e-2 at K = 8192, 2.0e-2 at
// 16384 and 3.6e-2 at 32768 (cuBLAS's identical), and with chunks of 4096 it is 0.41e-2 at
// K = 32768 (8192-long chunks: 1.03e-2). v8 always chunks; v9 chunks from K = kPromoteMinK
// on (below it one chunk: the whole tile).
constexpr int kPromoteKb = 64;
constexpr int kPromoteMinK = 16384;

int promote_chunk_kb(int version_promote_kind, int num_kb, int Kp) {
    if (version_promote_kind == 1) // v8
        return kPromoteKb;
    if (Kp < kPromoteMinK) // v9 below the threshold: the whole tile is one chunk
        return num_kb;
    return kPromoteKb;
}

// Per-shape choice among the ladder, from the measured sweep over the BASELINE shapes:
// the 256×512 pair tile (v3) wins whenever K is not short and there is at least one
// full wave of pair tiles; short K (< 1024) favours the double-buffered 256×256 pair
// (v2), whose epilogue fully overlaps the next tile; grids too small to fill the
// pairs favour 128×256 single-CTA tiles (v1), which occupy twice as many SMs.
// Grids with fewer 256×256 tiles than pair slots cannot fill the GPU with one wave of
// pairs; among the 256×256 pair (v2), 128×256 (v1) and 128×192 (v5) tiles pick the least
// estimated time, waves × tile width / relative per-SM efficiency (pairs 1.1, 128×256 1.0,
// 128×192 0.95: measured on the BASELINE shapes), the same 128×192 tile with a fifth stage
// (v7: one staging box per epilogue warp; +14 % at 1000×3000×8192, -3..5 % at K <= 2048,
// where the shorter epilogue matters more) and stream-K (v4, only for long K over few
// tiles: its fp32 fix-up costs about 28 k-blocks per split tile).
// `allow_split` is false for the fused all-gather, which has no split-K or stream-K form and
// keeps v2 at short K.
int select_version(int M, int N, int K, int num_sms, bool allow_split = true) {
    const long long pairs = num_sms / 2;
    const long long t3 = (long long)ceil_div_i(M, 256) * ceil_div_i(N, 512);
    const long long t2 = (long long)ceil_div_i(M, 256) * ceil_div_i(N, 256);
    // From K = kPromoteMinK on every output's sum is split into chains of at most 4096 (one
    // tensor-core chain per output exceeds the 1e-2 bound from K ~ 10000 on, 3.6e-2 at
    // 32768). Over at least a wave of 256×256 tiles: v9, the 256×512 pair whose running sums
    // live in the epilogue warps' registers (sustained at 32768³ 1207–1243 TFLOP/s, level
    // with one chain, v10, at 1216–1222), or v8, the 256×256 pair with its sums in TMEM
    // (1077 there, 1.12x slower per tile), whichever needs fewer tile-waves by that ratio.
    // Over fewer tiles, split-K v11 or v8 (below).
    const bool split_chains = K >= kPromoteMinK;
    if (split_chains && t2 >= pairs) {
        const double e9 = (double)((t3 + pairs - 1) / pairs) * 512 / 1.12;
        const double e8 = (double)((t2 + pairs - 1) / pairs) * 256;
        return e9 <= e8 ? 9 : 8;
    }
    // Full waves of pair tiles: 256×512 (v3, ~6 % more work per pair-cycle than 256×256 at
    // 8192³) against 256×256 (v2), each charged for its last partial wave. Within 1.5 % v3
    // wins: it moves a quarter less data, which the estimate does not credit (8191×8193×4099:
    // estimates 0.9 % apart, v3 measured 7.8 % faster; 4096×14336×4096: 1.9 % apart, v2
    // 1.8 % faster).
    if (K >= 1024 && t3 >= pairs) {
        const double e3 = (double)((t3 + pairs - 1) / pairs) * 512 / 1.057;
        const double e2 = (double)((t2 + pairs - 1) / pairs) * 256;
        return e3 <= 1.015 * e2 ? 3 : 2;
    }
    // Short K over at least a wave of 256×256 tiles: v2, or at K <= 256 v12, v2's tile with A
    // resident in shared memory (measured against v2, TFLOP/s burst / sustained: 8192²×256
    // 827 / 715 vs 804 / 685, 8192²×128 466 / 440 vs 453 / 422, 4096×14336×256 736 / 671 vs
    // 725 / 645, 16384×8192×256 838 / 727 vs 840 / 713; at K = 384 and 512 v2 is level or ahead).
    // (The fused all-gather keeps v2 there: its peer-store epilogue is tested on v2's schedule.)
    if (t2 >= pairs)
        return (K <= 256 && allow_split) ? 12 : 2;
    // Under-filled grid: estimated time in (tile columns × k-blocks) per SM for 128×256
    // (v1), pair 256×256 (v2), 128×192 (v5) and a K split over pair tiles (estimated as
    // stream-K, v4, whose split tiles pay a fix-up of about 28 k-blocks: partials out, owner
    // reads them back, the flag reset). Splitting K wins only when K is long and the tiles are
    // few (e.g. 256×2048×32768); it also splits each output's accumulation chain.
    // Each wave also pays a fixed cost (prologue, last epilogue), in k-blocks: ~10 for single
    // CTAs and ~30 for pairs, whose main loop runs ~1.2x faster per SM (fitted to one-wave
    // runs: 2048×2048×4096 v1 1270 vs v2 1190 TFLOP/s, 512×8192×32768 v2 1335 vs v1 1161).
    const long long kb = ceil_div_i(K, 64);
    const long long t1 = (long long)ceil_div_i(M, 128) * ceil_div_i(N, 256);
    const long long t5 = (long long)ceil_div_i(M, 128) * ceil_div_i(N, 192);
    const double e2 = (double)((t2 + pairs - 1) / pairs) * 256 * (kb + 30) / 1.2;
    const double e1 = (double)((t1 + num_sms - 1) / num_sms) * 256 * (kb + 10) / 1.0;
    const double e5 = (double)((t5 + num_sms - 1) / num_sms) * 192 * (kb + 10) / 0.95;
    // (K split over the pairs only for grids at most half full: a single wave on most pairs
    // runs at a higher clock under the power cap than the estimate credits, e.g.
    // 512×8192×32768 measured v2 1320 vs v4 1047 TFLOP/s.) The estimate is stream-K's; where it
    // wins, split-K (v11, fp32 partials added in split order by a reduction kernel) was measured
    // faster than stream-K on every such shape: 256×2048×32768 754 vs 566 TFLOP/s,
    // 1024×1024×16384 856 vs 735, 256×4096×8192 590 vs 478, 1024×2048×8192 864 vs 801.
    const double e4 = (allow_split && 2 * t2 <= pairs)
                          ? (double)((t2 * kb + pairs - 1) / pairs + 28 + 10) * 256 / 1.1
                          : 1e300;
    const double e7 = e5 * (kb >= 64 ? 0.88 : 1.04);
    if (split_chains)
        return e4 <= e2 * 1.1 ? 11 : 8;
    const double best = std::min({e1, e2, e4, e5, e7});
    if (e7 == best)
        return 7;
    if (e4 == best)
        return 11;
    if (e5 == best)
        return 5;
    return e2 <= e1 ? 2 : 1;
}

constexpr int kMinSkIters = 4; // k-blocks per stream-K worker at least
constexpr int kMaxDevices = 64;
constexpr unsigned long long kDefaultTimeoutNs = 2000000000ull;

// Raster group height override (0 = the version's default). Set through
// vg_b200_set_raster_group or the VG_RASTER_GROUP_M environment variable.
std::atomic<int> g_group_override{-1};

int raster_group_override() {
    int g = g_group_override.load(std::memory_order_relaxed);
    if (g < 0) {
        g = 0;
        if (const char *env = std::getenv("VG_RASTER_GROUP_M"))
            g = std::max(0, std::atoi(env));
        g_group_override.store(g, std::memory_order_relaxed);
    }
    return g;
}

struct Plan {
    int version = 0; // resolved version (never kAutoVersion)
    int stream_k = 0;
    int cta_group = 1;
    int bn = 256;
    int stages = 4;
    int epi = kEpiTmaF16;
    int pad_a = 0, pad_b = 0;
    int Kp = 0;
    int num_m_tiles = 0, num_n_tiles = 0, num_kb = 0;
    int group_m = 8;
    int grid = 0;
    int persistent = 0;
    int promote = 0;
    int dyn = 0;
    int promote_kb = 0; // k-blocks per accumulation chunk (num_kb: one chunk)
    int splits = 1;     // split-K parts (1: none)
    int a_resident = 0; // A row-block resident in shared memory (stages = B stages)
};

inline bool aligned16(uintptr_t p) { return (p & 15u) == 0; }

// Pure host planning (no CUDA calls): what the launcher will do for this problem.
int make_plan(int version, int M, int N, int K, uintptr_t A, uintptr_t B, uintptr_t C, bool f32_out,
              int num_sms, int max_clusters, Plan &p, bool peers = false) {
    if (M < 0 || N < 0 || K < 0 || num_sms <= 0)
        return cudaErrorInvalidValue;
    if (version == kAutoVersion) // the fused all-gather epilogue has no stream-K / split-K form
        version = select_version(M, N, K, num_sms, !peers);
    if (version < 0 || version >= kNumVersions)
        return cudaErrorInvalidValue;
    const VersionDesc &v = kVersions[version];
    p = Plan{};
    p.version = version;
    p.cta_group = v.cta_group;
    p.bn = v.bn;
    p.stages = v.stages;
    p.group_m = raster_group_override() > 0 ? raster_group_override() : v.group_m;
    p.persistent = v.persistent ? 1 : 0;
    p.pad_a = (K % 8 != 0) || !aligned16(A);
    p.pad_b = (K % 8 != 0) || !aligned16(B);
    p.Kp = (K % 8 == 0) ? K : (K + 7) / 8 * 8;
    if (peers) {
        // Fused all-gather: TMA-store epilogue plus 16-B peer stores (C rows 16-B aligned).
        if (f32_out || !v.tma_store || N % 8 != 0 || !aligned16(C))
            return cudaErrorInvalidValue;
        p.epi = kEpiTmaF16Peers;
    } else if (f32_out)
        p.epi = kEpiDirectF32;
    else if (v.tma_store && N % 8 == 0 && aligned16(C))
        p.epi = kEpiTmaF16;
    else if (v.tma_store)
        p.epi = kEpiStagedF16; // C rows TMA cannot describe: staged, coalesced row stores
    else
        p.epi = kEpiDirectF16;
    p.num_m_tiles = ceil_div_i(M, 128 * v.cta_group);
    p.num_n_tiles = ceil_div_i(N, v.bn);
    p.num_kb = ceil_div_i(p.Kp, 64);
    const long long tiles = (long long)p.num_m_tiles * p.num_n_tiles;
    p.stream_k = v.stream_k ? 1 : 0;
    p.promote = v.promote ? 1 : 0;
    p.dyn = v.dyn ? 1 : 0;
    p.promote_kb = v.promote ? promote_chunk_kb(v.cta_group == 2 && v.bn == 512 ? 2 : 1, p.num_kb, p.Kp)
                             : p.num_kb;
    if (v.a_resident && p.num_kb <= kAresMaxKb)
        p.a_resident = 1; // otherwise v2's plan
    if (v.split_k) {
        // Enough K splits to give every slot (pair or SM) a unit (one wave), at least 8
        // k-blocks per split, and from K = kPromoteMinK on chains of at most kPromoteKb k-blocks.
        const int slots = (v.cta_group == 2) ? std::max(1, max_clusters) : num_sms;
        long long S = std::max(1LL, slots / std::max(1LL, tiles));
        S = std::min<long long>(S, std::max(1, p.num_kb / 8));
        if (p.Kp >= kPromoteMinK)
            S = std::max<long long>(S, ceil_div_i(p.num_kb, kPromoteKb));
        p.splits = (int)std::max(1LL, std::min<long long>(S, p.num_kb));
        if (p.splits > 1 && peers)
            return cudaErrorInvalidValue; // the all-gather epilogue has no split-K form
        if (p.splits > 1)
            p.epi = f32_out ? kEpiDirectF32 : kEpiSplitF16; // the reduction kernel's output
    }
    if (v.stream_k) {
        if (peers)
            return cudaErrorInvalidValue;
        const int slots = (v.cta_group == 2) ? std::max(1, max_clusters) : num_sms;
        const long long iters = tiles * p.num_kb;
        const long long workers = std::max(1LL, std::min<long long>(slots, iters / kMinSkIters));
        p.grid = (int)workers * v.cta_group;
    } else if (v.persistent) {
        const int slots = (v.cta_group == 2) ? std::max(1, max_clusters) : num_sms;
        p.grid = (int)std::min<long long>(tiles * p.splits, slots) * v.cta_group;
    } else {
        p.grid = (int)tiles * v.cta_group;
    }
    return cudaSuccess;
}

// ── per-device facts ─────────────────────────────────────────────────────────
struct DeviceInfo {
    int num_sms = 0;
    int major = 0, minor = 0;
    bool ok = false;
};
DeviceInfo g_dev[kMaxDevices];
std::once_flag g_dev_once[kMaxDevices];

const DeviceInfo *device_info(int dev) {
    if (dev < 0 || dev >= kMaxDevices)
        return nullptr;
    std::call_once(g_dev_once[dev], [dev] {
        DeviceInfo &d = g_dev[dev];
        if (cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) {
            (void)cudaGetLastError();
            return;
        }
        d.ok = true;
    });
    return &g_dev[dev];
}

std::atomic<unsigned long long> g_timeout_ns{0};

unsigned long long wait_timeout_ns() {
    unsigned long long t = g_timeout_ns.load(std::memory_order_relaxed);
    if (t == 0) {
        t = kDefaultTimeoutNs;
        if (const char *env = std::getenv("VG_WAIT_TIMEOUT_MS")) {
            const long long ms = std::atoll(env);
            if (ms > 0)
                t = (unsigned long long)ms * 1000000ull;
        }
        g_timeout_ns.store(t, std::memory_order_relaxed);
    }
    return t;
}

// Programmatic dependent launch of the GEMM kernels (VG_PDL=0 turns it off): the kernel's
// set-up overlaps the tail of the previous kernel in the stream, and the kernel waits for
// that kernel's completion (griddepcontrol.wait) before it touches global memory.
bool pdl_enabled() {
    static const bool on = [] {
        const char *env = std::getenv("VG_PDL");
        return !(env && env[0] == '0');
    }();
    return on;
}

// ── TMA descriptors ──────────────────────────────────────────────────────────
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                             &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            (void)cudaGetLastError();
            p = nullptr;
        }
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

struct MapKey {
    const void *base;
    uint64_t cols, rows, ld;
    uint32_t box_cols, box_rows;
    int dev;
    bool operator==(const MapKey &o) const {
        return base == o.base && cols == o.cols && rows == o.rows && ld == o.ld &&
               box_cols == o.box_cols && box_rows == o.box_rows && dev == o.dev;
    }
};

struct MapCache {
    static constexpr int kSize = 16;
    MapKey key[kSize];
    CUtensorMap map[kSize];
    int used = 0, next = 0;
    void clear() { used = next = 0; }
};
thread_local MapCache t_maps;

// Row-major fp16 matrix of `rows` × `cols` with row stride `ld` elements, loaded or
// stored in boxes of box_rows × box_cols with 128-B swizzle (box_cols·2 = 128 B).
// Out-of-range elements read as zero and are clipped on store.
bool get_map(CUtensorMap &out, const void *base, uint64_t cols, uint64_t rows, uint64_t ld,
             uint32_t box_cols, uint32_t box_rows, int dev) {
    const MapKey k{base, cols, rows, ld, box_cols, box_rows, dev};
    for (int i = 0; i < t_maps.used; ++i)
        if (t_maps.key[i] == k) {
            out = t_maps.map[i];
            return true;
        }
    EncodeTiledFn fn = encode_fn();
    if (!fn)
        return false;
    CUtensorMap m;
    std::memset(&m, 0, sizeof(m));
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {ld * sizeof(__half)};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t elem_strides[2] = {1, 1};
    const CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims,
                          strides, box, elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return false;
    const int slot = t_maps.next;
    t_maps.key[slot] = k;
    t_maps.map[slot] = m;
    t_maps.next = (slot + 1) % MapCache::kSize;
    t_maps.used = std::min(t_maps.used + 1, MapCache::kSize);
    out = m;
    return true;
}

// ── workspace pool ───────────────────────────────────────────────────────────
// Per-call workspaces (pad copies, stream-K partials) come from a stream-ordered pool
// owned by the library, one per device, that keeps its memory across synchronisations
// (release threshold = max) so repeated calls never go back to the driver.
cudaMemPool_t g_pool[kMaxDevices];
cudaError_t g_pool_err[kMaxDevices];
std::once_flag g_pool_once[kMaxDevices];

cudaError_t workspace_pool(int dev, cudaMemPool_t &pool) {
    std::call_once(g_pool_once[dev], [dev] {
        cudaMemPoolProps props{};
        props.allocType = cudaMemAllocationTypePinned;
        props.handleTypes = cudaMemHandleTypeNone;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = dev;
        cudaError_t e = cudaMemPoolCreate(&g_pool[dev], &props);
        if (e == cudaSuccess) {
            uint64_t keep = ~0ull;
            e = cudaMemPoolSetAttribute(g_pool[dev], cudaMemPoolAttrReleaseThreshold, &keep);
        }
        if (e != cudaSuccess)
            (void)cudaGetLastError();
        g_pool_err[dev] = e;
    });
    pool = g_pool[dev];
    return g_pool_err[dev];
}

// ── pad pre-pass ─────────────────────────────────────────────────────────────
// dst[r, 0:ld_dst] = src[r, 0:cols] followed by zeros; ld_dst % 8 == 0, dst 16-B
// aligned. One thread writes one 16-B group; reads are coalesced 2-B loads (src
// may be arbitrarily aligned).
__global__ void pad_rows_f16(const __half *__restrict__ src, long long rows, int cols,
                             long long ld_src, __half *__restrict__ dst, int ld_dst) {
    // Blocks stride over rows, threads over 8-element groups of a row (no index division).
    // Source rows may start on any 2-B boundary, so the loads are 2-B; the warp's loads of a
    // row cover 512 contiguous bytes per element step and coalesce in L1. Stores are 16 B.
    const int groups_per_row = ld_dst / 8;
    const unsigned short *s16 = reinterpret_cast<const unsigned short *>(src);
    for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
        const unsigned short *row = s16 + r * ld_src;
        uint4 *out = reinterpret_cast<uint4 *>(dst + r * ld_dst);
        for (int g = threadIdx.x; g < groups_per_row; g += blockDim.x) {
            const int c0 = g * 8;
            unsigned short v[8];
#pragma unroll
            for (int e = 0; e < 8; ++e)
                v[e] = (c0 + e < cols) ? row[c0 + e] : (unsigned short)0;
            uint4 q;
            q.x = v[0] | ((unsigned)v[1] << 16);
            q.y = v[2] | ((unsigned)v[3] << 16);
            q.z = v[4] | ((unsigned)v[5] << 16);
            q.w = v[6] | ((unsigned)v[7] << 16);
            out[g] = q;
        }
    }
}

cudaError_t launch_pad(const void *src, long long rows, int cols, __half *dst, int ld_dst,
                       int num_sms, cudaStream_t s) {
    if (rows == 0)
        return cudaSuccess;
    const int threads = 256;
    const int blocks = (int)std::min<long long>(rows, (long long)num_sms * 16);
    pad_rows_f16<<<blocks, threads, 0, s>>>(static_cast<const __half *>(src), rows, cols, cols, dst,
                                            ld_dst);
    return cudaGetLastError();
}

// ── split-K reduction ────────────────────────────────────────────────────────
// C[r, c] = Σ_{s = 0..S-1} ws[s][r][c] (fp32, in split order, from 0), stored as fp16 (round
// to nearest) or fp32. ws holds S row-major M × N partials. One thread per 4 consecutive
// columns of a row; 16-byte loads when N % 4 == 0.
__global__ void splitk_reduce(const float *__restrict__ ws, int S, long long stride, int M, int N,
                              void *__restrict__ C, long long ldc, int f32_out) {
    const int groups = (N + 3) / 4;
    const long long total = (long long)M * groups;
    const bool vec = (N % 4) == 0;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / groups;
        const int c0 = (int)(i - r * groups) * 4;
        const float *src = ws + r * N + c0;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int s = 0; s < S; ++s) {
            const float *p = src + (long long)s * stride;
            if (vec) {
                const float4 v = *reinterpret_cast<const float4 *>(p);
                acc[0] += v.x;
                acc[1] += v.y;
                acc[2] += v.z;
                acc[3] += v.w;
            } else {
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    if (c0 + e < N)
                        acc[e] += p[e];
            }
        }
        if (f32_out) {
            float *crow = static_cast<float *>(C) + r * ldc;
#pragma unroll
            for (int e = 0; e < 4; ++e)
                if (c0 + e < N)
                    crow[c0 + e] = acc[e];
        } else {
            __half *crow = static_cast<__half *>(C) + r * ldc;
#pragma unroll
            for (int e = 0; e < 4; ++e)
                if (c0 + e < N)
                    crow[c0 + e] = __float2half_rn(acc[e]);
        }
    }
}

cudaError_t launch_splitk_reduce(const float *ws, int S, int M, int N, void *C, long long ldc, bool f32_out,
                                 int num_sms, cudaStream_t s) {
    const long long total = (long long)M * ((N + 3) / 4);
    if (total == 0)
        return cudaSuccess;
    const int threads = 256;
    const int blocks = (int)std::min<long long>((total + threads - 1) / threads, (long long)num_sms * 8);
    splitk_reduce<<<blocks, threads, 0, s>>>(ws, S, (long long)M * N, M, N, C, ldc, f32_out ? 1 : 0);
    return cudaGetLastError();
}

// ── kernel launch ────────────────────────────────────────────────────────────
template <int CG, int BN, int STAGES, int EPI, bool SK, bool PROMOTE, bool DYN, bool ARES> struct Inst {
    using T = TileCfg<CG, BN, PROMOTE && BN == 512>;
    static constexpr int kSmem = SmemLayout<CG, BN, STAGES, EPI, ARES>::DYN_BYTES;
    static std::atomic<unsigned long long> attr_ready; // bit per device
    static int max_clusters[kMaxDevices];

    static cudaError_t prepare(int dev) {
        if ((attr_ready.load(std::memory_order_acquire) >> dev) & 1ull)
            return cudaSuccess;
        auto kern = &gemm_f16_tcgen05<CG, BN, STAGES, EPI, SK, PROMOTE, DYN, ARES>;
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
        if (e != cudaSuccess)
            return e;
        if constexpr (T::RSUM) {
            // The warpgroups' setmaxnreg budgets must fit in what the CTA is launched with, or
            // the epilogue's setmaxnreg.inc would wait forever: refuse the kernel instead.
            cudaFuncAttributes fa{};
            e = cudaFuncGetAttributes(&fa, kern);
            if (e != cudaSuccess)
                return e;
            if (T::RSUM_REGS_LOW + 2 * T::RSUM_REGS_HIGH > 3 * fa.numRegs)
                return cudaErrorInvalidConfiguration;
        }
        int clusters = 0;
        if (CG == 2) {
            cudaLaunchConfig_t cfg{};
            cfg.gridDim = dim3(2 * 1024, 1, 1);
            cfg.blockDim = dim3(T::THREADS, 1, 1);
            cfg.dynamicSmemBytes = kSmem;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = 2;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
            if (e != cudaSuccess)
                return e;
        }
        max_clusters[dev] = clusters;
        attr_ready.fetch_or(1ull << dev, std::memory_order_acq_rel);
        return cudaSuccess;
    }

    static cudaError_t launch(const CUtensorMap &ma, const CUtensorMap &mb, const CUtensorMap &mc,
                              const GemmArgs &args, int grid, cudaStream_t s) {
        auto kern = &gemm_f16_tcgen05<CG, BN, STAGES, EPI, SK, PROMOTE, DYN, ARES>;
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(grid, 1, 1);
        cfg.blockDim = dim3(T::THREADS, 1, 1);
        cfg.dynamicSmemBytes = kSmem;
        cfg.stream = s;
        cudaLaunchAttribute attr[2];
        unsigned n = 0;
        if (CG == 2) {
            attr[n].id = cudaLaunchAttributeClusterDimension;
            attr[n].val.clusterDim.x = 2;
            attr[n].val.clusterDim.y = 1;
            attr[n].val.clusterDim.z = 1;
            ++n;
        }
        if (pdl_enabled()) {
            attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[n].val.programmaticStreamSerializationAllowed = 1;
            ++n;
        }
        cfg.attrs = n ? attr : nullptr;
        cfg.numAttrs = n;
        return cudaLaunchKernelEx(&cfg, kern, ma, mb, mc, args);
    }
};
template <int CG, int BN, int STAGES, int EPI, bool SK, bool PROMOTE, bool DYN, bool ARES>
std::atomic<unsigned long long> Inst<CG, BN, STAGES, EPI, SK, PROMOTE, DYN, ARES>::attr_ready{0};
template <int CG, int BN, int STAGES, int EPI, bool SK, bool PROMOTE, bool DYN, bool ARES>
int Inst<CG, BN, STAGES, EPI, SK, PROMOTE, DYN, ARES>::max_clusters[kMaxDevices] = {};

template <int CG, int BN, int STAGES, bool SK = false, bool PROMOTE = false, bool DYN = false,
          bool ARES = false>
cudaError_t dispatch_epi(int epi, int dev, int &max_clusters, bool query_only,
                         const CUtensorMap *ma, const CUtensorMap *mb, const CUtensorMap *mc,
                         const GemmArgs *args, int grid, cudaStream_t s) {
#define VG_EPI_CASE(E)                                                                             \
    case E: {                                                                                      \
        cudaError_t e = Inst<CG, BN, STAGES, E, SK, PROMOTE, DYN, ARES>::prepare(dev);                   \
        if (e != cudaSuccess)                                                                      \
            return e;                                                                              \
        max_clusters = Inst<CG, BN, STAGES, E, SK, PROMOTE, DYN, ARES>::max_clusters[dev];               \
        if (query_only)                                                                            \
            return cudaSuccess;                                                                    \
        return Inst<CG, BN, STAGES, E, SK, PROMOTE, DYN, ARES>::launch(*ma, *mb, *mc, *args, grid, s);   \
    }
    if constexpr (SK) {
        switch (epi) {
            VG_EPI_CASE(kEpiTmaF16)
            VG_EPI_CASE(kEpiDirectF16)
            VG_EPI_CASE(kEpiDirectF32)
            VG_EPI_CASE(kEpiStagedF16)
        default:
            return cudaErrorInvalidValue;
        }
    } else {
        switch (epi) {
            VG_EPI_CASE(kEpiTmaF16)
            VG_EPI_CASE(kEpiDirectF16)
            VG_EPI_CASE(kEpiDirectF32)
            VG_EPI_CASE(kEpiTmaF16Peers)
            VG_EPI_CASE(kEpiStagedF16)
        default:
            return cudaErrorInvalidValue;
        }
    }
#undef VG_EPI_CASE
}

cudaError_t dispatch(const Plan &p, int dev, int &max_clusters, bool query_only,
                     const CUtensorMap *ma, const CUtensorMap *mb, const CUtensorMap *mc,
                     const GemmArgs *args, int grid, cudaStream_t s) {
    if (p.a_resident) // v12 with K <= 256
        return dispatch_epi<2, 256, 6, false, false, false, true>(p.epi, dev, max_clusters, query_only, ma, mb,
                                                                  mc, args, grid, s);
    if (p.cta_group == 1 && p.bn == 256 && p.stages == 4)
        return dispatch_epi<1, 256, 4>(p.epi, dev, max_clusters, query_only, ma, mb, mc, args, grid, s);
    if (p.cta_group == 1 && p.bn == 192 && p.stages == 4)
        return dispatch_epi<1, 192, 4>(p.epi, dev, max_clusters, query_only, ma, mb, mc, args, grid, s);
    if (p.promote && p.cta_group == 2 && p.bn == 256 && p.stages == 6) // v8
        return dispatch_epi<2, 256, 6, false, true, true>(p.epi, dev, max_clusters, query_only, ma, mb, mc,
                                                          args, grid, s);
    if (!p.stream_k && p.cta_group == 2 && p.bn == 256 && p.stages == 6)
        return dispatch_epi<2, 256, 6>(p.epi, dev, max_clusters, query_only, ma, mb, mc, args, grid, s);
    if (p.cta_group == 1 && p.bn == 192 && p.stages == 5)
        return dispatch_epi<1, 192, 5>(p.epi, dev, max_clusters, query_only, ma, mb, mc, args, grid, s);
    if (p.dyn && p.promote && p.cta_group == 2 && p.bn == 512 && p.stages == 4) // v9
        return dispatch_epi<2, 512, 4, false, true, true>(p.epi, dev, max_clusters, query_only, ma, mb, mc,
                                                          args, grid, s);
    if (p.dyn && !p.promote && p.cta_group == 2 && p.bn == 512 && p.stages == 4) // v10
        return dispatch_epi<2, 512, 4, false, false, true>(p.epi, dev, max_clusters, query_only, ma, mb, mc,
                                                           args, grid, s);
    if (!p.dyn && p.cta_group == 2 && p.bn == 512 && p.stages == 4) // v3 and v6 (grid differs)
        return dispatch_epi<2, 512, 4>(p.epi, dev, max_clusters, query_only, ma, mb, mc, args, grid, s);
    if (p.stream_k && p.cta_group == 2 && p.bn == 256 && p.stages == 6)
        return dispatch_epi<2, 256, 6, true>(p.epi, dev, max_clusters, query_only, ma, mb, mc, args, grid, s);
    return cudaErrorInvalidValue;
}

inline size_t round_up_256(size_t x) { return (x + 255) / 256 * 256; }

// Byte layout of a call's workspace: padded A, padded B, stream-K partials, split-K partials,
// then the words zeroed before every launch (stream-K ready flags, the run-time tile counter).
struct WsLayout {
    size_t a_off = 0, b_off = 0, part_off = 0, split_off = 0, flag_off = 0, ctr_off = 0;
    size_t flag_bytes = 0, total = 0;
};

WsLayout workspace_layout(const Plan &p, int M, int N, int grid) {
    WsLayout w;
    const size_t a = p.pad_a ? round_up_256((size_t)M * p.Kp * sizeof(__half)) : 0;
    const size_t b = p.pad_b ? round_up_256((size_t)N * p.Kp * sizeof(__half)) : 0;
    const size_t sk_slots = p.stream_k ? (size_t)grid : 0; // one per (worker, CTA rank)
    const size_t part = sk_slots * 128 * (size_t)p.bn * sizeof(float);
    // Split-K: one fp32 M × N partial per split.
    const size_t split = p.splits > 1 ? round_up_256((size_t)p.splits * M * N * sizeof(float)) : 0;
    const size_t words = sk_slots + (p.dyn ? 1 : 0);
    w.a_off = 0;
    w.b_off = a;
    w.part_off = a + b;
    w.split_off = a + b + part;
    w.flag_off = a + b + part + split;
    w.ctr_off = w.flag_off + sk_slots * sizeof(unsigned);
    w.flag_bytes = words ? round_up_256(words * sizeof(unsigned)) : 0;
    w.total = a + b + part + split + w.flag_bytes;
    return w;
}

// ── workspaces ───────────────────────────────────────────────────────────────
// Workspace of vg_b200_gemm_f16_noalloc (K-padded operands, stream-K or split-K partials,
// stream-K flags and the tile counter):
// a fixed array in the module's device memory instead of the stream-ordered pool. A GPU
// reserves these kNoAllocScratchBytes when this module is first loaded on it (with lazy
// module loading: the first GEMM call on that device) and holds them until the process
// exits. In host code the name `noalloc_scratch` is only a host-side stand-in for the
// symbol; its device address comes from cudaGetSymbolAddress, looked up per device with
// that device current.
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20; // 32 MiB
static __device__ __align__(256) unsigned char noalloc_scratch[kNoAllocScratchBytes];

// Device address of the array on device `dev` (current). A successful lookup is kept; a
// failed one is returned to the caller and tried again on the next call.
std::atomic<void *> g_scratch[kMaxDevices];
std::mutex g_scratch_mu;

cudaError_t noalloc_scratch_addr(int dev, void *&out) {
    out = g_scratch[dev].load(std::memory_order_acquire);
    if (out)
        return cudaSuccess;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    out = g_scratch[dev].load(std::memory_order_acquire);
    if (out)
        return cudaSuccess;
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, noalloc_scratch);
    if (e != cudaSuccess || !p) {
        (void)cudaGetLastError();
        out = nullptr;
        return e != cudaSuccess ? e : cudaErrorInvalidSymbol;
    }
    g_scratch[dev].store(p, std::memory_order_release);
    out = p;
    return cudaSuccess;
}

// Where a call's workspace (K-padded operands, stream-K partials and flags) lives: the
// library's stream-ordered pool (allocated and freed on the caller's stream) or the fixed
// no-allocation array (nothing is allocated; problems that need more return
// VG_ERROR_NOALLOC_SCRATCH_LIMIT).
enum class WsSource { Pool, Scratch };

// One GEMM launch: validation, plan, workspace, pre-passes, tensor maps, kernel.
// Returns a cudaError_t value or VG_ERROR_NOALLOC_SCRATCH_LIMIT.
int launch_gemm(int version, const void *A, const void *B, void *C, int M, int N, int K,
                bool f32_out, cudaStream_t s, void *const *peers, int num_peers, void *c_multicast,
                WsSource src) {
    if ((version != kAutoVersion && (version < 0 || version >= kNumVersions)) || M < 0 || N < 0 || K < 0)
        return cudaErrorInvalidValue;
    if (M == 0 || N == 0)
        return cudaSuccess;
    if (!C)
        return cudaErrorInvalidValue;
    const size_t out_elt = f32_out ? sizeof(float) : sizeof(__half);
    if (K == 0) // empty sum: C = 0 (A and B may be empty allocations)
        return cudaMemsetAsync(C, 0, (size_t)M * N * out_elt, s);
    if (!A || !B)
        return cudaErrorInvalidValue;

    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess)
        return e;
    const DeviceInfo *di = device_info(dev);
    if (!di || !di->ok)
        return cudaErrorInvalidDevice;
    if (di->major != 10 || di->minor != 0)
        return cudaErrorNoKernelImageForDevice;

    if (num_peers < 0 || num_peers > kMaxPeers)
        return cudaErrorInvalidValue;
    for (int i = 0; i < num_peers; ++i)
        if (!peers || !peers[i] || !aligned16((uintptr_t)peers[i]))
            return cudaErrorInvalidValue;
    if (c_multicast && (num_peers == 0 || !aligned16((uintptr_t)c_multicast)))
        return cudaErrorInvalidValue;
    Plan p;
    e = (cudaError_t)make_plan(version, M, N, K, (uintptr_t)A, (uintptr_t)B, (uintptr_t)C, f32_out,
                               di->num_sms, di->num_sms / 2, p, num_peers > 0);
    if (e != cudaSuccess)
        return e;

    // The kernel that runs: split-K writes fp32 partials (its plan's epilogue names the
    // reduction kernel's output).
    Plan pk = p;
    if (p.splits > 1)
        pk.epi = kEpiDirectF32;
    // Occupancy-limited cluster count for the persistent pair kernel.
    int max_clusters = 0;
    e = dispatch(pk, dev, max_clusters, true, nullptr, nullptr, nullptr, nullptr, 0, s);
    if (e != cudaSuccess)
        return e;
    int grid = p.grid;
    if (p.cta_group == 2 && p.persistent && max_clusters > 0)
        grid = std::min(grid, 2 * max_clusters);

    // One workspace: K-padded copies of operands TMA cannot describe, and the stream-K
    // partial slots + ready flags (zeroed here, every launch).
    const void *A_use = A, *B_use = B;
    const int Kp = p.Kp;
    const WsLayout wl = workspace_layout(p, M, N, grid);
    if (src == WsSource::Scratch && wl.total > kNoAllocScratchBytes)
        return VG_ERROR_NOALLOC_SCRATCH_LIMIT;
    void *owned = nullptr; // pool allocation to free after the launch
    float *sk_partials = nullptr;
    unsigned *sk_flags = nullptr;
    unsigned *sched_ctr = nullptr;
    float *split_ws = nullptr;
    if (wl.total) {
        char *base = nullptr;
        if (src == WsSource::Pool) {
            cudaMemPool_t pool;
            e = workspace_pool(dev, pool);
            if (e == cudaSuccess)
                e = cudaMallocFromPoolAsync(&owned, wl.total, pool, s);
            if (e != cudaSuccess)
                return e;
            base = static_cast<char *>(owned);
        } else {
            void *sc = nullptr;
            e = noalloc_scratch_addr(dev, sc);
            if (e != cudaSuccess)
                return e;
            base = static_cast<char *>(sc);
        }
        __half *wa = reinterpret_cast<__half *>(base + wl.a_off);
        __half *wb = reinterpret_cast<__half *>(base + wl.b_off);
        if (p.pad_a) {
            e = launch_pad(A, M, K, wa, Kp, di->num_sms, s);
            A_use = wa;
        }
        if (e == cudaSuccess && p.pad_b) {
            e = launch_pad(B, N, K, wb, Kp, di->num_sms, s);
            B_use = wb;
        }
        if (p.stream_k) {
            sk_partials = reinterpret_cast<float *>(base + wl.part_off);
            sk_flags = reinterpret_cast<unsigned *>(base + wl.flag_off);
        }
        if (p.splits > 1)
            split_ws = reinterpret_cast<float *>(base + wl.split_off);
        if (p.dyn)
            sched_ctr = reinterpret_cast<unsigned *>(base + wl.ctr_off);
        if (e == cudaSuccess && wl.flag_bytes)
            e = cudaMemsetAsync(base + wl.flag_off, 0, wl.flag_bytes, s);
        if (e != cudaSuccess) {
            if (owned)
                (void)cudaFreeAsync(owned, s);
            return e;
        }
    }

    CUtensorMap ma, mb, mc;
    std::memset(&mc, 0, sizeof(mc));
    const uint32_t b_box_rows = (uint32_t)(p.bn / p.cta_group);
    bool ok = get_map(ma, A_use, (uint64_t)Kp, (uint64_t)M, (uint64_t)Kp, 64u, 128u, dev) &&
              get_map(mb, B_use, (uint64_t)Kp, (uint64_t)N, (uint64_t)Kp, 64u, b_box_rows, dev);
    if (ok && p.splits == 1 && (p.epi == kEpiTmaF16 || p.epi == kEpiTmaF16Peers))
        ok = get_map(mc, C, (uint64_t)N, (uint64_t)M, (uint64_t)N, 64u, 32u, dev);
    if (!ok) {
        if (owned)
            (void)cudaFreeAsync(owned, s);
        return cudaErrorInvalidValue;
    }

    GemmArgs args{};
    args.M = M;
    args.N = N;
    args.K = Kp;
    args.num_m_tiles = p.num_m_tiles;
    args.num_n_tiles = p.num_n_tiles;
    args.num_kb = p.num_kb;
    args.group_m = p.group_m;
    args.c_vec_ok = (N % (f32_out ? 4 : 8) == 0) && aligned16((uintptr_t)C);
    args.C = C;
    args.ldc = N;
    args.timeout_ns = wait_timeout_ns();
    args.sk_partials = sk_partials;
    args.sk_flags = sk_flags;
    args.promote_kb = p.promote_kb;
    args.sched_ctr = sched_ctr;
    args.num_peers = num_peers;
    for (int i = 0; i < num_peers; ++i)
        args.peers[i] = peers[i];
    args.mc = c_multicast;
    args.splits = 1;

    if (p.splits > 1) {
        // Split-K: the kernel writes each split's fp32 partial into the workspace (row-major,
        // ld = N), then the reduction kernel adds the splits in order and writes C.
        args.C = split_ws;
        args.ldc = N;
        args.c_vec_ok = (N % 4 == 0);
        args.splits = p.splits;
        args.split_stride = (long long)M * N;
        e = dispatch(pk, dev, max_clusters, false, &ma, &mb, &mc, &args, grid, s);
        if (e == cudaSuccess)
            e = launch_splitk_reduce(split_ws, p.splits, M, N, C, N, f32_out, di->num_sms, s);
    } else {
        e = dispatch(p, dev, max_clusters, false, &ma, &mb, &mc, &args, grid, s);
    }
    if (owned) {
        const cudaError_t f = cudaFreeAsync(owned, s);
        if (e == cudaSuccess)
            e = f;
    }
    return e;
}

cudaError_t run_gemm(int version, const void *A, const void *B, void *C, int M, int N, int K,
                     bool f32_out, cudaStream_t s, void *const *peers = nullptr, int num_peers = 0,
                     void *c_multicast = nullptr) {
    return (cudaError_t)launch_gemm(version, A, B, C, M, N, K, f32_out, s, peers, num_peers,
                                    c_multicast, WsSource::Pool);
}

// The default entry point's launch with the workspace in the fixed array.
int run_gemm_noalloc(const void *A, const void *B, void *C, int M, int N, int K, cudaStream_t s) {
    return launch_gemm(kAutoVersion, A, B, C, M, N, K, false, s, nullptr, 0, nullptr,
                       WsSource::Scratch);
}

} // namespace
} // namespace vg

// ── C ABI ────────────────────────────────────────────────────────────────────
extern "C" {

int vg_b200_gemm_f16_version(int version, const void *A, const void *B, void *C, int M, int N,
                             int K, vg_stream_t stream) {
    return (int)vg::run_gemm(version, A, B, C, M, N, K, false, (cudaStream_t)stream);
}

int vg_b200_gemm_f16(const void *A, const void *B, void *C, int M, int N, int K,
                     vg_stream_t stream) {
    return (int)vg::run_gemm(vg::kAutoVersion, A, B, C, M, N, K, false, (cudaStream_t)stream);
}

int vg_b200_gemm_f16_f32out(int version, const void *A, const void *B, float *C, int M, int N,
                            int K, vg_stream_t stream) {
    return (int)vg::run_gemm(version, A, B, C, M, N, K, true, (cudaStream_t)stream);
}

int vg_b200_gemm_f16_noalloc(const void *A, const void *B, void *C, int M, int N, int K,
                             vg_stream_t stream) {
    return vg::run_gemm_noalloc(A, B, C, M, N, K, (cudaStream_t)stream);
}

int vg_b200_gemm_f16_allgather(const void *A_local, const void *B, void *const *C_ranks,
                               void *C_multicast, int world, int rank, long long row0, int M_local,
                               int N, int K, vg_stream_t stream) {
    // K == 0 would only zero the local rows (the kernel, which also writes the peers' rows,
    // never runs), so it is rejected instead of leaving the other ranks' copies stale.
    if (!C_ranks || world < 1 || world > vg::kMaxPeers + 1 || rank < 0 || rank >= world || row0 < 0 ||
        M_local < 0 || N < 0 || K <= 0)
        return (int)cudaErrorInvalidValue;
    const size_t off = (size_t)row0 * (size_t)N * sizeof(__half);
    void *peers[vg::kMaxPeers];
    int np = 0;
    for (int r = 0; r < world; ++r) {
        if (!C_ranks[r])
            return (int)cudaErrorInvalidValue;
        if (r != rank)
            peers[np++] = static_cast<char *>(C_ranks[r]) + off;
    }
    void *C_local = static_cast<char *>(C_ranks[rank]) + off;
    void *c_mc = C_multicast ? static_cast<char *>(C_multicast) + off : nullptr;
    return (int)vg::run_gemm(vg::kAutoVersion, A_local, B, C_local, M_local, N, K, false,
                             (cudaStream_t)stream, peers, np, c_mc);
}

int vg_b200_num_versions(void) { return vg::kNumVersions; }

const char *vg_b200_version_name(int version) {
    if (version == vg::kAutoVersion)
        return "VibeGEMM B200 auto";
    if (version < 0 || version >= vg::kNumVersions)
        return nullptr;
    return vg::kVersions[version].name;
}

int vg_b200_default_version(void) { return vg::kAutoVersion; }

int vg_b200_is_available(int device) {
    const vg::DeviceInfo *di = vg::device_info(device);
    if (!di || !di->ok || di->major != 10 || di->minor != 0)
        return 0;
    cudaFuncAttributes fa;
    int prev = 0;
    if (cudaGetDevice(&prev) != cudaSuccess) {
        (void)cudaGetLastError();
        return 0;
    }
    if (prev != device && cudaSetDevice(device) != cudaSuccess) {
        (void)cudaGetLastError();
        return 0;
    }
    const cudaError_t e = cudaFuncGetAttributes(&fa, vg::gemm_f16_tcgen05<2, 256, 6, vg::kEpiTmaF16>);
    if (prev != device)
        (void)cudaSetDevice(prev);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        return 0;
    }
    return 1;
}

void vg_b200_teardown(void) { vg::t_maps.clear(); }

unsigned vg_b200_device_status(int reset) {
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, vg::vg_status_word, sizeof(v)) != cudaSuccess) {
        (void)cudaGetLastError();
        return 0xFFFFFFFFu;
    }
    if (reset) {
        const unsigned zero = 0;
        if (cudaMemcpyToSymbol(vg::vg_status_word, &zero, sizeof(zero)) != cudaSuccess)
            (void)cudaGetLastError();
    }
    return v;
}

int vg_b200_set_raster_group(int group_m) {
    if (group_m < 0)
        return (int)cudaErrorInvalidValue;
    vg::g_group_override.store(group_m, std::memory_order_relaxed);
    return 0;
}

int vg_b200_set_wait_timeout_ns(unsigned long long ns) {
    vg::g_timeout_ns.store(ns == 0 ? vg::kDefaultTimeoutNs : ns, std::memory_order_relaxed);
    return 0;
}

int vg_b200_selftest_wait_timeout(unsigned long long timeout_ns) {
    unsigned *d_ok = nullptr;
    if (cudaMalloc(&d_ok, sizeof(unsigned)) != cudaSuccess) {
        (void)cudaGetLastError();
        return 0;
    }
    const unsigned sentinel = 7;
    int result = 0;
    (void)vg_b200_device_status(1);
    if (cudaMemcpy(d_ok, &sentinel, sizeof(unsigned), cudaMemcpyHostToDevice) == cudaSuccess) {
        vg::wait_timeout_selftest<<<1, 32>>>(timeout_ns, d_ok);
        unsigned ok = sentinel;
        if (cudaDeviceSynchronize() == cudaSuccess &&
            cudaMemcpy(&ok, d_ok, sizeof(unsigned), cudaMemcpyDeviceToHost) == cudaSuccess) {
            const unsigned status = vg_b200_device_status(1);
            result = (ok == 0u && status == (unsigned)vg::kStatusTimeoutSelftest) ? 1 : 0;
        }
    }
    (void)cudaGetLastError();
    cudaFree(d_ok);
    return result;
}

void vg_shard_rows(long long M, int world, int rank, long long *row0, long long *rows) {
    long long r0 = 0, n = 0;
    if (world > 0 && rank >= 0 && rank < world && M > 0)
        vg::shard_rows(M, world, rank, r0, n);
    if (row0)
        *row0 = r0;
    if (rows)
        *rows = n;
}

int vg_work_units(int stream_k, int worker, int workers, int num_m, int num_n, int group_m,
                  int num_kb, int splits, int *out, int max_units) {
    if (worker < 0 || workers <= 0 || worker >= workers || num_m <= 0 || num_n <= 0 ||
        group_m <= 0 || num_kb <= 0 || max_units < 0 || splits < 1 || stream_k < 0 || stream_k > 2 ||
        (stream_k != 0 && splits != 1))
        return -1;
    vg::UnitIter it;
    it.init(stream_k, worker, workers, num_m, num_n, group_m, num_kb, splits);
    vg::WorkUnit u;
    int n = 0;
    while (it.next(u)) {
        if (out && n < max_units) {
            int *o = out + 8 * n;
            o[0] = u.tile_m;
            o[1] = u.tile_n;
            o[2] = u.kb0;
            o[3] = u.kb1;
            o[4] = u.kind;
            o[5] = u.first_contrib;
            o[6] = u.last_contrib;
            o[7] = u.split;
        }
        ++n;
    }
    return n;
}

void vg_raster_tile(int t, int num_m, int num_n, int group_m, int *tile_m, int *tile_n) {
    int tm = -1, tn = -1;
    if (num_m > 0 && num_n > 0 && group_m > 0 && t >= 0 && t < num_m * num_n)
        vg::raster_tile(t, num_m, num_n, group_m, tm, tn);
    if (tile_m)
        *tile_m = tm;
    if (tile_n)
        *tile_n = tn;
}

int vg_b200_plan(int version, int M, int N, int K, uintptr_t A, uintptr_t B, uintptr_t C,
                 int mode, int num_sms, int *out) {
    if (mode < 0 || mode > 2)
        return (int)cudaErrorInvalidValue;
    vg::Plan p;
    const int e = vg::make_plan(version, M, N, K, A, B, C, mode == 1, num_sms, num_sms / 2, p,
                                mode == 2);
    if (e != 0 || !out)
        return e ? e : (int)cudaErrorInvalidValue;
    const int vals[20] = {p.cta_group, p.stages,      p.epi,         p.pad_a,   p.pad_b,
                          p.Kp,        p.num_m_tiles, p.num_n_tiles, p.num_kb,  p.group_m,
                          p.grid,      p.persistent,  p.bn,          p.version, p.stream_k,
                          p.promote,   p.dyn,         p.promote_kb,  p.splits,  p.a_resident};
    std::memcpy(out, vals, sizeof(vals));
    return 0;
}

} // extern "C"
