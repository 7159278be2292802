// FP16 GEMM on sm_100a tensor cores: C[M,N] = A[M,K] · B[N,K]^T, fp32 accumulate.
//
// Semantics follow the reference layout convention (A row-major M×K, B stored N×K
// with K contiguous, C row-major M×N; csrc/a100/gemm_8192x8192_v0.cuh:45,54,72 and
// the naive kernel csrc/h100/gemm_8192x8192_v8.cuh:347-358). Design is B200-native:
//
//   warp 0      TMA producer: A and B k-blocks (64 fp16 = one 128-B swizzle row)
//               into a STAGES-deep shared-memory ring guarded by full/empty mbarriers.
//   warp 1      TMEM owner (alloc 512 columns = two 128×256 fp32 accumulators) and,
//               in the leader CTA, the single-thread tcgen05.mma issuer.
//   warps 2..   epilogue (4 warps for single CTAs, 8 for CTA pairs): tcgen05.ld
//               (32 lanes × 32 columns) → cvt.rn fp16 → 128-B-swizzled smem staging,
//               then a TMA store (aligned C) or coalesced row stores (unaligned C);
//               predicated direct stores for v0 and the fp32 validation output.
//
// CG = 1: one CTA computes a 128×256 tile with tcgen05.mma.cta_group::1 (M=128,N=256).
// CG = 2: a CTA pair computes a 256×BN tile with tcgen05.mma.cta_group::2 (M=256,
//         N=256 per instruction). Each CTA loads its own 128 rows of A and its own
//         BN/2 rows of B with ordinary (non-multicast) TMA loads whose completion is
//         counted on the leader's barrier; the leader issues the MMAs, and
//         tcgen05.commit arrives on both CTAs' barriers. Each CTA's TMEM holds its
//         128 rows of the tile.
//
// BN = 256: the 128×256 fp32 accumulator is double-buffered in TMEM (2 × 256
//           columns), so the epilogue of tile i overlaps the main loop of tile i+1.
// BN = 512: one 128×512 accumulator fills TMEM; each K step issues two N=256 MMAs
//           (the "halves"). The epilogue hands each half back as soon as it has read
//           it, and the next tile runs half 0 ahead over the first STAGES k-blocks
//           while half 1 is still being drained. Per FLOP this moves 3/4 of the
//           L2→SMEM bytes of BN = 256 and issues half as many TMA loads.
// Tiles are visited persistently with a grouped raster.
//
// Every mbarrier wait is bounded: after `timeout_ns` without progress the waiting
// thread records a code in `vg_status_word`, raises a CTA-local abort flag and all
// roles unwind to the common exit, which still drains outstanding copies and frees
// TMEM. A healthy wait lasts microseconds.
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

#include "ptx.cuh"
#include "schedule.cuh"

namespace vg {

enum EpiKind : int {
    kEpiTmaF16 = 0,    // smem staging + TMA store (C 16-B aligned, ldc % 8 == 0)
    kEpiDirectF16 = 1, // predicated global stores (any C alignment / ldc)
    kEpiDirectF32 = 2, // fp32 output, validation build of the same main loop
    kEpiTmaF16Peers = 3, // TMA store to local C + the same rows into every peer GPU's C
    kEpiStagedF16 = 4,   // smem staging + row-cooperative coalesced stores (any C alignment)
    // Split-K with fp16 C: the kernel runs kEpiDirectF32 into an fp32 workspace and a
    // reduction kernel writes C (a launch-plan value; no kernel is built for it).
    kEpiSplitF16 = 5,
};

constexpr int kMaxPeers = 7; // peers of one node (8 GPUs per NVSwitch domain)

// Status codes written to vg_status_word (first writer wins).
enum StatusCode : unsigned {
    kStatusOk = 0,
    kStatusTimeoutProducer = 0x101,
    kStatusTimeoutMma = 0x102,
    kStatusTimeoutEpilogue = 0x103,
    kStatusTimeoutDrain = 0x104,
    kStatusTimeoutPartial = 0x105,
    kStatusTimeoutSelftest = 0x1FF,
};

struct GemmArgs {
    int M, N, K;
    int num_m_tiles; // tiles of 128*CG rows
    int num_n_tiles; // tiles of 256 columns
    int num_kb;      // ceil(K / 64)
    int group_m;     // raster group height (in M tiles)
    int c_vec_ok;    // direct epilogue may use 16-B stores
    void *C;         // direct epilogues only
    long long ldc;   // elements
    unsigned long long timeout_ns;
    // kEpiTmaF16Peers: peer GPUs' copies of this shard's rows (row 0 of the shard, ld = ldc),
    // or, when `mc` is set, the NVLink-multicast address of that row in every rank's C: one
    // multimem store reaches all ranks through the switch.
    void *peers[kMaxPeers];
    int num_peers;
    void *mc;
    // Stream-K: per-(worker, CTA rank) fp32 partial slots (128 × BN floats each, column-quad
    // major) and ready flags (zeroed before the launch).
    float *sk_partials;
    unsigned *sk_flags;
    int promote_kb; // PROMOTE kernels: k-blocks per accumulation chunk
    // DYN kernels: tile claim counter, zeroed before the launch.
    unsigned *sched_ctr;
    // Split-K (fp32 output only): the K range is cut into `splits` parts; the partial of split
    // s is written at C + s * split_stride elements. 1 = no split.
    int splits;
    long long split_stride;
};

// DYN: depth of the tile-index ring through which the leader CTA's producer hands each
// claimed tile to the other roles of the pair.
constexpr int kSchedDepth = 4;

// RSUM: the pair 256×512 tile with chunked accumulation whose running sums live in the
// epilogue warps' registers (three warpgroups: producer / MMA / two idle warps, then eight
// epilogue warps with most of the register file).
template <int CG, int BN_, bool RSUM_ = false> struct TileCfg {
    static_assert(BN_ == 256 || (BN_ == 192 && CG == 1) || (BN_ == 512 && CG == 2),
                  "tile: 128x256, 128x192, pair 256x256 or pair 256x512");
    static_assert(!RSUM_ || (CG == 2 && BN_ == 512), "register sums: the pair 256x512 tile");
    static constexpr bool RSUM = RSUM_;
    static constexpr int BM = 128;          // accumulator rows per CTA (TMEM lanes)
    static constexpr int BN = BN_;          // tile columns
    static constexpr int BK = 64;           // fp16 per 128-B swizzle row
    static constexpr int NSUB = BN > 256 ? BN / 256 : 1; // MMAs per K step (N <= 256 each)
    static constexpr int ACC_BUFS = (NSUB == 1) ? 2 : 1;
    static constexpr int NCHUNK = BN / 64; // 64-column epilogue chunks per tile
    static constexpr int B_ROWS = BN / CG;  // rows of B each CTA loads (one TMA box, <= 256)
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = B_ROWS * BK * 2;
    static constexpr int B_SUB_BYTES = B_BYTES / NSUB; // this CTA's B rows feeding one MMA
    static constexpr int STAGE_TX = CG * (A_BYTES + B_BYTES); // bytes landing per stage
    static constexpr int TMEM_COLS = 512;
    static constexpr int ACC_STRIDE = 256; // TMEM columns between the two accumulator buffers
    static constexpr uint32_t IDESC = idesc_f16_f32acc(BM * CG, BN / NSUB);
#ifndef VG_EPI_WARPS_PAIR
#define VG_EPI_WARPS_PAIR 8
#endif
    // Epilogue warps: a multiple of 4, since warp w reads TMEM lanes [32·(w % 4), +32). With
    // 4·G warps, group g = (w - 2) / 4 takes the 64-column chunks c ≡ g (mod G). CTA pairs
    // use 8: their epilogue chunks take ~1.6-2.5x as long as a single CTA's (measured), and
    // splitting a tile's chunks over two warp groups gained 3-8 % on short-K and unaligned
    // shapes; single CTAs keep 4 (8 cost them 2-3 %).
    static constexpr int EPI_WARPS = RSUM ? 8 : (CG == 2) ? VG_EPI_WARPS_PAIR : 4;
    static constexpr int EPI_GROUPS = EPI_WARPS / 4;
    static constexpr int EPI_WARP0 = RSUM ? 4 : 2; // first epilogue warp
    static constexpr int THREADS = 32 * EPI_WARP0 + 32 * EPI_WARPS;
    // RSUM register budgets per thread (launched with 168 = 65536 / 384, rounded down to a
    // multiple of 8): warpgroup 0 gives up 128 registers per thread, which the two epilogue
    // warpgroups take, 64 each (40 + 2 * 232 = 3 * 168).
    static constexpr int RSUM_REGS_LOW = 40;
    static constexpr int RSUM_REGS_HIGH = 232;
    // Chunks per TMEM release unit: a whole buffer, or one 256-column half of the BN = 512
    // accumulator.
    static constexpr int CHUNKS_PER_UNIT = (ACC_BUFS == 2) ? NCHUNK : 4;
    static constexpr int STG_BYTES = 32 * 128; // one 32-row × 64-col fp16 box
};

// Column of C (relative to the tile's first column) held in accumulator column t.
// With two MMAs per K step, MMA h reads rows [128h, 128h+128) of each CTA's B slab,
// and CTA q's slab holds C columns [256q, 256q+256) of the tile.
template <int NSUB> __host__ __device__ __forceinline__ int acc_col_to_c(int t) {
    if constexpr (NSUB == 1)
        return t;
    else
        return ((t & 255) >> 7 << 8) + ((t >> 8) << 7) + (t & 127);
}

// A-resident kernels (ARES) keep a CTA's whole A row-block of K <= kAresMaxKb k-blocks in
// shared memory, one slot per k-block, and stream only B through the pipeline stages. Four
// slots (64 KB) leave room for six 16 KB B stages and two staging boxes per epilogue warp.
constexpr int kAresMaxKb = 4;

template <int CG, int BN, int STAGES, int EPI, bool ARES = false> struct SmemLayout {
    using T = TileCfg<CG, BN>;
    static constexpr int A_SLOTS = ARES ? kAresMaxKb : STAGES;
    static constexpr int A_OFF = 0;
    static constexpr int B_OFF = A_OFF + A_SLOTS * T::A_BYTES;
    static constexpr int EPI_OFF = B_OFF + STAGES * T::B_BYTES;
    // Staging boxes per epilogue warp: two (a TMA store drains while the next box is
    // written) unless that would not leave room for the pipeline stages.
    static constexpr int kSmemLimit = 232448; // 227 KB of dynamic shared memory per CTA
    static constexpr int EPI_BUFS =
        (A_SLOTS * T::A_BYTES + STAGES * T::B_BYTES + T::EPI_WARPS * 2 * T::STG_BYTES + 2048 <= kSmemLimit)
            ? 2
            : 1;
    static constexpr int EPI_BYTES = (EPI == kEpiTmaF16 || EPI == kEpiTmaF16Peers || EPI == kEpiStagedF16)
                                         ? T::EPI_WARPS * EPI_BUFS * T::STG_BYTES
                                         : 0;
    static constexpr int BAR_OFF = EPI_OFF + EPI_BYTES;
    // full/empty per stage, tfull/tempty per accumulator, drain, the DYN ring's full/empty
    // per entry, then (ARES) full/empty per A slot.
    static constexpr int NUM_BARS = 2 * STAGES + 4 + 1 + 2 * kSchedDepth + (ARES ? 2 * kAresMaxKb : 0);
    static constexpr int SLOT_OFF = BAR_OFF + 8 * NUM_BARS;
    static constexpr int ABORT_OFF = SLOT_OFF + 4;
    static constexpr int RING_OFF = ABORT_OFF + 4; // int tile[kSchedDepth]
    static constexpr int BYTES = RING_OFF + 4 * kSchedDepth;
    static constexpr int DYN_BYTES = BYTES + 1024; // slack for 1024-B alignment
    static_assert(DYN_BYTES <= kSmemLimit, "pipeline stages do not fit in shared memory");
};

__device__ unsigned int vg_status_word;

// Back-off between barrier probes of the epilogue warps, which wait a whole main loop
// (tens of microseconds) for each accumulator; the producer and MMA warps, whose waits
// gate the tensor pipe, probe without sleeping.
#ifndef VG_EPI_BACKOFF_NS
#define VG_EPI_BACKOFF_NS 0
#endif

// The slow path of a bounded wait. Kernels that shift registers between warpgroups
// (setmaxnreg) take it inlined: a called function has one register allocation, which cannot
// serve warpgroups with different budgets (ptxas refuses such a kernel); the others share one
// out-of-line copy.
__device__ __forceinline__ bool wait_slow_inline(uint32_t bar, uint32_t parity, volatile int *abort_flag,
                                                 unsigned long long timeout_ns, unsigned code,
                                                 unsigned backoff_ns) {
    const uint64_t t0 = ptx::global_timer_ns();
    for (uint32_t it = 1;; ++it) {
        // Suspend in hardware (up to ~0.1 ms per probe) rather than spin.
        if (ptx::mbar_try_wait_sleep(bar, parity, 100000u))
            return true;
        if (backoff_ns)
            __nanosleep(backoff_ns);
        if ((it & 7u) == 0) {
            if (*abort_flag)
                return false;
            if (ptx::global_timer_ns() - t0 > timeout_ns) {
                *abort_flag = 1;
                atomicCAS(&vg_status_word, 0u, code);
                return false;
            }
        }
    }
}

__device__ __noinline__ bool wait_slow(uint32_t bar, uint32_t parity, volatile int *abort_flag,
                                       unsigned long long timeout_ns, unsigned code,
                                       unsigned backoff_ns) {
    return wait_slow_inline(bar, parity, abort_flag, timeout_ns, code, backoff_ns);
}

template <bool INLINE = false>
__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, volatile int *abort_flag,
                                         unsigned long long timeout_ns, unsigned code,
                                         unsigned backoff_ns = 0) {
    if (ptx::mbar_try_wait(bar, parity))
        return true;
    if constexpr (INLINE)
        return wait_slow_inline(bar, parity, abort_flag, timeout_ns, code, backoff_ns);
    else
        return wait_slow(bar, parity, abort_flag, timeout_ns, code, backoff_ns);
}

__device__ __forceinline__ uint32_t pack_half2(uint32_t lo_bits, uint32_t hi_bits) {
    __half2 h = __floats2half2_rn(__uint_as_float(lo_bits), __uint_as_float(hi_bits));
    return *reinterpret_cast<uint32_t *>(&h);
}

// Waits (bounded) until flag `f` reads nonzero, with GPU-scope acquire.
__device__ __forceinline__ bool wait_flag(const unsigned *f, volatile int *abort_flag,
                                          unsigned long long timeout_ns) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
    if (v)
        return true;
    const uint64_t t0 = ptx::global_timer_ns();
    for (uint32_t it = 1;; ++it) {
        __nanosleep(64);
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
        if (v)
            return true;
        if ((it & 15u) == 0) {
            if (*abort_flag)
                return false;
            if (ptx::global_timer_ns() - t0 > timeout_ns) {
                *abort_flag = 1;
                atomicCAS(&vg_status_word, 0u, (unsigned)kStatusTimeoutPartial);
                return false;
            }
        }
    }
}

// PROMOTE: each tile's K range is cut into chunks of args.promote_kb k-blocks, and the
// epilogue warps carry a running sum across them in fp32 arithmetic (round to nearest). Each
// output then sums short tensor-core chains instead of one long one (the tensor cores'
// accumulation rounds toward zero, an error that grows with the chain). With two TMEM buffers
// (BN = 256) every chunk is accumulated from zero in buffer 0 and added into the running sum
// in TMEM buffer 1. The 256×512 pair tile fills TMEM, so its running sums live in the
// registers of the eight epilogue warps (RSUM, three warpgroups: 256 sums per thread as 128
// bf16 pairs, with the register file shifted to the epilogue by setmaxnreg): at a chunk
// boundary each thread forms s = sum + chunk, keeps sum = bf16(s) and writes the remainder
// s - sum (exact in fp32) back into TMEM, on which the next chunk's MMAs accumulate. The sum
// is therefore carried without loss; the only roundings outside the tensor cores are the
// fp32 additions. The MMA issuer waits while a half is read out and written back (the other
// half's MMAs run ahead meanwhile). Every element is only ever touched by one thread, in
// chunk order (deterministic). No stream-K.
//
// DYN (CTA pairs): tiles are claimed at run time instead of by the static walk. Each pair
// starts with tile cluster_id; afterwards the leader CTA's producer claims the next tile
// with an atomic counter (args.sched_ctr, zeroed before the launch) and posts its index into
// a kSchedDepth-deep ring in both CTAs' shared memory, from which the other roles of both
// CTAs take it (full/empty mbarriers per entry; the peer's roles arrive remotely). Pairs that
// finish early take more tiles, as with hardware-placed pairs, while the epilogue of one
// tile still overlaps the next tile's main loop.
//
// ARES (A resident; the 256×256 pair with K <= kAresMaxKb k-blocks): each pair walks a
// contiguous run of tiles in row-major order, so consecutive tiles share their A row-block.
// The producer loads A once per row-block into per-k-block slots (slot k waits for the MMA
// issuer to have finished the previous row-block's last use of it) and streams only B
// through the stages; the MMA issuer frees the slots after the last tile of a row-block.
template <int CG, int BN, int STAGES, int EPI, bool SK = false, bool PROMOTE = false, bool DYN = false,
          bool ARES = false>
__global__ void __launch_bounds__((TileCfg<CG, BN, PROMOTE && BN == 512>::THREADS), 1)
    gemm_f16_tcgen05(const __grid_constant__ CUtensorMap mapA,
                     const __grid_constant__ CUtensorMap mapB,
                     const __grid_constant__ CUtensorMap mapC, const GemmArgs args) {
#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ >= 1000)
    using T = TileCfg<CG, BN, PROMOTE && BN == 512>;
    using L = SmemLayout<CG, BN, STAGES, EPI, ARES>;
    static_assert(L::T::EPI_WARPS == T::EPI_WARPS, "shared-memory layout sized for these warps");
    static_assert(!ARES || (CG == 2 && BN == 256 && !SK && !PROMOTE && !DYN),
                  "A-resident: the 256x256 pair tile with the static walk");
    constexpr int kUnitMode = SK ? kModeStreamK : (ARES ? kModeContiguous : kModeRaster);
    // Single-accumulator tiles of the static walk (v3, v6) end half by half (tfull(0), then
    // tfull(1)). Measured at 8192³: +0.4–0.7 % (burst 1514–1520 vs 1509–1510 TFLOP/s, sustained
    // 1307–1312 vs 1302–1306); with run-time claims at 32768³ (v10) it lost 1.5 % sustained.
    constexpr bool kHalfEnds = T::ACC_BUFS == 1 && !PROMOTE && !DYN;
    static_assert(!PROMOTE || ((T::ACC_BUFS == 2 || CG == 2) && !SK),
                  "PROMOTE: two TMEM buffers or the pair tile, no stream-K");
    static_assert(!DYN || (CG == 2 && !SK), "DYN: CTA pairs, no stream-K");

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const uint32_t raw = ptx::smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *const base_ptr = smem_raw + (base - raw);

    const int warp = __shfl_sync(0xffffffffu, static_cast<int>(threadIdx.x >> 5), 0);
    const int lane = static_cast<int>(threadIdx.x & 31);
    const uint32_t rank = (CG == 2) ? ptx::cluster_ctarank() : 0u;

    const uint32_t sA = base + L::A_OFF;
    const uint32_t sB = base + L::B_OFF;
    const uint32_t sEpi = base + L::EPI_OFF;
    const uint32_t sBar = base + L::BAR_OFF;
    const uint32_t slot = base + L::SLOT_OFF;
    volatile uint32_t *slot_ptr = reinterpret_cast<volatile uint32_t *>(base_ptr + L::SLOT_OFF);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(base_ptr + L::ABORT_OFF);

    auto full_bar = [&](int s) { return sBar + 8u * s; };
    auto empty_bar = [&](int s) { return sBar + 8u * (STAGES + s); };
    auto tfull_bar = [&](int a) { return sBar + 8u * (2 * STAGES + a); };
    auto tempty_bar = [&](int a) { return sBar + 8u * (2 * STAGES + 2 + a); };
    const uint32_t drain_bar = sBar + 8u * (2 * STAGES + 4);
    auto sfull_bar = [&](int i) { return sBar + 8u * (2 * STAGES + 5 + i); };
    auto sempty_bar = [&](int i) { return sBar + 8u * (2 * STAGES + 5 + kSchedDepth + i); };
    auto afull_bar = [&](int k) { return sBar + 8u * (2 * STAGES + 5 + 2 * kSchedDepth + k); };
    auto aempty_bar = [&](int k) { return sBar + 8u * (2 * STAGES + 5 + 2 * kSchedDepth + kAresMaxKb + k); };
    const uint32_t ring = base + L::RING_OFF;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            ptx::mbar_init(full_bar(s), 1);
            ptx::mbar_init(empty_bar(s), 1);
        }
        for (int a = 0; a < 2; ++a) {
            ptx::mbar_init(tfull_bar(a), 1);
            ptx::mbar_init(tempty_bar(a), T::EPI_WARPS * CG);
        }
        ptx::mbar_init(drain_bar, 1);
        if constexpr (ARES) {
            for (int k = 0; k < kAresMaxKb; ++k) {
                ptx::mbar_init(afull_bar(k), 1);
                ptx::mbar_init(aempty_bar(k), 1);
            }
        }
        // DYN ring (leader's entries are released by: its MMA thread, its epilogue warps,
        // the peer's producer and the peer's epilogue warps).
        for (int i = 0; i < kSchedDepth; ++i) {
            ptx::mbar_init(sfull_bar(i), 1);
            ptx::mbar_init(sempty_bar(i), 2 + 2 * T::EPI_WARPS);
        }
        *abort_flag = 0;
        ptx::fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        ptx::prefetch_tmap(&mapA);
        ptx::prefetch_tmap(&mapB);
        if (EPI == kEpiTmaF16 || EPI == kEpiTmaF16Peers)
            ptx::prefetch_tmap(&mapC);
    }
    if (warp == 1) {
        ptx::tmem_alloc<CG>(slot, T::TMEM_COLS);
        ptx::tmem_relinquish<CG>();
    }
    ptx::tc_fence_before();
    if constexpr (CG == 2)
        ptx::cluster_sync();
    else
        __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem_base = *slot_ptr;
    // Programmatic dependent launch: the set-up above (barriers, TMEM, descriptor
    // prefetch) may overlap the previous kernel of the stream; no global memory is read
    // or written before that kernel has completed. Every CTA is resident when it lets the
    // next grid be scheduled, so the next grid's CTAs never hold an SM that one of ours
    // still waits for. Both are no-ops without the launch attribute.
    ptx::grid_dep_wait();
    ptx::grid_dep_launch();

    const int cluster_id = static_cast<int>(blockIdx.x) / CG;
    const int num_clusters = static_cast<int>(gridDim.x) / CG;
    const unsigned long long tmo = args.timeout_ns;

    // ── DYN tile ring ──
    const int total_tiles = args.num_m_tiles * args.num_n_tiles;
    int ring_seq = 0; // entries this thread has posted or taken
    auto dyn_fill = [&](int t, WorkUnit &u) {
        raster_tile(t, args.num_m_tiles, args.num_n_tiles, args.group_m, u.tile_m, u.tile_n);
        u.kb0 = 0;
        u.kb1 = args.num_kb;
        u.kind = kUnitFull;
        u.first_contrib = u.last_contrib = -1;
        u.split = 0;
    };
    // Leader producer: claim the next tile (>= total_tiles: none left) and post it to both CTAs.
    auto ring_post = [&](int &t) -> bool {
        const int i = ring_seq % kSchedDepth;
        const uint32_t ph = static_cast<uint32_t>(ring_seq / kSchedDepth) & 1u;
        t = (ring_seq == 0) ? cluster_id : num_clusters + static_cast<int>(atomicAdd(args.sched_ctr, 1u));
        if (t > total_tiles)
            t = total_tiles;
        if (!wait_bar<T::RSUM>(sempty_bar(i), ph ^ 1u, abort_flag, tmo, kStatusTimeoutProducer))
            return false;
        ptx::st_shared_u32(ring + 4u * i, static_cast<uint32_t>(t));
        ptx::st_shared_cluster_u32(ptx::mapa(ring + 4u * i, 1), static_cast<uint32_t>(t));
        ptx::mbar_arrive(sfull_bar(i));
        ptx::mbar_arrive_cluster(ptx::mapa(sfull_bar(i), 1));
        ++ring_seq;
        return true;
    };
    // Any other role (one thread): take the next entry and release it on the leader.
    auto ring_release = [&](int i) {
        if (rank == 0)
            ptx::mbar_arrive(sempty_bar(i));
        else
            ptx::mbar_arrive_cluster(ptx::mapa(sempty_bar(i), 0));
    };
    auto ring_take = [&](int &t, unsigned code, unsigned backoff_ns) -> bool {
        const int i = ring_seq % kSchedDepth;
        const uint32_t ph = static_cast<uint32_t>(ring_seq / kSchedDepth) & 1u;
        if (!wait_bar<T::RSUM>(sfull_bar(i), ph, abort_flag, tmo, code, backoff_ns))
            return false;
        t = static_cast<int>(ptx::ld_shared_u32(ring + 4u * i));
        ring_release(i);
        ++ring_seq;
        return true;
    };

    if (warp < T::EPI_WARP0) {
        // Warpgroup 0 of the RSUM kernels (producer, MMA issuer, two idle warps) needs few
        // registers; the epilogue warpgroups hold the running sums. Each warpgroup executes
        // its setmaxnreg together, at the head of its branch.
        if constexpr (T::RSUM)
            ptx::setmaxnreg_dec<T::RSUM_REGS_LOW>();
        if (warp == 0) {
            // ───────────────────────── TMA producer ─────────────────────────
            if (lane == 0) {
                int stage = 0;
                uint32_t phase = 0;
                int issued = 0;
                bool ok = true;
                UnitIter it;
                it.init(kUnitMode, cluster_id, num_clusters, args.num_m_tiles, args.num_n_tiles, args.group_m,
                        args.num_kb, args.splits);
                WorkUnit u;
                auto next_unit = [&]() -> bool {
                    if constexpr (DYN) {
                        int t = total_tiles;
                        ok = (rank == 0) ? ring_post(t) : ring_take(t, kStatusTimeoutProducer, 0);
                        if (!ok || t >= total_tiles)
                            return false;
                        dyn_fill(t, u);
                        return true;
                    } else {
                        return it.next(u);
                    }
                };
                int a_gen = 0;            // ARES: A row-blocks loaded so far
                int a_m = -1;             // ARES: the row-block in the slots
                uint32_t a_used = 0;      // ARES: slots ever loaded
                uint32_t a_par = 0;       // ARES: parity of each slot's latest load
                auto producer_wait = [&](uint32_t bar, uint32_t parity) {
                    return wait_bar<T::RSUM>(bar, parity, abort_flag, tmo, kStatusTimeoutProducer);
                };
                while (ok && next_unit()) {
                    const int a_row = u.tile_m * (T::BM * CG) + static_cast<int>(rank) * T::BM;
                    const int b_row = u.tile_n * T::BN + static_cast<int>(rank) * T::B_ROWS;
                    const bool load_a = ARES && u.tile_m != a_m;
                    for (int kb = u.kb0; kb < u.kb1; ++kb) {
                        if constexpr (ARES) {
                            if (load_a) {
                                // Slot kb is free once the MMAs of the previous row-block's
                                // last tile have read it.
                                if (!producer_wait(aempty_bar(kb), (static_cast<uint32_t>(a_gen) & 1u) ^ 1u)) {
                                    ok = false;
                                    break;
                                }
                                const uint32_t ab = afull_bar(kb);
                                if (rank == 0)
                                    ptx::mbar_arrive_expect_tx(ab, CG * T::A_BYTES);
                                ptx::tma_load_2d_pair(sA + kb * T::A_BYTES, &mapA, ptx::mapa(ab, 0), kb * T::BK,
                                                      a_row);
                                a_used |= 1u << kb;
                                a_par = (a_par & ~(1u << kb)) | ((static_cast<uint32_t>(a_gen) & 1u) << kb);
                            }
                        }
                        if (!producer_wait(empty_bar(stage), phase ^ 1u)) {
                            ok = false;
                            break;
                        }
                        const uint32_t fb = full_bar(stage);
                        if constexpr (ARES) {
                            if (rank == 0)
                                ptx::mbar_arrive_expect_tx(fb, CG * T::B_BYTES);
                            ptx::tma_load_2d_pair(sB + stage * T::B_BYTES, &mapB, ptx::mapa(fb, 0), kb * T::BK,
                                                  b_row);
                        } else if constexpr (CG == 1) {
                            ptx::mbar_arrive_expect_tx(fb, T::STAGE_TX);
                            ptx::tma_load_2d(sA + stage * T::A_BYTES, &mapA, fb, kb * T::BK, a_row);
                            ptx::tma_load_2d(sB + stage * T::B_BYTES, &mapB, fb, kb * T::BK, b_row);
                        } else {
                            if (rank == 0)
                                ptx::mbar_arrive_expect_tx(fb, T::STAGE_TX);
                            const uint32_t leader_fb = ptx::mapa(fb, 0);
                            ptx::tma_load_2d_pair(sA + stage * T::A_BYTES, &mapA, leader_fb,
                                                  kb * T::BK, a_row);
                            ptx::tma_load_2d_pair(sB + stage * T::B_BYTES, &mapB, leader_fb,
                                                  kb * T::BK, b_row);
                        }
                        ++issued;
                        if (++stage == STAGES) {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                    if (load_a) {
                        a_m = u.tile_m;
                        ++a_gen;
                    }
                }
                // ARES: the latest load of every slot must have landed before this CTA exits
                // (true on the normal path, where the MMAs read them; bounded otherwise).
                if (ARES && rank == 0 && !ok) {
                    for (int k = 0; k < kAresMaxKb; ++k) {
                        if (!((a_used >> k) & 1u))
                            continue;
                        const uint32_t par = (a_par >> k) & 1u;
                        const uint64_t t0 = ptx::global_timer_ns();
                        while (!ptx::mbar_try_wait(afull_bar(k), par) && ptx::global_timer_ns() - t0 < tmo) {
                        }
                    }
                }
                // Drain: the most recent phase issued on each stage must have landed before
                // this CTA may exit (already true on the normal path; bounded otherwise).
                if ((CG == 1 || rank == 0) && !ok) {
                    const int n = issued < STAGES ? issued : STAGES;
                    for (int i = 0; i < n; ++i) {
                        int s = stage - 1 - i;
                        uint32_t ph = phase;
                        if (s < 0) {
                            s += STAGES;
                            ph ^= 1u;
                        }
                        if (!ptx::mbar_try_wait(full_bar(s), ph)) {
                            const uint64_t t0 = ptx::global_timer_ns();
                            while (!ptx::mbar_try_wait(full_bar(s), ph) &&
                                   ptx::global_timer_ns() - t0 < tmo) {
                            }
                        }
                    }
                }
            }
        } else if (warp == 1) {
            // ───────────────────────── MMA issuer ─────────────────────────
            if (rank == 0 && lane == 0) {
                int stage = 0;
                uint32_t phase = 0;
                int acc = 0;
                uint32_t acc_phase = 0;
                bool ok = true;
                bool any = false;
                int a_m = -1;  // ARES: the row-block whose A is in the slots
                int a_gen = 0; // ARES: row-blocks started
                auto mma_wait = [&](uint32_t bar, uint32_t parity) {
                    return wait_bar<T::RSUM>(bar, parity, abort_flag, tmo, kStatusTimeoutMma);
                };
                auto advance = [&]() {
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                };
                // MMAs of one k-block for accumulator half `h` (columns [256h, 256h+256)). `kb` counts
                // the k-blocks of the accumulation run: at 0 the first MMA overwrites D.
                auto issue = [&](uint32_t d, int h, int kb) {
                    // ARES: A from the resident slot of k-block kb, B from the stage.
                    const uint64_t a0 = ptx::smem_desc_k_sw128(sA + (ARES ? kb : stage) * T::A_BYTES);
                    const uint64_t b0 = ptx::smem_desc_k_sw128(sB + stage * T::B_BYTES + h * T::B_SUB_BYTES);
#pragma unroll
                    for (int k = 0; k < T::BK / 16; ++k) {
                        // +32 B per 16-element K step = +2 in the start-address field.
                        ptx::mma_f16<CG>(d + 256u * h, a0 + 2u * k, b0 + 2u * k, T::IDESC,
                                         (kb | k) != 0 ? 1u : 0u);
                    }
                };
                auto commit_to = [&](uint32_t bar) {
                    if constexpr (CG == 1)
                        ptx::mma_commit(bar);
                    else
                        ptx::mma_commit_pair(bar, 0x3);
                };
                UnitIter it;
                it.init(kUnitMode, cluster_id, num_clusters, args.num_m_tiles, args.num_n_tiles, args.group_m,
                        args.num_kb, args.splits);
                WorkUnit u;
                auto next_unit = [&]() -> bool {
                    if constexpr (DYN) {
                        int t = total_tiles;
                        ok = ring_take(t, kStatusTimeoutMma, 0);
                        if (!ok || t >= total_tiles)
                            return false;
                        dyn_fill(t, u);
                        return true;
                    } else {
                        return it.next(u);
                    }
                };
                while (ok && next_unit()) {
                    const int nkb = u.kb1 - u.kb0; // k-blocks of this unit; MMAs index them from 0
                    if constexpr (PROMOTE && T::ACC_BUFS == 2) {
                        for (int c0 = 0; c0 < nkb && ok; c0 += args.promote_kb) {
                            const int c1 = min(nkb, c0 + args.promote_kb);
                            if (!mma_wait(tempty_bar(0), acc_phase ^ 1u)) {
                                ok = false;
                                break;
                            }
                            ptx::tc_fence_after();
                            for (int kb = c0; kb < c1; ++kb) {
                                if (!mma_wait(full_bar(stage), phase)) {
                                    ok = false;
                                    break;
                                }
                                ptx::tc_fence_after();
                                issue(tmem_base, 0, kb - c0); // a fresh chain at each chunk start
                                any = true;
                                commit_to(empty_bar(stage));
                                advance();
                            }
                            if (!ok)
                                break;
                            commit_to(tfull_bar(0));
                            acc_phase ^= 1u;
                        }
                        if (!ok)
                            break;
                    } else if constexpr (T::ACC_BUFS == 2) {
                        if (!mma_wait(tempty_bar(acc), acc_phase ^ 1u)) {
                            ok = false;
                            break;
                        }
                        ptx::tc_fence_after();
                        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * T::ACC_STRIDE);
                        // ARES: the row-block's generation (its slots' full phase) and whether
                        // this tile is its last user (then its MMAs free the slots).
                        bool a_last = false;
                        if constexpr (ARES) {
                            if (u.tile_m != a_m) {
                                a_m = u.tile_m;
                                ++a_gen;
                            }
                            a_last = it.last_of_row(u.tile_m);
                        }
                        for (int kb = 0; kb < nkb; ++kb) {
                            if constexpr (ARES) {
                                if (!mma_wait(afull_bar(kb), static_cast<uint32_t>(a_gen - 1) & 1u)) {
                                    ok = false;
                                    break;
                                }
                            }
                            if (!mma_wait(full_bar(stage), phase)) {
                                ok = false;
                                break;
                            }
                            ptx::tc_fence_after();
                            issue(d, 0, kb);
                            any = true;
                            commit_to(empty_bar(stage));
                            if (ARES && a_last)
                                commit_to(aempty_bar(kb));
                            advance();
                        }
                        if (!ok)
                            break;
                        commit_to(tfull_bar(acc));
                        acc ^= 1;
                        if (acc == 0)
                            acc_phase ^= 1u;
                    } else {
                        // One accumulator (both halves of TMEM). PROMOTE cuts the tile's K range
                        // into chunks; otherwise one chunk = the tile. The first chunk starts from
                        // zero, every later one from the value the epilogue left in TMEM (the
                        // rounding remainder of its register-held running sum). Per chunk, half 0
                        // runs ahead over the first `run` k-blocks while the epilogue still drains
                        // half 1 of the previous chunk or tile. With kHalfEnds a tile also ends
                        // half first: its last `tail` k-blocks issue half 0, signal it on
                        // tfull(0), then issue half 1 and signal tfull(1), so the epilogue
                        // drains half 0 while the tensor pipe works through half 1's tail, and
                        // the next tile's half 0 can start as soon as that drain is done.
                        const int chunk = PROMOTE ? args.promote_kb : nkb;
                        for (int c0 = 0; c0 < nkb && ok; c0 += chunk) {
                            const int n = (nkb - c0) < chunk ? (nkb - c0) : chunk;
                            const int kb_base = (PROMOTE && c0 > 0) ? 1 : 0; // carry: accumulate
                            if (!mma_wait(tempty_bar(0), acc_phase ^ 1u)) {
                                ok = false;
                                break;
                            }
                            ptx::tc_fence_after();
                            const int run = n < STAGES ? n : STAGES;
                            const int s0 = stage;
                            const uint32_t p0 = phase;
                            for (int kb = 0; kb < run; ++kb) {
                                if (!mma_wait(full_bar(stage), phase)) {
                                    ok = false;
                                    break;
                                }
                                ptx::tc_fence_after();
                                issue(tmem_base, 0, kb_base + kb);
                                any = true;
                                advance();
                            }
                            if (!ok)
                                break;
                            if (!mma_wait(tempty_bar(1), acc_phase ^ 1u)) {
                                ok = false;
                                break;
                            }
                            ptx::tc_fence_after();
                            stage = s0;
                            phase = p0;
                            for (int kb = 0; kb < run; ++kb) {
                                issue(tmem_base, 1, kb_base + kb);
                                commit_to(empty_bar(stage));
                                advance();
                            }
                            const int tail = kHalfEnds ? min(n - run, STAGES / 2) : 0;
                            for (int kb = run; kb < n - tail; ++kb) {
                                if (!mma_wait(full_bar(stage), phase)) {
                                    ok = false;
                                    break;
                                }
                                ptx::tc_fence_after();
                                issue(tmem_base, 0, kb_base + kb);
                                issue(tmem_base, 1, kb_base + kb);
                                commit_to(empty_bar(stage));
                                advance();
                            }
                            if (!ok)
                                break;
                            if constexpr (kHalfEnds) {
                                const int s1 = stage;
                                const uint32_t p1 = phase;
                                for (int kb = n - tail; kb < n; ++kb) {
                                    if (!mma_wait(full_bar(stage), phase)) {
                                        ok = false;
                                        break;
                                    }
                                    ptx::tc_fence_after();
                                    issue(tmem_base, 0, kb_base + kb);
                                    advance();
                                }
                                if (!ok)
                                    break;
                                commit_to(tfull_bar(0));
                                stage = s1;
                                phase = p1;
                                for (int kb = n - tail; kb < n; ++kb) {
                                    issue(tmem_base, 1, kb_base + kb);
                                    commit_to(empty_bar(stage));
                                    advance();
                                }
                                commit_to(tfull_bar(1));
                            } else {
                                commit_to(tfull_bar(0));
                            }
                            acc_phase ^= 1u;
                        }
                        if (!ok)
                            break;
                    }
                }
                // Every MMA issued by this thread must complete before TMEM is freed.
                if (any) {
                    if constexpr (CG == 1)
                        ptx::mma_commit(drain_bar);
                    else
                        ptx::mma_commit_pair(drain_bar, 0x1);
                    if (!ptx::mbar_try_wait(drain_bar, 0)) {
                        const uint64_t t0 = ptx::global_timer_ns();
                        while (!ptx::mbar_try_wait(drain_bar, 0)) {
                            if (ptx::global_timer_ns() - t0 > tmo) {
                                atomicCAS(&vg_status_word, 0u, (unsigned)kStatusTimeoutDrain);
                                break;
                            }
                        }
                    }
                }
            }
        }
    } else {
        if constexpr (T::RSUM)
            ptx::setmaxnreg_inc<T::RSUM_REGS_HIGH>();
        // ───────────────────────── epilogue ─────────────────────────
        const int sub = warp & 3;           // TMEM sub-partition this warp may read
        const int ew = warp - T::EPI_WARP0; // staging-buffer owner index
        const int group = ew >> 2;          // which chunks of the tile this warp handles
        int acc = 0;
        uint32_t acc_phase = 0;
        int buf = 0;
        UnitIter it;
        it.init(kUnitMode, cluster_id, num_clusters, args.num_m_tiles, args.num_n_tiles, args.group_m,
                args.num_kb, args.splits);
        WorkUnit u;
        // Stream-K partial slot of (worker, CTA rank): 128 × BN floats.
        auto slot_of = [&](int worker) {
            return args.sk_partials + static_cast<long long>(worker * CG + static_cast<int>(rank)) *
                                          (T::BM * T::BN);
        };
        bool epi_ok = true;
        auto next_unit = [&]() -> bool {
            if constexpr (DYN) {
                // Lane 0 takes the ring entry; the warp shares it.
                int t = total_tiles, got = 1;
                if (lane == 0)
                    got = ring_take(t, kStatusTimeoutEpilogue, VG_EPI_BACKOFF_NS) ? 1 : 0;
                got = __shfl_sync(0xffffffffu, got, 0);
                t = __shfl_sync(0xffffffffu, t, 0);
                if (!got) {
                    epi_ok = false;
                    return false;
                }
                if (t >= total_tiles)
                    return false;
                dyn_fill(t, u);
                return true;
            } else {
                return it.next(u);
            }
        };
        while (epi_ok && next_unit()) {
          // PROMOTE: one pass per K chunk; only the last one stores C.
          const int nkc = PROMOTE ? (u.kb1 - u.kb0 + args.promote_kb - 1) / args.promote_kb : 1;
          const int row0 = u.tile_m * (T::BM * CG) + static_cast<int>(rank) * T::BM + sub * 32;
          const int col0 = u.tile_n * T::BN;
          const int cend = min(args.N, col0 + T::BN); // columns of this tile that exist
          const uint32_t t_row =
              tmem_base + (static_cast<uint32_t>(sub * 32) << 16) + static_cast<uint32_t>(acc * T::ACC_STRIDE);
          // Stores one 64-column chunk (accumulator chunk c, 32 rows per warp) of C in the
          // epilogue's output form.
          auto emit = [&](int c, uint32_t (&v0)[32], uint32_t (&v1)[32]) {
              const int ccol = col0 + acc_col_to_c<T::NSUB>(c * 64);
              if constexpr (EPI == kEpiStagedF16) {
                  // C rows are not 16-B aligned (N % 8 != 0 or an offset base): stage the
                  // 32 × 64 box, then write it row by row, 32 lanes covering 64 contiguous
                  // bytes per store instruction.
                  uint32_t p[32];
#pragma unroll
                  for (int i = 0; i < 16; ++i) {
                      p[i] = pack_half2(v0[2 * i], v0[2 * i + 1]);
                      p[16 + i] = pack_half2(v1[2 * i], v1[2 * i + 1]);
                  }
                  const uint32_t stg = sEpi + static_cast<uint32_t>(ew * L::EPI_BUFS * T::STG_BYTES);
                  __syncwarp(); // previous chunk's reads of this buffer are done
                  const uint32_t row_addr = stg + static_cast<uint32_t>(lane) * 128u;
#pragma unroll
                  for (int j = 0; j < 8; ++j) {
                      const uint32_t a = row_addr + (static_cast<uint32_t>(j ^ (lane & 7)) << 4);
                      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a),
                                   "r"(p[4 * j]), "r"(p[4 * j + 1]), "r"(p[4 * j + 2]),
                                   "r"(p[4 * j + 3])
                                   : "memory");
                  }
                  __syncwarp();
                  __half *cbase = static_cast<__half *>(args.C);
#pragma unroll 4
                  for (int r = 0; r < 32; ++r) {
                      const int grow = row0 + r;
                      if (grow >= args.M)
                          break;
                      __half *crow = cbase + static_cast<long long>(grow) * args.ldc;
#pragma unroll
                      for (int h = 0; h < 2; ++h) {
                          const int col = h * 32 + lane; // column within the box
                          const uint32_t a = stg + static_cast<uint32_t>(r) * 128u +
                                             (static_cast<uint32_t>((col >> 3) ^ (r & 7)) << 4) +
                                             static_cast<uint32_t>(col & 7) * 2u;
                          unsigned short bits;
                          asm volatile("ld.shared.u16 %0, [%1];" : "=h"(bits) : "r"(a));
                          if (ccol + col < cend)
                              reinterpret_cast<unsigned short *>(crow)[ccol + col] = bits;
                      }
                  }
              } else if constexpr (EPI == kEpiTmaF16 || EPI == kEpiTmaF16Peers) {
                  uint32_t p[32];
#pragma unroll
                  for (int i = 0; i < 16; ++i) {
                      p[i] = pack_half2(v0[2 * i], v0[2 * i + 1]);
                      p[16 + i] = pack_half2(v1[2 * i], v1[2 * i + 1]);
                  }
                  const uint32_t stg = sEpi + static_cast<uint32_t>((ew * L::EPI_BUFS + buf) * T::STG_BYTES);
                  if (lane == 0)
                      ptx::bulk_wait_group_read<L::EPI_BUFS - 1>();
                  __syncwarp();
                  const uint32_t row_addr = stg + static_cast<uint32_t>(lane) * 128u;
#pragma unroll
                  for (int j = 0; j < 8; ++j) {
                      const uint32_t a = row_addr + (static_cast<uint32_t>(j ^ (lane & 7)) << 4);
                      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a),
                                   "r"(p[4 * j]), "r"(p[4 * j + 1]), "r"(p[4 * j + 2]),
                                   "r"(p[4 * j + 3])
                                   : "memory");
                  }
                  ptx::fence_proxy_async_smem();
                  __syncwarp();
                  if (lane == 0) {
                      if (row0 < args.M && ccol < args.N)
                          ptx::tma_store_2d(&mapC, stg, ccol, row0);
                      ptx::bulk_commit_group();
                  }
                  if constexpr (EPI == kEpiTmaF16Peers) {
                      // Fused all-gather: the staged 32 × 64 box goes to every peer's C
                      // over NVLink, eight lanes per row so that each row leaves as one
                      // contiguous 128-B write (reads undo the 128-B swizzle).
                      const int sub_row = lane >> 3, j = lane & 7;
#pragma unroll
                      for (int i = 0; i < 8; ++i) {
                          const int r = i * 4 + sub_row;
                          const uint32_t a = stg + static_cast<uint32_t>(r) * 128u +
                                             (static_cast<uint32_t>(j ^ (r & 7)) << 4);
                          uint4 q;
                          asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                                       : "=r"(q.x), "=r"(q.y), "=r"(q.z), "=r"(q.w)
                                       : "r"(a));
                          const int grow = row0 + r;
                          const int gcol = ccol + 8 * j;
                          if (grow < args.M && gcol < cend) {
                              const long long off = static_cast<long long>(grow) * args.ldc + gcol;
                              if (args.mc) {
                                  const __half *dst = static_cast<__half *>(args.mc) + off;
                                  asm volatile("multimem.st.global.v4.f16x2 [%0], {%1, %2, %3, %4};" ::"l"(dst),
                                               "r"(q.x), "r"(q.y), "r"(q.z), "r"(q.w)
                                               : "memory");
                              } else {
                                  for (int pr = 0; pr < args.num_peers; ++pr)
                                      *reinterpret_cast<uint4 *>(static_cast<__half *>(args.peers[pr]) + off) = q;
                              }
                          }
                      }
                  }
                  buf = (buf + 1) % L::EPI_BUFS;
              } else if constexpr (EPI == kEpiDirectF16) {
                  const int row = row0 + lane;
                  if (row < args.M) {
                      __half *crow = static_cast<__half *>(args.C) + static_cast<long long>(row) * args.ldc;
#pragma unroll
                      for (int j = 0; j < 8; ++j) {
                          const uint32_t *v = (j < 4) ? (v0 + 8 * j) : (v1 + 8 * (j - 4));
                          const int col = ccol + 8 * j;
                          if (args.c_vec_ok && col + 8 <= cend) {
                              uint4 q;
                              q.x = pack_half2(v[0], v[1]);
                              q.y = pack_half2(v[2], v[3]);
                              q.z = pack_half2(v[4], v[5]);
                              q.w = pack_half2(v[6], v[7]);
                              *reinterpret_cast<uint4 *>(crow + col) = q;
                          } else {
#pragma unroll
                              for (int e = 0; e < 8; ++e)
                                  if (col + e < cend)
                                      crow[col + e] = __float2half_rn(__uint_as_float(v[e]));
                          }
                      }
                  }
              } else {
                  const int row = row0 + lane;
                  if (row < args.M) {
                      float *crow = static_cast<float *>(args.C) + u.split * args.split_stride +
                                    static_cast<long long>(row) * args.ldc;
#pragma unroll
                      for (int j = 0; j < 8; ++j) {
                          const uint32_t *v = (j < 4) ? (v0 + 8 * j) : (v1 + 8 * (j - 4));
                          const int col = ccol + 8 * j;
                          if (args.c_vec_ok && col + 8 <= cend) {
                              float4 q0 = make_float4(__uint_as_float(v[0]), __uint_as_float(v[1]),
                                                      __uint_as_float(v[2]), __uint_as_float(v[3]));
                              float4 q1 = make_float4(__uint_as_float(v[4]), __uint_as_float(v[5]),
                                                      __uint_as_float(v[6]), __uint_as_float(v[7]));
                              *reinterpret_cast<float4 *>(crow + col) = q0;
                              *reinterpret_cast<float4 *>(crow + col + 4) = q1;
                          } else {
#pragma unroll
                              for (int e = 0; e < 8; ++e)
                                  if (col + e < cend)
                                      crow[col + e] = __uint_as_float(v[e]);
                          }
                      }
                  }
              }
          };
          if constexpr (T::RSUM) {
            if (nkc > 1) {
              // This thread's running sums over the tile's chunks, as bf16 pairs (one row,
              // the warp's 256 columns: [half][chunk of the half][32-column piece][pair]).
              // Each chunk boundary rounds sum + chunk to bf16 here and leaves the exact
              // remainder in TMEM, where the next chunk's MMAs accumulate on top of it.
              constexpr int RS_CPH = T::CHUNKS_PER_UNIT / T::EPI_GROUPS;
              uint32_t rsum[T::NSUB][RS_CPH][2][16];
              auto add_sum = [](uint32_t &x0, uint32_t &x1, uint32_t pair) {
                  x0 = __float_as_uint(__uint_as_float(x0) + ptx::bf16_lo(pair));
                  x1 = __float_as_uint(__uint_as_float(x1) + ptx::bf16_hi(pair));
              };
              auto release_half = [&](int h) {
                  ptx::tc_fence_before();
                  __syncwarp();
                  if (lane == 0)
                      ptx::mbar_arrive_cluster(ptx::mapa(tempty_bar(h), 0));
              };
              for (int j = 0; j < nkc && epi_ok; ++j) {
                if (!wait_bar<T::RSUM>(tfull_bar(0), acc_phase, abort_flag, tmo, kStatusTimeoutEpilogue,
                                       VG_EPI_BACKOFF_NS)) {
                    epi_ok = false;
                    break;
                }
                ptx::tc_fence_after();
                // Per half: for each of this warp's 32-column pieces, s = sum + chunk (the
                // chunk accumulated on top of the previous remainder); not the last chunk:
                // sum = bf16(s) and TMEM = s - sum, then the half back to the MMA issuer;
                // the last chunk: the half back once loaded, C = s.
                const bool last = (j + 1 == nkc);
#pragma unroll
                for (int h = 0; h < T::NSUB; ++h) {
#pragma unroll
                    for (int i = 0; i < RS_CPH; ++i) {
                        const int c = h * T::CHUNKS_PER_UNIT + group + i * T::EPI_GROUPS;
                        if (!last) {
#pragma unroll
                            for (int p = 0; p < 2; ++p) {
                                uint32_t v[32];
                                ptx::tmem_ld_32x32b_x32(t_row + c * 64 + 32 * p, v);
                                ptx::tmem_wait_ld();
#pragma unroll
                                for (int e = 0; e < 16; ++e) {
                                    if (j > 0)
                                        add_sum(v[2 * e], v[2 * e + 1], rsum[h][i][p][e]);
                                    const float s0 = __uint_as_float(v[2 * e]);
                                    const float s1 = __uint_as_float(v[2 * e + 1]);
                                    const uint32_t r = ptx::pack_bf16x2_rn(s0, s1);
                                    rsum[h][i][p][e] = r;
                                    v[2 * e] = __float_as_uint(s0 - ptx::bf16_lo(r));
                                    v[2 * e + 1] = __float_as_uint(s1 - ptx::bf16_hi(r));
                                }
                                ptx::tmem_st_32x32b_x32(t_row + c * 64 + 32 * p, v);
                            }
                        } else {
                            uint32_t v0[32], v1[32];
                            ptx::tmem_ld_32x32b_x32(t_row + c * 64, v0);
                            ptx::tmem_ld_32x32b_x32(t_row + c * 64 + 32, v1);
                            ptx::tmem_wait_ld();
                            if (i == RS_CPH - 1)
                                release_half(h);
#pragma unroll
                            for (int e = 0; e < 16; ++e) {
                                add_sum(v0[2 * e], v0[2 * e + 1], rsum[h][i][0][e]);
                                add_sum(v1[2 * e], v1[2 * e + 1], rsum[h][i][1][e]);
                            }
                            emit(c, v0, v1);
                        }
                    }
                    if (!last) {
                        ptx::tmem_wait_st(); // the remainders are in TMEM before the hand-back
                        release_half(h);
                    }
                }
                acc_phase ^= 1u; // every chunk lands in the one accumulator
              }
              continue;
            }
          }
          for (int j = 0; j < nkc && epi_ok; ++j) {
            if (!wait_bar<T::RSUM>(tfull_bar(acc), acc_phase, abort_flag, tmo, kStatusTimeoutEpilogue,
                          VG_EPI_BACKOFF_NS)) {
                epi_ok = false;
                break;
            }
            ptx::tc_fence_after();
            // Owner of a split tile: the contributors' partials must have landed.
            if (SK && u.kind == kUnitOwner) {
                for (int c = u.first_contrib; c <= u.last_contrib && epi_ok; ++c)
                    epi_ok = wait_flag(args.sk_flags + c * CG + rank, abort_flag, tmo);
                __syncwarp();
            }
            bool drained = false; // this chunk was handled by a PROMOTE path below
            if constexpr (PROMOTE && T::ACC_BUFS == 2) {
                // The warp's chunks of buffer 0 into registers, buffer 0 back to the MMA issuer
                // at once (the next chunk's MMAs overlap the rest), then the running sum in
                // TMEM buffer 1: sum = chunk (first), sum += chunk, or C = sum + chunk (last).
                constexpr int CPW = T::NCHUNK / T::EPI_GROUPS;
                uint32_t v[CPW][2][32];
#pragma unroll
                for (int i = 0; i < CPW; ++i) {
                    const int c = group + i * T::EPI_GROUPS;
                    ptx::tmem_ld_32x32b_x32(t_row + c * 64, v[i][0]);
                    ptx::tmem_ld_32x32b_x32(t_row + c * 64 + 32, v[i][1]);
                }
                ptx::tmem_wait_ld();
                ptx::tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    if constexpr (CG == 1)
                        ptx::mbar_arrive(tempty_bar(0));
                    else
                        ptx::mbar_arrive_cluster(ptx::mapa(tempty_bar(0), 0));
                }
#pragma unroll
                for (int i = 0; i < CPW; ++i) {
                    const int c = group + i * T::EPI_GROUPS;
                    const uint32_t s_row = tmem_base + (static_cast<uint32_t>(sub * 32) << 16) +
                                           static_cast<uint32_t>(T::ACC_STRIDE + c * 64);
#pragma unroll
                    for (int p = 0; p < 2; ++p) {
                        if (j > 0) {
                            uint32_t sv[32];
                            ptx::tmem_ld_32x32b_x32(s_row + 32 * p, sv);
                            ptx::tmem_wait_ld();
#pragma unroll
                            for (int e = 0; e < 32; ++e)
                                v[i][p][e] = __float_as_uint(__uint_as_float(v[i][p][e]) + __uint_as_float(sv[e]));
                        }
                        if (j + 1 < nkc)
                            ptx::tmem_st_32x32b_x32(s_row + 32 * p, v[i][p]);
                    }
                    if (j + 1 < nkc)
                        ptx::tmem_wait_st();
                    else
                        emit(c, v[i][0], v[i][1]);
                }
                drained = true;
            }
#pragma unroll 1
            for (int c = group; c < T::NCHUNK && !drained; c += T::EPI_GROUPS) {
                if constexpr (kHalfEnds) {
                    // This warp's first chunk of half 1: wait for half 1's own completion.
                    if (c >= T::CHUNKS_PER_UNIT && c - T::EPI_GROUPS < T::CHUNKS_PER_UNIT) {
                        if (!wait_bar<T::RSUM>(tfull_bar(1), acc_phase, abort_flag, tmo,
                                               kStatusTimeoutEpilogue, VG_EPI_BACKOFF_NS)) {
                            epi_ok = false;
                            break;
                        }
                        ptx::tc_fence_after();
                    }
                }
                uint32_t v0[32], v1[32];
                ptx::tmem_ld_32x32b_x32(t_row + c * 64, v0);
                ptx::tmem_ld_32x32b_x32(t_row + c * 64 + 32, v1);
                ptx::tmem_wait_ld();
                // This warp's last read of a release unit (a whole buffer, or one half of the
                // BN=512 accumulator): hand those TMEM columns back to the MMA issuer.
                const int unit_end = (c / T::CHUNKS_PER_UNIT + 1) * T::CHUNKS_PER_UNIT;
                if (c + T::EPI_GROUPS >= unit_end) {
                    const int unit = (T::ACC_BUFS == 2) ? acc : (c / T::CHUNKS_PER_UNIT);
                    ptx::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        if constexpr (CG == 1)
                            ptx::mbar_arrive(tempty_bar(unit));
                        else
                            ptx::mbar_arrive_cluster(ptx::mapa(tempty_bar(unit), 0));
                    }
                }
                if constexpr (SK) {
                    // Partial slot layout [BN/4 column quads][128 rows][4 floats]: for a
                    // fixed quad the 32 lanes (32 consecutive rows) touch 512 contiguous
                    // bytes, so every partial store / load is one coalesced warp access.
                    const long long row_off = (static_cast<long long>(sub) * 32 + lane) * 4;
                    const long long quad0 = static_cast<long long>(c) * 16; // 64 cols = 16 quads
                    if (u.kind == kUnitPartial) {
                        float *dst = slot_of(it.w) + row_off;
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            *reinterpret_cast<uint4 *>(dst + (quad0 + q) * (T::BM * 4)) =
                                make_uint4(v0[4 * q], v0[4 * q + 1], v0[4 * q + 2], v0[4 * q + 3]);
                            *reinterpret_cast<uint4 *>(dst + (quad0 + 8 + q) * (T::BM * 4)) =
                                make_uint4(v1[4 * q], v1[4 * q + 1], v1[4 * q + 2], v1[4 * q + 3]);
                        }
                        continue;
                    }
                    if (u.kind == kUnitOwner && epi_ok) {
                        // Partials of two contributors per round trip (their 32 loads are in
                        // flight together; reading them one by one was latency-bound), added
                        // in contributor order.
                        auto add4 = [](uint32_t *v, const float4 &a) {
                            v[0] = __float_as_uint(__uint_as_float(v[0]) + a.x);
                            v[1] = __float_as_uint(__uint_as_float(v[1]) + a.y);
                            v[2] = __float_as_uint(__uint_as_float(v[2]) + a.z);
                            v[3] = __float_as_uint(__uint_as_float(v[3]) + a.w);
                        };
                        auto ld4 = [&](const float *src, long long quad) {
                            return *reinterpret_cast<const float4 *>(src + quad * (T::BM * 4));
                        };
                        int w2 = u.first_contrib;
                        for (; w2 + 1 <= u.last_contrib; w2 += 2) {
                            const float *s0 = slot_of(w2) + row_off;
                            const float *s1 = slot_of(w2 + 1) + row_off;
                            float4 a0[8], b0[8], a1[8], b1[8];
#pragma unroll
                            for (int q = 0; q < 8; ++q) {
                                a0[q] = ld4(s0, quad0 + q);
                                b0[q] = ld4(s0, quad0 + 8 + q);
                                a1[q] = ld4(s1, quad0 + q);
                                b1[q] = ld4(s1, quad0 + 8 + q);
                            }
#pragma unroll
                            for (int q = 0; q < 8; ++q) {
                                add4(v0 + 4 * q, a0[q]);
                                add4(v1 + 4 * q, b0[q]);
                                add4(v0 + 4 * q, a1[q]);
                                add4(v1 + 4 * q, b1[q]);
                            }
                        }
                        if (w2 <= u.last_contrib) {
                            const float *s0 = slot_of(w2) + row_off;
#pragma unroll
                            for (int q = 0; q < 8; ++q) {
                                add4(v0 + 4 * q, ld4(s0, quad0 + q));
                                add4(v1 + 4 * q, ld4(s0, quad0 + 8 + q));
                            }
                        }
                    }
                }
                emit(c, v0, v1);
            }
            if (SK && u.kind == kUnitPartial) {
                // All epilogue warps' partial stores, then one release of the ready flag.
                asm volatile("bar.sync 1, %0;" ::"n"(32 * T::EPI_WARPS) : "memory");
                if (warp == T::EPI_WARP0 && lane == 0) {
                    __threadfence();
                    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(args.sk_flags + it.w * CG + rank),
                                 "r"(1u)
                                 : "memory");
                }
            }
            if constexpr (PROMOTE) {
                acc_phase ^= 1u; // every chunk lands in buffer 0
            } else if constexpr (T::ACC_BUFS == 2) {
                acc ^= 1;
                if (acc == 0)
                    acc_phase ^= 1u;
            } else {
                acc_phase ^= 1u;
            }
          } // K chunks
        }
        if constexpr (EPI == kEpiTmaF16 || EPI == kEpiTmaF16Peers) {
            if (lane == 0)
                ptx::bulk_wait_group<0>();
        }
        if constexpr (EPI == kEpiTmaF16Peers)
            __threadfence_system(); // peer stores visible before the kernel's completion
        ptx::tc_fence_before();
    }

    // ───────────────────────── teardown ─────────────────────────
    __syncthreads();
    if constexpr (CG == 2)
        ptx::cluster_sync();
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc<CG>(tmem_base, T::TMEM_COLS);
    }
#endif
}

// Failure-detection self test: one CTA waits, with the same bounded wait the GEMM
// uses, on an mbarrier that nothing ever arrives on, and must come back with
// kStatusTimeoutSelftest recorded instead of hanging.
__global__ void wait_timeout_selftest(unsigned long long timeout_ns, unsigned *out_ok) {
#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ >= 1000)
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        ptx::mbar_init(ptx::smem_u32(&bar), 1);
        abort_flag = 0;
        ptx::fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const bool ok = wait_bar(ptx::smem_u32(&bar), 0, &abort_flag, timeout_ns,
                                 kStatusTimeoutSelftest);
        *out_ok = ok ? 1u : 0u;
    }
#endif
}

} // namespace vg
