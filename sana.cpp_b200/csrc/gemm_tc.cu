// Tensor-core GEMM for sm_100a: tcgen05.mma (kind::f16, bf16 x bf16 -> fp32 in TMEM),
// operands staged by TMA (cp.async.bulk.tensor, 128-byte swizzle, no multicast), a
// persistent warp-specialised pipeline and the fused epilogue of gemm.h.
//
//   warp 0      TMA producer (one lane): A tile [128 x 64] and B tile [BN x 64] per stage
//   warp 1      TMEM allocator + MMA issuer (one lane): 4 x (128 x BN x 16) MMAs per stage
//   warps 2..9  epilogue: two warps per 32-lane TMEM quarter, each taking half of the tile's
//               columns; tcgen05.ld, bias/act/gate/residual, stores to global, with the
//               residual / gate of the next 16 columns fetched while the current ones finish
// Two TMEM accumulators (2 x BN fp32 columns) let the epilogue of one tile overlap the
// MMAs of the next. Every mbarrier wait is bounded (common.cuh); on expiry the kernel
// records kTimeout in the device error word, drains its own TMA copies and MMAs with
// bounded waits, frees TMEM and returns.
#include <cuda.h>

#include <atomic>
#include <cstdlib>
#include <mutex>

#include "gemm.h"
#include "tcgen05.cuh"
#include "tma.h"

namespace sana {
namespace tc {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one swizzle row

// Bytes of one residual chunk (32 rows x 16 fp32); a configuration sets how many each
// epilogue warp keeps in flight.
constexpr int kRingChunk = 32 * 16 * 4;
constexpr int kEpiWarpsCfg = 8;
constexpr int kEpiStageBytes = 32 * 64;  // one staging buffer: 32 rows x 64 bytes
constexpr int kSideWarpBytes = 2 * 128 * 4;  // bias and gate of a warp's (at most 128) columns

// Shared-memory layout of a CTA: [A stages][B stages][epilogue staging (8 warps x kStoreBufs
// x 2 KB)][residual ring (8 warps x kRing x 2 KB) and side vectors (8 warps x 1 KB), residual
// epilogues only][barriers][tmem slot]. Residual epilogues are HBM-bound, so they trade
// pipeline stages for the residual ring and for staging buffers, which their TMA stores
// drain asynchronously; long-K residual products (the deep variant) keep more stages and a
// shallower ring instead, their epilogue having time to spare.
template <int kStagesV, int kABytesV, int kBBytesV, bool kResid, int kStoreBufsV = 1, int kRingV = 3>
struct Layout {
    static constexpr int kRing = kRingV;
    static constexpr int kStages = kStagesV;
    static constexpr int kABytes = kABytesV;
    static constexpr int kBBytes = kBBytesV;
    static constexpr int kStoreBufs = kStoreBufsV;
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kEpiOffset = kStages * kStageBytes;
    static constexpr int kRingOffset = kEpiOffset + kEpiWarpsCfg * kStoreBufs * kEpiStageBytes;
    static constexpr int kRingBytes = kResid ? kEpiWarpsCfg * kRingV * kRingChunk : 0;
    static constexpr int kSideOffset = kRingOffset + kRingBytes;  // per warp: its span's bias and gate row
    static constexpr int kSideBytes = kResid ? kEpiWarpsCfg * kSideWarpBytes : 0;
    static constexpr int kBarOffset = kSideOffset + kSideBytes;
    static constexpr int kBars = 2 * kStages + 5 + (kResid ? kEpiWarpsCfg * kRingV : 0);
    static constexpr int kSmemBytes = kBarOffset + kBars * 8 + 16 + 1024;
    static_assert(kSmemBytes <= 232448, "shared memory of one CTA");
};

template <int BN, bool kResid = false>
struct Cfg : Layout<kResid ? (BN == 128 ? 4 : 3) : (BN == 128 ? 6 : (BN == 192 ? 5 : 4)), BM * BK * 2, BN * BK * 2,
                    kResid, kResid ? (BN == 128 ? 2 : 1) : 1> {
    static constexpr int kTmemCols = 2 * BN <= 256 ? 256 : 512;  // power of two >= two accumulators
};

// --- CTA-pair (cta_group::2) primitives ---------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// All threads of both CTAs of the cluster (release / acquire).
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The shared::cluster address of this CTA's shared-memory address `a` in CTA `rank`.
__device__ __forceinline__ uint32_t mapa(uint32_t a, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void tmem_alloc2(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish2() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// M = 256 across the pair: rows 0-127 of A and columns [0, N/2) of B from the issuing CTA's
// shared memory, rows 128-255 and columns [N/2, N) from the peer's, at the same addresses.
__device__ __forceinline__ void umma2_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrives on the barrier at the same offset in both CTAs once this thread's MMAs complete.
__device__ __forceinline__ void umma2_commit_both(uint32_t bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            bar),
        "h"(static_cast<uint16_t>(3))
        : "memory");
}
__device__ __forceinline__ void umma2_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}
// TMA load into this CTA's shared memory that completes its bytes on `bar_cluster`, a
// barrier of either CTA of the pair (here always the leader's). No multicast.
__device__ __forceinline__ void tma_load_2d_pair(const CUtensorMap* map, uint32_t dst, uint32_t bar_cluster, int c0,
                                                 int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
        "%4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1)
        : "memory");
}

// The same for a 4-D box (implicit-convolution A tiles: channels, x, y, image).
__device__ __forceinline__ void tma_load_4d_pair(const CUtensorMap* map, uint32_t dst, uint32_t bar_cluster, int c0,
                                                 int c1, int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
        "%4, %5, %6}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

// Geometry of an implicit-convolution A operand (ConvA) as the producer uses it.
struct ConvGeom {
    int H = 0, W = 0, cchunks = 0, kw = 1, oy = 0, ox = 0;
    int pair = 0, cin = 0;  // pixel-pair rows: tap column e reads super-pixel floor(e/2), channels (e & 1) * cin
};

// --- epilogue -------------------------------------------------------------------------
__device__ __forceinline__ void store_val(void* out, int is_bf16, long long idx, float v) {
    if (is_bf16) {
        static_cast<bf16*>(out)[idx] = __float2bfloat16_rn(v);
    } else {
        static_cast<float*>(out)[idx] = v;
    }
}

// Residual and gate values of 16 consecutive columns [n0, n0+16) of one row.
struct Side16 {
    float r[16];
    float g[16];
};

// v = resid + gate * v on 16 columns, as fused multiply-adds on pairs.
__device__ __forceinline__ void resid16(float (&v)[16], const float (&rv)[16], const float (&gv)[16]) {
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
        const float2 y = f2_split(fma2(f2_make(gv[j], gv[j + 1]), f2_make(v[j], v[j + 1]), f2_make(rv[j], rv[j + 1])));
        v[j] = y.x;
        v[j + 1] = y.y;
    }
}

// Bias, activation and gated residual on 16 consecutive columns [n0, n0+16) of one row,
// all of them in range (the fast path); the stores are the caller's.
template <bool kResid>
__device__ __forceinline__ void compute16(const Epilogue& ep, const float (&bv)[16], float (&v)[16],
                                          const float (&rv)[16], const float (&gv)[16]) {
    if (ep.act == kActSilu) {  // bias and SiLU on pairs
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
            uint64_t x = f2_make(v[j], v[j + 1]);
            if (ep.bias) x = add2(x, f2_make(bv[j], bv[j + 1]));
            const float2 y = f2_split(silu2(x));
            v[j] = y.x;
            v[j + 1] = y.y;
        }
        if (kResid) resid16(v, rv, gv);
        return;
    }
    if (ep.bias) {
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
            const float2 y = f2_split(add2(f2_make(v[j], v[j + 1]), f2_make(bv[j], bv[j + 1])));
            v[j] = y.x;
            v[j + 1] = y.y;
        }
    }
    if (ep.act == kActGelu) {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = gelu_tanh(v[j]);
    }
    if (kResid) resid16(v, rv, gv);
}

// --- coalesced stores through a per-warp staging block ----------------------------------
// Each lane holds one row of the tile; storing straight from there writes 32 rows x 16 bytes
// per instruction. Instead a warp writes its 32 rows x 64 bytes into shared memory and
// stores them back as 8 rows x 64 bytes per instruction (full 32-byte sectors). 16-byte slot
// k of row r sits at slot 4r + (k ^ ((r >> 1) & 3)): both the row writes and the row-group
// reads then touch eight distinct bank groups per quarter-warp.
__device__ __forceinline__ uint32_t stage_slot(int r, int k) { return static_cast<uint32_t>(4 * r + (k ^ ((r >> 1) & 3))) * 16u; }

// The lane's 64 bytes (4 x 16) into its staging row.
__device__ __forceinline__ void stage_put(uint8_t* stg, int lane, const uint4 (&w)[4]) {
#pragma unroll
    for (int k = 0; k < 4; ++k) *reinterpret_cast<uint4*>(stg + stage_slot(lane, k)) = w[k];
}
// The staged 32 x 64 bytes to global rows row0 .. row0+31 (rows >= M skipped) at byte
// offset col_bytes of rows ld_bytes apart.
__device__ __forceinline__ void stage_flush(const uint8_t* stg, int lane, uint8_t* gout, long long ld_bytes,
                                            long long col_bytes, int row0, int M) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = 8 * i + lane / 4, k = lane % 4;
        if (row0 + r < M)
            *reinterpret_cast<uint4*>(gout + static_cast<long long>(row0 + r) * ld_bytes + col_bytes + 16 * k) =
                *reinterpret_cast<const uint4*>(stg + stage_slot(r, k));
    }
}
__device__ __forceinline__ void pack_bf16x16(const float (&v)[16], uint4 (&w)[2]) {
    uint32_t* u = reinterpret_cast<uint32_t*>(w);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
        u[j] = *reinterpret_cast<uint32_t*>(&h);
    }
}
// Stores 32 columns [n0, n0+32) of the warp's 32 rows to one output (bf16 or fp32).
__device__ __forceinline__ void store32(uint8_t* stg, int lane, void* out, int is_bf16, long long ld, int row0,
                                        int M, int n0, const float (&v0)[16], const float (&v1)[16]) {
    uint8_t* g = static_cast<uint8_t*>(out);
    if (is_bf16) {
        uint4 w[4];
        pack_bf16x16(v0, *reinterpret_cast<uint4(*)[2]>(&w[0]));
        pack_bf16x16(v1, *reinterpret_cast<uint4(*)[2]>(&w[2]));
        stage_put(stg, lane, w);
        __syncwarp();
        stage_flush(stg, lane, g, ld * 2, static_cast<long long>(n0) * 2, row0, M);
        __syncwarp();
    } else {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const float(&v)[16] = h ? v1 : v0;
            uint4 w[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) w[k] = make_uint4(__float_as_uint(v[4 * k]), __float_as_uint(v[4 * k + 1]),
                                                          __float_as_uint(v[4 * k + 2]), __float_as_uint(v[4 * k + 3]));
            stage_put(stg, lane, w);
            __syncwarp();
            stage_flush(stg, lane, g, ld * 4, static_cast<long long>(n0 + 16 * h) * 4, row0, M);
            __syncwarp();
        }
    }
}

// Applies the epilogue to 16 consecutive columns [n0, n0+16) of one row.
template <bool kResid>
__device__ __forceinline__ void epilogue16(const Epilogue& ep, int row, int n0, int N, float (&v)[16], bool vec,
                                           const Side16& sd) {
    const bool full = vec && n0 + 16 <= N;
    if (ep.bias) {
        if (full) {
#pragma unroll
            for (int j = 0; j < 16; j += 4) {
                const float4 b = *reinterpret_cast<const float4*>(ep.bias + n0 + j);
                v[j] += b.x;
                v[j + 1] += b.y;
                v[j + 2] += b.z;
                v[j + 3] += b.w;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (n0 + j < N) v[j] += ep.bias[n0 + j];
        }
    }
    if (ep.act == kActSilu) {
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
            const float2 y = f2_split(silu2(f2_make(v[j], v[j + 1])));
            v[j] = y.x;
            v[j + 1] = y.y;
        }
    } else if (ep.act == kActGelu) {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = gelu_tanh(v[j]);
    }
    if (kResid) {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = sd.r[j] + sd.g[j] * v[j];
    }
    if (full) {
        void* outs[2] = {ep.out, ep.out2};
        const int bfs[2] = {ep.out_bf16, ep.out2_bf16};
        const long long lds[2] = {ep.ldo, ep.ldo2};
#pragma unroll
        for (int o = 0; o < 2; ++o) {
            if (!outs[o]) continue;
            if (o == 1 && ep.act2 == kActSilu) {
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = silu(v[j]);
            }
            const long long base = static_cast<long long>(row) * lds[o] + n0;
            if (bfs[o]) {
                uint4 pk[2];
                uint32_t* w = reinterpret_cast<uint32_t*>(pk);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
                    w[j] = *reinterpret_cast<uint32_t*>(&h);
                }
                uint4* dst = reinterpret_cast<uint4*>(static_cast<bf16*>(outs[o]) + base);
                dst[0] = pk[0];
                dst[1] = pk[1];
            } else {
                float4* dst = reinterpret_cast<float4*>(static_cast<float*>(outs[o]) + base);
#pragma unroll
                for (int j = 0; j < 4; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            }
        }
        return;
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const int n = n0 + j;
        if (n >= N) break;
        const float x = v[j];
        if (ep.out) store_val(ep.out, ep.out_bf16, static_cast<long long>(row) * ep.ldo + n, x);
        if (ep.out2) store_val(ep.out2, ep.out2_bf16, static_cast<long long>(row) * ep.ldo2 + n,
                               ep.act2 == kActSilu ? silu(x) : x);
    }
}

// The residual chunks an epilogue warp will need, in the order it needs them: chunk j is the
// warp's 32 rows x 16 fp32 columns number j % kchunks of its span of the (j / kchunks)-th
// tile it processes. Lane 0 keeps `depth` chunks in flight with TMA (64-byte swizzle: 16-byte
// slot k of row r lands at stage_slot(r, k), so each lane reads its own row without bank
// conflicts); every lane takes the chunks in order. Boxes past M or N read as zeros.
struct ResidRing {
    const CUtensorMap* map;
    const uint8_t* buf;   // slot 0, generic address
    uint32_t buf_s, bar;  // slot 0 and its barrier, shared-window addresses
    int first, stride, num_tiles, num_n, bn, tile_rows, row_off, col0, kchunks;
    int issued, used;
    int* err;
    // the next chunk to issue: its tile, its index in the span, the span's origin in that tile
    int it_tile = 0, it_chunk = 0, it_x = 0, it_y = 0;
    int depth = 3;  // chunks in flight

    __device__ void set_tile() {
        it_x = (it_tile % num_n) * bn + col0;
        it_y = (it_tile / num_n) * tile_rows + row_off;
    }
    // Lane 0: positions the cursor on the first chunk and fills the ring.
    __device__ void start() {
        it_tile = first;
        it_chunk = 0;
        if (it_tile < num_tiles) set_tile();
        refill();
    }
    // Lane 0: keeps the ring full.
    __device__ void refill() {
        while (issued < used + depth && it_tile < num_tiles) {
            const uint32_t s = static_cast<uint32_t>(issued % depth);
            mbar_arrive_expect_tx(bar + 8u * s, kRingChunk);
            tma_load_2d(map, buf_s + s * kRingChunk, bar + 8u * s, it_x + 16 * it_chunk, it_y);
            ++issued;
            if (++it_chunk == kchunks) {
                it_chunk = 0;
                it_tile += stride;
                if (it_tile < num_tiles) set_tile();
            }
        }
    }
    // Every lane: its row of the next chunk. A wait that gives up has recorded the error.
    __device__ void take(float (&rv)[16]) {
        const int lane = threadIdx.x & 31;
        const uint32_t s = static_cast<uint32_t>(used % depth);
        if (mbar_wait(bar + 8u * s, static_cast<uint32_t>((used / depth) & 1), err, kTimeout)) {
            const uint8_t* b = buf + s * kRingChunk;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint4 w = *reinterpret_cast<const uint4*>(b + stage_slot(lane, k));
                rv[4 * k] = __uint_as_float(w.x);
                rv[4 * k + 1] = __uint_as_float(w.y);
                rv[4 * k + 2] = __uint_as_float(w.z);
                rv[4 * k + 3] = __uint_as_float(w.w);
            }
        }
        __syncwarp();  // the slot is free once every lane has read it
        ++used;
        if (lane == 0) refill();
    }
    // Lane 0: waits (bounded) for chunks issued and never taken, so no copy lands after exit.
    __device__ void drain() {
        for (int j = used; j < issued; ++j)
            mbar_wait_quiet(bar + 8u * static_cast<uint32_t>(j % depth), static_cast<uint32_t>((j / depth) & 1));
    }
};

// The gate values of one row's 16 columns (1 when the epilogue has no gate).
__device__ __forceinline__ void gate16(const Epilogue& ep, int row, int n0, float (&gv)[16]) {
    if (ep.gate) {
        const float* g = ep.gate + static_cast<long long>(row / ep.rows_per_gate) * ep.gate_ld + n0;
#pragma unroll
        for (int j = 0; j < 16; j += 4) {
            const float4 v = *reinterpret_cast<const float4*>(g + j);
            gv[j] = v.x;
            gv[j + 1] = v.y;
            gv[j + 2] = v.z;
            gv[j + 3] = v.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) gv[j] = 1.f;
    }
}

// A warp's output staging for TMA stores: kBufs buffers of 32 rows x 64 bytes in the layout of
// stage_slot (the 64-byte swizzle of the output tensor maps), used round robin. Before a
// buffer is rewritten, lane 0 waits until the store that last read it has finished reading
// (at most kBufs - 1 younger stores pending); every lane fences its writes to the async
// proxy, and lane 0 issues the store of the box at (x, y).
template <int kBufs>
struct TmaStage {
    uint8_t* buf;    // buffer 0, generic address
    uint32_t buf_s;  // buffer 0, shared-window address
    int issued;

    __device__ __forceinline__ void put(int lane, const uint4 (&w)[4], const CUtensorMap* map, int x, int y) {
        const int b = issued % kBufs;
        if (lane == 0 && issued >= kBufs) bulk_wait_read<kBufs - 1>();
        __syncwarp();
        stage_put(buf + b * kEpiStageBytes, lane, w);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            tma_store_2d(map, buf_s + static_cast<uint32_t>(b * kEpiStageBytes), x, y);
            bulk_commit();
        }
        ++issued;
    }
    // 32 columns [n0, n0+32) of the warp's rows to an fp32 (two boxes) or bf16 (one) output.
    __device__ __forceinline__ void put32(int lane, const CUtensorMap* map, int is_bf16, int row0, int n0,
                                          const float (&v0)[16], const float (&v1)[16]) {
        if (is_bf16) {
            uint4 w[4];
            pack_bf16x16(v0, *reinterpret_cast<uint4(*)[2]>(&w[0]));
            pack_bf16x16(v1, *reinterpret_cast<uint4(*)[2]>(&w[2]));
            put(lane, w, map, n0, row0);
        } else if (kBufs >= 2) {  // both boxes staged behind one wait and one fence
            const int b0 = issued % kBufs, b1 = (issued + 1) % kBufs;
            if (lane == 0 && issued + 2 > kBufs) bulk_wait_read<(kBufs >= 2 ? kBufs - 2 : 0)>();
            __syncwarp();
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const float(&v)[16] = h ? v1 : v0;
                uint4 w[4];
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    w[k] = make_uint4(__float_as_uint(v[4 * k]), __float_as_uint(v[4 * k + 1]),
                                      __float_as_uint(v[4 * k + 2]), __float_as_uint(v[4 * k + 3]));
                stage_put(buf + (h ? b1 : b0) * kEpiStageBytes, lane, w);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                tma_store_2d(map, buf_s + static_cast<uint32_t>(b0 * kEpiStageBytes), n0, row0);
                bulk_commit();
                tma_store_2d(map, buf_s + static_cast<uint32_t>(b1 * kEpiStageBytes), n0 + 16, row0);
                bulk_commit();
            }
            issued += 2;
        } else {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const float(&v)[16] = h ? v1 : v0;
                uint4 w[4];
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    w[k] = make_uint4(__float_as_uint(v[4 * k]), __float_as_uint(v[4 * k + 1]),
                                      __float_as_uint(v[4 * k + 2]), __float_as_uint(v[4 * k + 3]));
                put(lane, w, map, n0 + 16 * h, row0);
            }
        }
    }
    // Lane 0: every store issued has completed (before the warp's shared memory goes away).
    __device__ __forceinline__ void finish(int lane) {
        if (lane == 0) bulk_wait_all();
        __syncwarp();
    }
};

// One epilogue warp's share of a tile: rows row0 .. row0+31 (lane = row - row0, the warp's
// TMEM lane quarter) and kCols columns from n_start, read from TMEM at t_addr. TMEM loads go
// out two 16-column chunks at a time (one wait per 32 columns). Residual epilogues take each
// chunk's residual from the warp's TMA ring. Batches of 32 columns inside N with aligned
// operands store through the staging block `stg` (residual epilogues: as TMA stores through
// `ts`, maps mo / mo2, reading the span's bias and, when the warp's rows share one, its gate
// row from `side`, which the warp fills once per tile); the rest go element by element.
template <int kCols, bool kResid, int kBufs>
__device__ __forceinline__ void epilogue_span(const Epilogue& ep, int row0, int M, int n_start, int N, bool vec,
                                              uint32_t t_addr, uint8_t* stg, ResidRing* ring, TmaStage<kBufs>* ts,
                                              const CUtensorMap* mo, const CUtensorMap* mo2, float* side) {
    constexpr int kChunks = kCols / 16;
    static_assert(kChunks % 2 == 0, "chunks go out in pairs");
    static_assert(kCols <= 128, "side vectors hold 128 columns");
    const int lane = threadIdx.x & 31;
    const int row = row0 + lane;
    const bool row_ok = row < M;
    bool side_gate = false;
    if (kResid && vec) {
        constexpr int kPer = kCols / 32;
        const int c0 = n_start + kPer * lane;
        const int g0 = row0 / ep.rows_per_gate;
        side_gate = ep.gate != nullptr && g0 == (min(row0 + 31, M - 1) / ep.rows_per_gate);
        const float* grow = side_gate ? ep.gate + static_cast<long long>(g0) * ep.gate_ld : nullptr;
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const bool in = c0 + k < N;
            side[kPer * lane + k] = ep.bias && in ? ep.bias[c0 + k] : 0.f;
            side[128 + kPer * lane + k] = grow && in ? grow[c0 + k] : 1.f;
        }
        __syncwarp();
    }
#pragma unroll 1
    for (int c = 0; c < kChunks; c += 2) {
        uint32_t r[2][16];
        tmem_ld16(t_addr + static_cast<uint32_t>(c * 16), r[0]);
        tmem_ld16(t_addr + static_cast<uint32_t>((c + 1) * 16), r[1]);
        tmem_wait_ld();
        float rv[2][16];
        if (kResid) {  // every chunk is taken, in order, even the ones past N
            ring->take(rv[0]);
            ring->take(rv[1]);
        }
        const int n0 = n_start + c * 16;
        if (n0 >= N) continue;  // uniform across the warp
        if (vec && n0 + 32 <= N) {
            float v[2][16];
#pragma unroll
            for (int g = 0; g < 2; ++g) {
#pragma unroll
                for (int j = 0; j < 16; ++j) v[g][j] = __uint_as_float(r[g][j]);
                float gv[16], bv[16];
                if (kResid) {
                    const float* sb = side + (n0 - n_start) + 16 * g;
#pragma unroll
                    for (int j = 0; j < 16; j += 4) {
                        const float4 b4 = *reinterpret_cast<const float4*>(sb + j);
                        bv[j] = b4.x, bv[j + 1] = b4.y, bv[j + 2] = b4.z, bv[j + 3] = b4.w;
                    }
                    if (side_gate) {
#pragma unroll
                        for (int j = 0; j < 16; j += 4) {
                            const float4 g4 = *reinterpret_cast<const float4*>(sb + 128 + j);
                            gv[j] = g4.x, gv[j + 1] = g4.y, gv[j + 2] = g4.z, gv[j + 3] = g4.w;
                        }
                    } else if (row_ok) {
                        gate16(ep, row, n0 + 16 * g, gv);
                    }
                } else if (ep.bias) {
#pragma unroll
                    for (int j = 0; j < 16; j += 4) {
                        const float4 b4 = *reinterpret_cast<const float4*>(ep.bias + n0 + 16 * g + j);
                        bv[j] = b4.x, bv[j + 1] = b4.y, bv[j + 2] = b4.z, bv[j + 3] = b4.w;
                    }
                }
                compute16<kResid>(ep, bv, v[g], rv[g], gv);
            }
            if (ep.out) {
                if (kResid) ts->put32(lane, mo, ep.out_bf16, row0, n0, v[0], v[1]);
                else store32(stg, lane, ep.out, ep.out_bf16, ep.ldo, row0, M, n0, v[0], v[1]);
            }
            if (ep.out2) {
                if (ep.act2 == kActSilu) {
#pragma unroll
                    for (int g = 0; g < 2; ++g)
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[g][j] = silu(v[g][j]);
                }
                if (kResid) ts->put32(lane, mo2, ep.out2_bf16, row0, n0, v[0], v[1]);
                else store32(stg, lane, ep.out2, ep.out2_bf16, ep.ldo2, row0, M, n0, v[0], v[1]);
            }
            continue;
        }
#pragma unroll
        for (int g = 0; g < 2; ++g) {
            const int n1 = n0 + g * 16;
            if (row_ok && n1 < N) {
                Side16 sd;
                if (kResid) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        sd.r[j] = rv[g][j];
                        sd.g[j] = (ep.gate && n1 + j < N)
                                      ? ep.gate[static_cast<long long>(row / ep.rows_per_gate) * ep.gate_ld + n1 + j]
                                      : 1.f;
                    }
                }
                float v[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[g][j]);
                epilogue16<kResid>(ep, row, n1, N, v, vec, sd);
            }
        }
    }
}

// --- the kernel ------------------------------------------------------------------------
constexpr int kEpiWarps = 8;
constexpr int kThreads = 32 * (2 + kEpiWarps);

// TMEM columns between the two accumulators: BN, or 256 for 192-column tiles (each
// accumulator then starts on a 256-column boundary).
template <int BN>
constexpr int kAccCols = BN <= 128 ? BN : 256;

template <int BN, bool kResid>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmR, const __grid_constant__ CUtensorMap tmO,
                   const __grid_constant__ CUtensorMap tmO2, int M, int N, int K, Epilogue ep, int vec, int* err) {
    using C = Cfg<BN, kResid>;
    constexpr int S = C::kStages;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* gbase = smem_raw + (base - raw);
    const uint32_t a_smem = base;                       // S x kABytes
    const uint32_t b_smem = base + S * C::kABytes;      // S x kBBytes
    const uint32_t bars = base + C::kBarOffset;
    auto full = [&](int s) { return bars + 8u * s; };
    auto empty = [&](int s) { return bars + 8u * (S + s); };
    auto tfull = [&](int a) { return bars + 8u * (2 * S + a); };
    auto tempty = [&](int a) { return bars + 8u * (2 * S + 2 + a); };
    const uint32_t done_bar = bars + 8u * (2 * S + 4);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + C::kBarOffset + C::kBars * 8);
    const uint32_t ring_bars = bars + 8u * (2 * S + 5);  // kEpiWarps x C::kRing, residual epilogues

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int num_m = (M + BM - 1) / BM;
    const int num_n = (N + BN - 1) / BN;
    const int num_tiles = num_m * num_n;
    const int num_kb = (K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull(a), 1);
            mbar_init(tempty(a), kEpiWarps);
        }
        mbar_init(done_bar, 1);
        if (kResid)
            for (int i = 0; i < kEpiWarps * C::kRing; ++i) mbar_init(ring_bars + 8u * i, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), C::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
            int stage = 0;
            uint32_t phase = 0;
            long long issued = 0;
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
                const int m_blk = tile / num_n;
                const int n_blk = tile % num_n;
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(empty(stage), phase ^ 1u, err, kTimeout)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(full(stage), C::kStageBytes);
                    tma_load_2d(&tmA, a_smem + stage * C::kABytes, full(stage), kb * BK, m_blk * BM);
                    tma_load_2d(&tmB, b_smem + stage * C::kBBytes, full(stage), kb * BK, n_blk * BN);
                    ++issued;
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok || *(volatile int*)err != 0) {
                // Drain: wait (bounded) until each of the last issued copies has landed.
                const long long first = issued > S ? issued - S : 0;
                for (long long i = first; i < issued; ++i) {
                    mbar_wait_quiet(full(static_cast<int>(i % S)), static_cast<uint32_t>((i / S) & 1));
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            int local = 0;
            for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x, ++local) {
                const int acc = local & 1;
                const uint32_t use = static_cast<uint32_t>(local >> 1);
                if (!mbar_wait(tempty(acc), (use & 1u) ^ 1u, err, kTimeout)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem + static_cast<uint32_t>(acc * kAccCols<BN>);
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(full(stage), phase, err, kTimeout)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = a_smem + stage * C::kABytes;
                    const uint32_t b_addr = b_smem + stage * C::kBBytes;
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k) {
                        umma_bf16(d_tmem, kmajor_sw128_desc(a_addr + k * 32), kmajor_sw128_desc(b_addr + k * 32),
                                  idesc, (kb | k) != 0 ? 1u : 0u);
                    }
                    umma_commit(empty(stage));
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                umma_commit(tfull(acc));
            }
            // All MMAs issued by this thread are complete once done_bar fires.
            umma_commit(done_bar);
            mbar_wait_quiet(done_bar, 0u);
        }
    } else {
        const int q = warp & 3;                   // TMEM lane quarter this warp may access
        const int chalf = (warp - 2) / 4;         // which half of the tile's columns
        const int ew = warp - 2;
        ResidRing ring{&tmR, gbase + C::kRingOffset + ew * C::kRing * kRingChunk,
                       base + C::kRingOffset + static_cast<uint32_t>(ew * C::kRing * kRingChunk),
                       ring_bars + 8u * static_cast<uint32_t>(ew * C::kRing), static_cast<int>(blockIdx.x),
                       static_cast<int>(gridDim.x), num_tiles, num_n, BN, BM, q * 32, chalf * (BN / 2), BN / 2 / 16,
                       0, 0, err};
        ring.depth = C::kRing;
        if (kResid && lane == 0) ring.start();
        uint8_t* stg = gbase + C::kEpiOffset + ew * C::kStoreBufs * kEpiStageBytes;
        TmaStage<C::kStoreBufs> ts{stg, base + static_cast<uint32_t>(C::kEpiOffset + ew * C::kStoreBufs * kEpiStageBytes),
                                   0};
        float* side = reinterpret_cast<float*>(gbase + C::kSideOffset + ew * kSideWarpBytes);
        int local = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
            const int acc = local & 1;
            const uint32_t use = static_cast<uint32_t>(local >> 1);
            if (!mbar_wait(tfull(acc), use & 1u, err, kTimeout)) break;
            tc_fence_after();
            const int m_blk = tile / num_n;
            const int n_blk = tile % num_n;
            const int col0 = chalf * (BN / 2);
            const uint32_t t_row = tmem + (static_cast<uint32_t>(q * 32) << 16) +
                                   static_cast<uint32_t>(acc * kAccCols<BN> + col0);
            epilogue_span<BN / 2, kResid, C::kStoreBufs>(ep, m_blk * BM + q * 32, M, n_blk * BN + col0, N,
                                                         vec != 0, t_row, stg, &ring, &ts, &tmO, &tmO2, side);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty(acc));
        }
        if (kResid) ts.finish(lane);
        if (kResid && lane == 0) ring.drain();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::kTmemCols);
    }
}

// --- the CTA-pair kernel -------------------------------------------------------------------
// The same pipeline over a cluster of two CTAs on two SMs computing 256 x BN tiles with
// tcgen05.mma.cta_group::2: each CTA stages its own 128 rows of A and BN/2 rows of B per
// k-block (the shared-memory traffic per FLOP drops by a quarter against 128 x BN tiles,
// and 7-8 stages fit), the leader CTA (rank 0) issues the MMAs, and each CTA's TMEM holds
// its 128 rows of the accumulator for its own epilogue warps.
//   full[s]    leader only: armed by the leader's producer with both CTAs' bytes; both
//              CTAs' TMA loads complete on it
//   empty[s]   both CTAs: the leader's MMA commit arrives on both
//   tfull[a]   both CTAs: the leader's commit after a tile's last MMA arrives on both
//   tempty[a]  leader only: one arrival per epilogue warp of either CTA
// Every wait is bounded; on expiry each role stops issuing work and every thread still
// reaches the final cluster barrier, so neither CTA leaves while its peer uses its memory.
template <int BN, bool kResid = false, bool kDeep = false>
struct Cfg2 : Layout<kResid ? (kDeep ? (BN == 128 ? 7 : 5) : (BN == 128 ? 5 : 4))
                            : (BN == 128 ? 8 : (BN == 192 ? 7 : 6)),
                     128 * BK * 2, (BN / 2) * BK * 2, kResid, kResid && !kDeep ? 2 : 1, kDeep ? 2 : 3> {
    static constexpr int kBH = BN / 2;  // B rows per CTA
    static constexpr int kTmemCols = 2 * BN <= 256 ? 256 : 512;
};

template <int BN, bool kResid, bool kDeep, bool kConv = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmR, const __grid_constant__ CUtensorMap tmO,
                    const __grid_constant__ CUtensorMap tmO2, int M, int N, int K, Epilogue ep, int vec, int* err,
                    ConvGeom cg) {
    using C = Cfg2<BN, kResid, kDeep>;
    constexpr int S = C::kStages;
    constexpr int BM2 = 2 * BM;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* gbase = smem_raw + (base - raw);
    const uint32_t a_smem = base;
    const uint32_t b_smem = base + S * C::kABytes;
    const uint32_t bars = base + C::kBarOffset;
    auto full = [&](int s) { return bars + 8u * s; };
    auto empty = [&](int s) { return bars + 8u * (S + s); };
    auto tfull = [&](int a) { return bars + 8u * (2 * S + a); };
    auto tempty = [&](int a) { return bars + 8u * (2 * S + 2 + a); };
    const uint32_t done_bar = bars + 8u * (2 * S + 4);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + C::kBarOffset + C::kBars * 8);
    const uint32_t ring_bars = bars + 8u * (2 * S + 5);  // kEpiWarps x C::kRing, residual epilogues

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1;
    const int npairs = gridDim.x >> 1;
    const int num_m = (M + BM2 - 1) / BM2;
    const int num_n = (N + BN - 1) / BN;
    const int num_tiles = num_m * num_n;
    const int num_kb = (K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull(a), 1);
            mbar_init(tempty(a), 2 * kEpiWarps);
        }
        mbar_init(done_bar, 1);
        if (kResid)
            for (int i = 0; i < kEpiWarps * C::kRing; ++i) mbar_init(ring_bars + 8u * i, 1);
        fence_barrier_init();
    }
    cluster_sync();  // barriers of both CTAs initialised before any remote arrival
    if (warp == 1) {
        tmem_alloc2(smem_u32(tmem_slot), C::kTmemCols);
        tmem_relinquish2();
    }
    tc_fence_before();
    cluster_sync();  // both CTAs' accumulator columns exist before the leader's first MMA
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t full_leader = mapa(full(0), 0);
    const uint32_t tempty_leader = mapa(tempty(0), 0);

    if (warp == 0) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
            int stage = 0;
            uint32_t phase = 0;
            long long issued = 0;
            bool ok = true;
            for (int tile = pair; ok && tile < num_tiles; tile += npairs) {
                const int m_blk = tile / num_n;
                const int n_blk = tile % num_n;
                // implicit convolution: this CTA's 128 rows are whole image rows from (img, y0, x0)
                int img = 0, y0 = 0, x0 = 0;
                if constexpr (kConv) {
                    const int m0 = m_blk * BM2 + static_cast<int>(rank) * BM;
                    const int hw = cg.H * cg.W;
                    img = m0 / hw;
                    const int rem = m0 - img * hw;
                    y0 = rem / cg.W;
                    x0 = rem - y0 * cg.W;
                }
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(empty(stage), phase ^ 1u, err, kTimeout)) {
                        ok = false;
                        break;
                    }
                    if (leader) mbar_arrive_expect_tx(full(stage), 2 * C::kStageBytes);
                    const uint32_t fb = full_leader + 8u * stage;
                    if constexpr (kConv) {
                        const int tap = kb / cg.cchunks;
                        const int cc = kb - tap * cg.cchunks;
                        const int ty = tap / cg.kw;
                        const int e = cg.ox + (tap - ty * cg.kw);  // tap column relative to the row's (first) pixel
                        int xc = x0 + e, ch = cc * BK;
                        if (cg.pair) {  // e >= -2: super-pixel floor(e / 2), its (e & 1)-th half
                            xc = x0 + (e + 2) / 2 - 1;
                            ch += (e & 1) * cg.cin;
                        }
                        tma_load_4d_pair(&tmA, a_smem + stage * C::kABytes, fb, ch, xc, y0 + cg.oy + ty, img);
                    } else {
                        tma_load_2d_pair(&tmA, a_smem + stage * C::kABytes, fb, kb * BK,
                                         m_blk * BM2 + static_cast<int>(rank) * BM);
                    }
                    tma_load_2d_pair(&tmB, b_smem + stage * C::kBBytes, fb, kb * BK,
                                     n_blk * BN + static_cast<int>(rank) * C::kBH);
                    ++issued;
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok || *(volatile int*)err != 0) {
                // Drain (bounded): the leader waits for its last armed stages to fill; the
                // peer for the MMAs that consume its last copies to release them.
                const long long first = issued > S ? issued - S : 0;
                for (long long i = first; i < issued; ++i) {
                    const int st = static_cast<int>(i % S);
                    const uint32_t ph = static_cast<uint32_t>((i / S) & 1);
                    if (leader) mbar_wait_quiet(full(st), ph);
                    else mbar_wait_quiet(empty(st), ph);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            constexpr uint32_t idesc = idesc_bf16_f32(BM2, BN);
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            int local = 0;
            for (int tile = pair; ok && tile < num_tiles; tile += npairs, ++local) {
                const int acc = local & 1;
                const uint32_t use = static_cast<uint32_t>(local >> 1);
                if (!mbar_wait(tempty(acc), (use & 1u) ^ 1u, err, kTimeout)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem + static_cast<uint32_t>(acc * kAccCols<BN>);
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(full(stage), phase, err, kTimeout)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = a_smem + stage * C::kABytes;
                    const uint32_t b_addr = b_smem + stage * C::kBBytes;
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k) {
                        umma2_bf16(d_tmem, kmajor_sw128_desc(a_addr + k * 32), kmajor_sw128_desc(b_addr + k * 32),
                                   idesc, (kb | k) != 0 ? 1u : 0u);
                    }
                    umma2_commit_both(empty(stage));
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                umma2_commit_both(tfull(acc));
            }
            umma2_commit(done_bar);
            mbar_wait_quiet(done_bar, 0u);
        }
    } else {
        const int q = warp & 3;
        const int chalf = (warp - 2) / 4;
        const int ew = warp - 2;
        ResidRing ring{&tmR, gbase + C::kRingOffset + ew * C::kRing * kRingChunk,
                       base + C::kRingOffset + static_cast<uint32_t>(ew * C::kRing * kRingChunk),
                       ring_bars + 8u * static_cast<uint32_t>(ew * C::kRing), pair, npairs, num_tiles, num_n, BN, BM2,
                       static_cast<int>(rank) * BM + q * 32, chalf * (BN / 2), BN / 2 / 16, 0, 0, err};
        ring.depth = C::kRing;
        if (kResid && lane == 0) ring.start();
        uint8_t* stg = gbase + C::kEpiOffset + ew * C::kStoreBufs * kEpiStageBytes;
        TmaStage<C::kStoreBufs> ts{stg, base + static_cast<uint32_t>(C::kEpiOffset + ew * C::kStoreBufs * kEpiStageBytes),
                                   0};
        float* side = reinterpret_cast<float*>(gbase + C::kSideOffset + ew * kSideWarpBytes);
        int local = 0;
        for (int tile = pair; tile < num_tiles; tile += npairs, ++local) {
            const int acc = local & 1;
            const uint32_t use = static_cast<uint32_t>(local >> 1);
            if (!mbar_wait(tfull(acc), use & 1u, err, kTimeout)) break;
            tc_fence_after();
            const int m_blk = tile / num_n;
            const int n_blk = tile % num_n;
            const int col0 = chalf * (BN / 2);
            const uint32_t t_row = tmem + (static_cast<uint32_t>(q * 32) << 16) +
                                   static_cast<uint32_t>(acc * kAccCols<BN> + col0);
            epilogue_span<BN / 2, kResid, C::kStoreBufs>(ep, m_blk * BM2 + static_cast<int>(rank) * BM + q * 32, M,
                                                         n_blk * BN + col0, N, vec != 0, t_row, stg, &ring, &ts,
                                                         &tmO, &tmO2, side);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(tempty_leader + 8u * acc);
        }
        if (kResid) ts.finish(lane);
        if (kResid && lane == 0) ring.drain();
    }

    tc_fence_before();
    __syncwarp();
    cluster_sync();  // no CTA leaves while its peer may still use its memory or TMEM
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc2(tmem, C::kTmemCols);
    }
}

// --- host side ---------------------------------------------------------------------------
// 2-D bf16 tensor map over a row-major [rows, cols] matrix with row stride ld elements;
// box = [box_rows, 64 columns], 128-byte swizzle, out-of-bounds elements read as zero.
static CUtensorMap make_map(const void* ptr, int rows, int cols, long long ld, int box_rows) {
    CUtensorMap m;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(BK), static_cast<cuuint32_t>(box_rows)};
    tma_encode_tiled(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ptr, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    return m;
}

// fp32 residual [M, N] (row stride ldr) in boxes of 32 rows x 16 columns with the 64-byte
// swizzle the epilogue's staging layout uses; out-of-range rows and columns read as zero.
static CUtensorMap resid_map(const GemmProblem& p) {
    CUtensorMap m;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(p.N), static_cast<cuuint64_t>(p.M)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(p.ep.ldr) * 4};
    const cuuint32_t box[2] = {16, 32};
    tma_encode_tiled(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, p.ep.resid, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_64B);
    return m;
}

// Output tensor map for the residual epilogues' TMA stores: [M, N] fp32 or bf16 with row
// stride ld elements, box = 32 rows x 64 bytes, 64-byte swizzle (the staging layout).
static CUtensorMap out_map(void* ptr, int is_bf16, long long ld, int M, int N) {
    CUtensorMap m;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(M)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * (is_bf16 ? 2 : 4)};
    const cuuint32_t box[2] = {is_bf16 ? 32u : 16u, 32};
    tma_encode_tiled(&m, is_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, ptr, dims,
                     strides, box, CU_TENSOR_MAP_SWIZZLE_64B);
    return m;
}

template <int BN, bool kResid>
static void launch(const GemmProblem& p, int* err, cudaStream_t stream, int num_sms) {
    using C = Cfg<BN, kResid>;
    static PerDeviceOnce attr_done;
    if (attr_done.pending()) {
        SANA_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<BN, kResid>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       C::kSmemBytes));
        attr_done.mark();
    }
    const CUtensorMap ma = make_map(p.A, p.M, p.K, p.lda, BM);
    const CUtensorMap mb = make_map(p.B, p.N, p.K, p.ldb, BN);
    const CUtensorMap mr = kResid ? resid_map(p) : ma;
    const Epilogue& e = p.ep;
    auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    bool vec = (p.N % 16 == 0);
    if (e.bias) vec = vec && a16(e.bias);
    if (e.resid) vec = vec && a16(e.resid) && (e.ldr % 4 == 0);
    if (e.gate) vec = vec && a16(e.gate) && (e.gate_ld % 4 == 0);
    if (e.out) vec = vec && a16(e.out) && (e.ldo % 8 == 0);
    if (e.out2) vec = vec && a16(e.out2) && (e.ldo2 % 8 == 0);
    // the residual epilogue's TMA stores need what `vec` already requires of the outputs
    const CUtensorMap mo = kResid && vec && e.out ? out_map(e.out, e.out_bf16, e.ldo, p.M, p.N) : ma;
    const CUtensorMap mo2 = kResid && vec && e.out2 ? out_map(e.out2, e.out2_bf16, e.ldo2, p.M, p.N) : ma;
    const int tiles = ((p.M + BM - 1) / BM) * ((p.N + BN - 1) / BN);
    const int grid = tiles < num_sms ? tiles : num_sms;
    gemm_tc_kernel<BN, kResid><<<grid, kThreads, C::kSmemBytes, stream>>>(ma, mb, mr, mo, mo2, p.M, p.N, p.K, e,
                                                                          vec ? 1 : 0, err);
    SANA_CUDA(cudaGetLastError());
}

// 4-D bf16 tensor map over an NHWC image batch [images, H, W, C] for implicit-convolution
// A tiles: box = 64 channels x (128 pixels of whole rows), 128-byte swizzle (the same shared
// layout as make_map's 128-row box); out-of-image pixels read as zero.
static CUtensorMap conv_map(const GemmProblem& p) {
    const ConvA& c = p.conv;
    const int images = (p.M + c.H * c.W - 1) / (c.H * c.W);
    const int bx = c.W >= BM ? BM : c.W;
    CUtensorMap m;
    const cuuint64_t dims[4] = {static_cast<cuuint64_t>(c.C), static_cast<cuuint64_t>(c.W),
                                static_cast<cuuint64_t>(c.H), static_cast<cuuint64_t>(images)};
    const cuuint64_t strides[3] = {static_cast<cuuint64_t>(c.C) * 2, static_cast<cuuint64_t>(c.W) * c.C * 2,
                                   static_cast<cuuint64_t>(c.H) * c.W * c.C * 2};
    const cuuint32_t box[4] = {static_cast<cuuint32_t>(BK), static_cast<cuuint32_t>(bx),
                               static_cast<cuuint32_t>(BM / bx), 1};
    tma_encode_tiled(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, p.A, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    return m;
}

template <int BN, bool kResid, bool kDeep = false, bool kConv = false>
static void launch2(const GemmProblem& p, int* err, cudaStream_t stream, int num_sms) {
    using C = Cfg2<BN, kResid, kDeep>;
    static PerDeviceOnce attr_done;
    if (attr_done.pending()) {
        SANA_CUDA(cudaFuncSetAttribute(gemm_tc2_kernel<BN, kResid, kDeep, kConv>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes));
        attr_done.mark();
    }
    const CUtensorMap ma = kConv ? conv_map(p) : make_map(p.A, p.M, p.K, p.lda, BM);
    ConvGeom cg;
    if (kConv) {
        cg.H = p.conv.H;
        cg.W = p.conv.W;
        cg.pair = p.conv.pair ? 1 : 0;
        cg.cin = p.conv.pair ? p.conv.C / 2 : p.conv.C;
        cg.cchunks = cg.cin / BK;
        cg.kw = p.conv.kw;
        cg.oy = p.conv.oy;
        cg.ox = p.conv.ox;
    }
    const CUtensorMap mb = make_map(p.B, p.N, p.K, p.ldb, C::kBH);
    const CUtensorMap mr = kResid ? resid_map(p) : ma;
    const Epilogue& e = p.ep;
    auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    bool vec = (p.N % 16 == 0);
    if (e.bias) vec = vec && a16(e.bias);
    if (e.resid) vec = vec && a16(e.resid) && (e.ldr % 4 == 0);
    if (e.gate) vec = vec && a16(e.gate) && (e.gate_ld % 4 == 0);
    if (e.out) vec = vec && a16(e.out) && (e.ldo % 8 == 0);
    if (e.out2) vec = vec && a16(e.out2) && (e.ldo2 % 8 == 0);
    const CUtensorMap mo = kResid && vec && e.out ? out_map(e.out, e.out_bf16, e.ldo, p.M, p.N) : ma;
    const CUtensorMap mo2 = kResid && vec && e.out2 ? out_map(e.out2, e.out2_bf16, e.ldo2, p.M, p.N) : ma;
    const int tiles = ((p.M + 2 * BM - 1) / (2 * BM)) * ((p.N + BN - 1) / BN);
    const int pairs = tiles < num_sms / 2 ? tiles : num_sms / 2;
    gemm_tc2_kernel<BN, kResid, kDeep, kConv><<<2 * pairs, kThreads, C::kSmemBytes, stream>>>(
        ma, mb, mr, mo, mo2, p.M, p.N, p.K, e, vec ? 1 : 0, err, cg);
    SANA_CUDA(cudaGetLastError());
}

// CTA-pair tiles for tall problems (the block projections: M = sequences x tokens); the
// single-CTA kernel otherwise. SANA_GEMM_PAIR=0 in the environment selects the single-CTA
// kernel for every shape.
static bool use_pair(const GemmProblem& p, int num_sms) {
    static const bool enabled = [] {
        const char* v = std::getenv("SANA_GEMM_PAIR");
        return !(v && v[0] == '0');
    }();
    return enabled && num_sms >= 2 && p.M >= 2048;
}

}  // namespace tc

bool gemm_conv_supported(const GemmProblem& p) {
    const ConvA& c = p.conv;
    auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    if (c.H <= 0 || c.W <= 0 || c.C <= 0 || c.kh < 1 || c.kw < 1) return false;
    constexpr int BM = tc::BM, BK = tc::BK;
    const bool rows_ok = (c.W % BM == 0) || (BM % c.W == 0 && (static_cast<long long>(c.H) * c.W) % BM == 0);
    const int cin = c.pair ? c.C / 2 : c.C;
    const bool pair_ok = !c.pair || (c.C % 2 == 0 && c.ox >= -2);
    return p.a_bf16 && p.b_bf16 && cin % BK == 0 && pair_ok && rows_ok && p.K == c.kh * c.kw * cin && p.N >= 16 &&
           (p.ldb % 8 == 0) && a16(p.A) && a16(p.B) && !p.ep.resid && p.M % (c.H * c.W) == 0 &&
           c.kh * c.kw <= 64;
}

bool gemm_tc_supported(const GemmProblem& p) {
    if (p.conv.H > 0) return gemm_conv_supported(p);
    auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    // the residual epilogue reads its fp32 residual with TMA: 16-byte aligned base and rows
    const bool resid_ok = !p.ep.resid || (a16(p.ep.resid) && p.ep.ldr % 4 == 0);
    return p.a_bf16 && p.b_bf16 && p.M > 0 && p.N > 0 && p.K > 0 && (p.K % 8 == 0) && (p.lda % 8 == 0) &&
           (p.ldb % 8 == 0) && a16(p.A) && a16(p.B) && p.N >= 16 && resid_ok;
}

void gemm_tc(const GemmProblem& p, int* err, cudaStream_t stream, int num_sms) {
    SANA_REQUIRE(gemm_tc_supported(p), "gemm_tc: unsupported problem");
    // The MMA costs the same issue time for any N up to 256, so tiles are 256 wide whenever
    // N allows (the last one ragged: its out-of-range B rows read as zero and its columns
    // are masked in the epilogue); narrow problems use 128 columns.
    if (p.conv.H > 0) {
        // implicit convolution: CTA-pair kernel at any M (its producer builds the 4-D tiles)
        if (p.N >= 256) tc::launch2<256, false, false, true>(p, err, stream, num_sms);
        else tc::launch2<128, false, false, true>(p, err, stream, num_sms);
        return;
    }
    const bool pair = tc::use_pair(p, num_sms);
    const bool resid = p.ep.resid != nullptr;
    // long reductions keep the MMA fed with deeper operand pipelines (their epilogue has slack)
    const bool deep = p.K >= 2048;
    // Short per-GPU batches (M <= 8192, the multi-GPU runs' shards) leave few 256 x 256 tiles per
    // CTA pair: the model's width 1152 then takes six 192-column tiles instead of four and a half
    // 256-column ones (measured 4-7 % faster at M = 4096 and 8192, slower at larger M or N).
    if (pair && p.M <= 8192 && p.N % 192 == 0 && p.N <= 1536) {
        if (resid && deep) tc::launch2<192, true, true>(p, err, stream, num_sms);
        else resid ? tc::launch2<192, true>(p, err, stream, num_sms) : tc::launch2<192, false>(p, err, stream, num_sms);
        return;
    }
    if (p.N >= 256) {
        if (pair && resid && deep) tc::launch2<256, true, true>(p, err, stream, num_sms);
        else if (pair) resid ? tc::launch2<256, true>(p, err, stream, num_sms) : tc::launch2<256, false>(p, err, stream, num_sms);
        else resid ? tc::launch<256, true>(p, err, stream, num_sms) : tc::launch<256, false>(p, err, stream, num_sms);
    } else {
        if (pair && resid && deep) tc::launch2<128, true, true>(p, err, stream, num_sms);
        else if (pair) resid ? tc::launch2<128, true>(p, err, stream, num_sms) : tc::launch2<128, false>(p, err, stream, num_sms);
        else resid ? tc::launch<128, true>(p, err, stream, num_sms) : tc::launch<128, false>(p, err, stream, num_sms);
    }
}

static std::atomic<long long> g_tc_launches{0}, g_simt_launches{0};

bool gemm_tc_shape_ok(const GemmProblem& p) { return p.K % 8 == 0 && p.N >= 16; }

void gemm(const GemmProblem& p, int* err, cudaStream_t stream, int num_sms, bool allow_tc) {
    if (p.M == 0 || p.N == 0) return;
    SANA_REQUIRE(p.conv.H == 0 || (allow_tc && gemm_conv_supported(p)),
                 "implicit convolution needs the tensor-core path and a supported shape");
    if (p.require_tc && allow_tc && p.a_bf16 && p.b_bf16 && gemm_tc_shape_ok(p) && !gemm_tc_supported(p))
        throw std::logic_error("gemm: a bf16 projection of shape M=" + std::to_string(p.M) + " N=" +
                               std::to_string(p.N) + " K=" + std::to_string(p.K) +
                               " has operands the tensor-core kernel cannot load (pointer or row stride "
                               "not 16-byte aligned); refusing the CUDA-core fallback");
    if (allow_tc && gemm_tc_supported(p)) {
        gemm_tc(p, err, stream, num_sms);
        ++g_tc_launches;
    } else {
        gemm_simt(p, stream);
        ++g_simt_launches;
    }
}

void gemm_counts(long long* tc, long long* simt) {
    if (tc) *tc = g_tc_launches.load();
    if (simt) *simt = g_simt_launches.load();
}

}  // namespace sana
