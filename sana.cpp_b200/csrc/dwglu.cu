// Mix-FFN middle: depthwise 3x3 conv with zero padding and bias over all E channels of the
// NHWC token grid, then the GLU gate out[c] = dw[c] * silu(dw[c + E/2])
// (depthwise_conv2d_3x3, common_ops.cpp:484-505, per-plane taps summed ky-major then kx,
// bias last; glumb_conv's split and gate, common_ops.cpp:745-758). The fp32 path keeps that
// order and CUDA's expf; the bf16 path starts each sum from the bias and takes the sigmoid
// from the hardware tanh (both differences sit far below the bf16 rounding of its output).
//
// The input is the SiLU-ed output of the inverted 1x1 conv, already token-major, so the
// reference's NCHW round trips (tokens_to_grid_4d / grid_to_tokens_3d) disappear.
#include <algorithm>

#include "kernels.h"
#include "tma.h"

#ifndef DW_SLOT_ROWS
#define DW_SLOT_ROWS 4
#endif
#ifndef DW_RING
#define DW_RING 4
#endif

namespace sana {
namespace {

// bf16 streaming path (half % 8 == 0, 16-byte aligned rows). A work item is one sequence,
// 64 channels of each half, a stripe of up to 32 image columns and a band of image rows; a
// persistent block walks its items in grid stride. The last warp is the producer: one lane
// streams the item's input rows (the band plus a one-row halo above and below) into a ring
// of shared-memory slots, one TMA copy of [kSlotRows rows, stripe + 2 pixels, 2 halves,
// 64 channels] per slot; pixels and rows outside the image read as zeros (the conv's zero
// padding). Warps 0-15 consume the rows: thread (warp w, lane p) owns channel pair p of both
// halves and the two columns 2w, 2w+1 of the stripe, and waits on the ring once per slot. Two
// columns per thread rather than four: 16 consumer warps (four per scheduler) hide the latency
// of the per-row FMA chains better than 8, for 6 % more instructions (measured 5.8 % faster).
constexpr int kSliceCh = 64;                          // channels per half in a work item
constexpr int kStripe = 32;                           // image columns per work item
constexpr int kCols = 2;                              // columns per thread
constexpr int kDwWarps = kStripe / kCols;             // consumer warps
constexpr int kStripePx = kStripe + 2;                // staged pixels per row
constexpr int kPxBytes = 2 * kSliceCh * 2;            // one pixel: 64 value + 64 gate channels, bf16
constexpr int kRowBytes = kStripePx * kPxBytes;       // 8704
constexpr int kSlotRows = DW_SLOT_ROWS;               // input rows per ring slot
constexpr int kSlotBytes = kSlotRows * kRowBytes;
constexpr int kDwRing = DW_RING;                      // slots
constexpr int kDwThreads = 32 * (kDwWarps + 1);
// Beside each ring slot: the taps and biases of the item whose first rows the slot holds
// ([64 value channels][9], [64 gate channels][9], then 64 + 64 biases, fp32), copied in with
// those rows, so a consumer reads its item's weights from shared memory once the first slot
// has landed instead of waiting on 72 global loads at every item.
constexpr int kWTapBytes = kSliceCh * 9 * 4;           // 2304
constexpr int kWBiasOffset = 2 * kWTapBytes;           // 4608
constexpr int kWAreaBytes = kWBiasOffset + 2 * kSliceCh * 4;  // 5120

// Untiled bulk copy global -> this CTA's shared memory, completing on `bar` (16-byte aligned
// addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

__device__ __forceinline__ float tanh_approx(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

struct DwItem {
    int s, c0, x0, y0, rows;
};

__device__ __forceinline__ DwItem dw_item(int it, int H, int band_rows, int bands, int stripes, int slices) {
    DwItem d;
    const int slice = it % slices;
    it /= slices;
    const int stripe = it % stripes;
    it /= stripes;
    const int band = it % bands;
    d.s = it / bands;
    d.c0 = slice * kSliceCh;
    d.x0 = stripe * kStripe;
    d.y0 = band * band_rows;
    d.rows = min(band_rows, H - d.y0);
    return d;
}

// Slots of an item: its R + 2 input rows (image rows y0 - 1 .. y0 + R).
__host__ __device__ __forceinline__ int dw_slots(int R) { return (R + 2 + kSlotRows - 1) / kSlotRows; }

// A thread's accumulators of one output row: [column][value, gate] fp32 channel pairs. The
// gate half's taps and bias are pre-halved (exactly), so it holds h = g / 2 and
// silu(g) = g (1 + tanh(g / 2)) / 2 = h + h tanh(h).
struct DwRow {
    uint64_t a[kCols][2];
};

template <int KY>
__device__ __forceinline__ void dw_taps(DwRow& r, const uint64_t (&fv)[kCols + 2], const uint64_t (&fg)[kCols + 2],
                                        const uint64_t (&wv)[9], const uint64_t (&wg)[9]) {
#pragma unroll
    for (int kx = 0; kx < 3; ++kx)
#pragma unroll
        for (int c = 0; c < kCols; ++c) {
            r.a[c][0] = fma2(fv[c + kx], wv[KY * 3 + kx], r.a[c][0]);
            r.a[c][1] = fma2(fg[c + kx], wg[KY * 3 + kx], r.a[c][1]);
        }
}

// This thread's staged values of one input row: pixels 2w - 1 .. 2w + 2 of the stripe,
// value and gate bf16 channel pairs.
struct DwRaw {
    uint32_t v[kCols + 2], g[kCols + 2];
};

// Per-item state of a consumer thread.
struct DwStep {
    const unsigned char* px;  // this thread's first staged pixel (column 2w - 1), channel pair p, slot 0, row 0
    uint64_t* full_bar;
    uint64_t* empty_bar;
    int* err;
    uint32_t slot0;           // ring index of the item's first slot
    int lane;
    bool pok;                 // the channel pair exists
    int ncols;                // columns of the thread inside the image (0..kCols)
    int y0, R, H;             // band's first row, its row count; image height
    bf16* orow;               // output row y0, column 2w, channel pair p
    long long orow_step, ldo;
};

// Copies input row i of the item out of its slot, waiting for the slot on its first row
// and releasing it after its last. A wait that gives up has recorded the error; the thread
// then goes on with whatever the slot holds (every access stays in bounds, later waits give
// up at once) and the kernel's result is discarded by the host.
__device__ __forceinline__ void dw_fetch(const DwStep& st, int i, DwRaw& raw) {
    const uint32_t n = st.slot0 + i / kSlotRows;
    const int slot = n % kDwRing;
    const int rs = i % kSlotRows;
    if (rs == 0) mbar_wait(smem_u32(&st.full_bar[slot]), (n / kDwRing) & 1, st.err, kTimeout);
    const uint32_t* px = reinterpret_cast<const uint32_t*>(st.px + slot * kSlotBytes + rs * kRowBytes);
#pragma unroll
    for (int j = 0; j < kCols + 2; ++j) {
        raw.v[j] = px[j * (kPxBytes / 4)];
        raw.g[j] = px[j * (kPxBytes / 4) + kSliceCh / 2];
    }
    if (rs == kSlotRows - 1 || i == st.R + 1) {
        __syncwarp();
        if (st.lane == 0) mbar_arrive(smem_u32(&st.empty_bar[slot]));
    }
}

// Step i of the band: input row i (image row y0 - 1 + i, in `raw`) feeds output rows i,
// i - 1, i - 2 through tap rows 0, 1, 2; output row i - 2 is then complete. The next input
// row is fetched before the finished row is gated and stored, so its shared-memory latency
// hides behind the GLU. kInner steps (2 <= i < R) take every tap and need no bounds tests.
template <bool kInner>
__device__ __forceinline__ void dw_step(const DwStep& st, int i, DwRow& oi, DwRow& oi1, DwRow& oi2, DwRaw& raw,
                                        const uint64_t (&wv)[9], const uint64_t (&wg)[9], uint64_t bv,
                                        uint64_t bg) {
    if (!kInner && i > st.R + 1) return;
    const int y = st.y0 - 1 + i;
    const bool fin = kInner || (i >= 2 && i - 2 < st.R);
    if (kInner || (y >= 0 && y < st.H)) {
        uint64_t fv[kCols + 2], fg[kCols + 2];
#pragma unroll
        for (int j = 0; j < kCols + 2; ++j) {
            fv[j] = f2_from_bf2(raw.v[j]);
            fg[j] = f2_from_bf2(raw.g[j]);
        }
        if (fin) dw_taps<2>(oi2, fv, fg, wv, wg);
        if (kInner || (i >= 1 && i - 1 < st.R)) dw_taps<1>(oi1, fv, fg, wv, wg);
        if (kInner || i < st.R) dw_taps<0>(oi, fv, fg, wv, wg);
    }
    uint64_t t[kCols];
    if (fin) {
#pragma unroll
        for (int c = 0; c < kCols; ++c) {
            const float2 hs = f2_split(oi2.a[c][1]);
            t[c] = f2_make(tanh_approx(hs.x), tanh_approx(hs.y));
        }
    }
    if (kInner || i + 1 <= st.R + 1) dw_fetch(st, i + 1, raw);
    if (fin) {
        bf16* o = st.orow + (i - 2) * st.orow_step;
#pragma unroll
        for (int c = 0; c < kCols; ++c) {
            const uint64_t h = oi2.a[c][1];
            const float2 v = f2_split(mul2(oi2.a[c][0], fma2(h, t[c], h)));
            if (st.pok && c < st.ncols)
                *reinterpret_cast<__nv_bfloat162*>(o + c * st.ldo) = __floats2bfloat162_rn(v.x, v.y);
            oi2.a[c][0] = bv;
            oi2.a[c][1] = bg;
        }
    }
}

__global__ void __launch_bounds__(kDwThreads, 1)
    dwglu_stream_kernel(const __grid_constant__ CUtensorMap map, int S, int H, int W, int half, int band_rows,
                        int bands, int stripes, const float* __restrict__ w, const float* __restrict__ b,
                        bf16* __restrict__ out, long long ldo, int* err) {
    extern __shared__ __align__(128) unsigned char dyn[];
    __shared__ __align__(8) uint64_t full_bar[kDwRing], empty_bar[kDwRing];
    unsigned char* ring = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(dyn) + 127) & ~uintptr_t(127));
    unsigned char* wts = ring + kDwRing * kSlotBytes;  // [kDwRing][kWAreaBytes]
    const int slices = (half + kSliceCh - 1) / kSliceCh;
    const int items = S * bands * stripes * slices;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kDwRing; ++i) {
            mbar_init(smem_u32(&full_bar[i]), 1);
            mbar_init(smem_u32(&empty_bar[i]), kDwWarps);
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == kDwWarps) {  // producer
        if (lane != 0) return;
        uint32_t n = 0;
        bool ok = true;
        for (int it = blockIdx.x; ok && it < items; it += gridDim.x) {
            const DwItem d = dw_item(it, H, band_rows, bands, stripes, slices);
            const int nslots = dw_slots(d.rows);
            for (int k = 0; k < nslots; ++k, ++n) {
                const int slot = n % kDwRing;
                if (!mbar_wait(smem_u32(&empty_bar[slot]), ((n / kDwRing) & 1) ^ 1, err, kTimeout)) {
                    ok = false;
                    break;
                }
                const uint32_t fb = smem_u32(&full_bar[slot]);
                if (k == 0) {  // the item's taps and biases come with its first rows
                    const uint32_t nch = static_cast<uint32_t>(min(kSliceCh, half - d.c0));
                    const uint32_t wa = smem_u32(wts + slot * kWAreaBytes);
                    mbar_arrive_expect_tx(fb, kSlotBytes + nch * (2 * 9 * 4 + 2 * 4));
                    bulk_load(wa, w + static_cast<long long>(d.c0) * 9, nch * 36, fb);
                    bulk_load(wa + kWTapBytes, w + static_cast<long long>(half + d.c0) * 9, nch * 36, fb);
                    bulk_load(wa + kWBiasOffset, b + d.c0, nch * 4, fb);
                    bulk_load(wa + kWBiasOffset + kSliceCh * 4, b + half + d.c0, nch * 4, fb);
                } else {
                    mbar_arrive_expect_tx(fb, kSlotBytes);
                }
                tma_load_5d(&map, smem_u32(ring + slot * kSlotBytes), fb, d.c0, 0, d.x0 - 1,
                            d.y0 - 1 + k * kSlotRows, d.s);
            }
        }
        if (!ok) {  // let the copies in flight land before the block exits
            for (uint32_t k = n > kDwRing ? n - kDwRing : 0; k < n; ++k)
                mbar_wait_quiet(smem_u32(&full_bar[k % kDwRing]), (k / kDwRing) & 1);
        }
        return;
    }

    // consumer
    const int p = lane;
    DwStep st;
    st.px = ring + kCols * warp * kPxBytes + 4 * p;
    st.full_bar = full_bar;
    st.empty_bar = empty_bar;
    st.err = err;
    st.slot0 = 0;
    st.lane = lane;
    st.H = H;
    st.ldo = ldo;
    st.orow_step = static_cast<long long>(W) * ldo;
    for (int it = blockIdx.x; it < items; it += gridDim.x) {
        const DwItem d = dw_item(it, H, band_rows, bands, stripes, slices);
        const int ch = d.c0 + 2 * p;
        st.pok = ch < half;  // half is a multiple of 8: both channels of the pair exist
        // the item's first rows, and with them its taps and biases (read before the slot is released)
        DwRaw raw;
        dw_fetch(st, 0, raw);
        uint64_t wv[9], wg[9], bv = 0, bg = 0;
        {
            const unsigned char* wa = wts + (st.slot0 % kDwRing) * kWAreaBytes;
            const float2* tv = reinterpret_cast<const float2*>(wa + 72 * p);  // taps of channels 2p, 2p + 1
            const float2* tg = reinterpret_cast<const float2*>(wa + kWTapBytes + 72 * p);
            float a[18], g[18];
#pragma unroll
            for (int j = 0; j < 9; ++j) {
                const float2 x = tv[j], y = tg[j];
                a[2 * j] = x.x, a[2 * j + 1] = x.y;
                g[2 * j] = y.x, g[2 * j + 1] = y.y;
            }
#pragma unroll
            for (int t = 0; t < 9; ++t) {
                wv[t] = st.pok ? f2_make(a[t], a[9 + t]) : 0;
                wg[t] = st.pok ? f2_make(0.5f * g[t], 0.5f * g[9 + t]) : 0;
            }
            if (st.pok) {
                const float2 x = *reinterpret_cast<const float2*>(wa + kWBiasOffset + 8 * p);
                const float2 y = *reinterpret_cast<const float2*>(wa + kWBiasOffset + kSliceCh * 4 + 8 * p);
                bv = f2_make(x.x, x.y);
                bg = f2_make(0.5f * y.x, 0.5f * y.y);
            }
        }
        const int xw = d.x0 + kCols * warp;  // first column of this thread
        st.ncols = min(kCols, W - xw);
        st.y0 = d.y0;
        st.R = d.rows;
        st.orow = out + (static_cast<long long>(d.s) * H + d.y0) * st.orow_step + static_cast<long long>(xw) * ldo + ch;
        DwRow acc[3];  // output row ol of the band accumulates in acc[ol % 3]
#pragma unroll
        for (int k = 0; k < 3; ++k)
#pragma unroll
            for (int c = 0; c < kCols; ++c) {
                acc[k].a[c][0] = bv;
                acc[k].a[c][1] = bg;
            }
        // step i passes (output i, output i - 1, output i - 2) =
        // (acc[i % 3], acc[(i + 2) % 3], acc[(i + 1) % 3])
        dw_step<false>(st, 0, acc[0], acc[2], acc[1], raw, wv, wg, bv, bg);
        dw_step<false>(st, 1, acc[1], acc[0], acc[2], raw, wv, wg, bv, bg);
        int i = 2;
        for (; i + 3 <= d.rows; i += 3) {
            dw_step<true>(st, i, acc[2], acc[1], acc[0], raw, wv, wg, bv, bg);
            dw_step<true>(st, i + 1, acc[0], acc[2], acc[1], raw, wv, wg, bv, bg);
            dw_step<true>(st, i + 2, acc[1], acc[0], acc[2], raw, wv, wg, bv, bg);
        }
        // the last two to four steps (through i = R + 1), with bounds tests
        dw_step<false>(st, i, acc[2], acc[1], acc[0], raw, wv, wg, bv, bg);
        dw_step<false>(st, i + 1, acc[0], acc[2], acc[1], raw, wv, wg, bv, bg);
        dw_step<false>(st, i + 2, acc[1], acc[0], acc[2], raw, wv, wg, bv, bg);
        dw_step<false>(st, i + 3, acc[2], acc[1], acc[0], raw, wv, wg, bv, bg);
        if (*reinterpret_cast<volatile int*>(err) != 0) return;
        st.slot0 += dw_slots(d.rows);
    }
}

size_t dwglu_stream_smem() { return static_cast<size_t>(kDwRing) * (kSlotBytes + kWAreaBytes) + 128; }

// Any type / channel count: one output channel per thread.
template <class T>
__global__ void dwglu_scalar_kernel(const T* __restrict__ in, long long ldi, int S, int H, int W, int half,
                                    const float* __restrict__ w, const float* __restrict__ b, T* __restrict__ out,
                                    long long ldo) {
    const long long total = static_cast<long long>(S) * H * W * half;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % half);
        const long long pix = i / half;
        const int x = static_cast<int>(pix % W);
        const int y = static_cast<int>((pix / W) % H);
        const long long s = pix / (static_cast<long long>(W) * H);
        float dv = 0.f, gv = 0.f;
        for (int ky = 0; ky < 3; ++ky) {
            const int iy = y + ky - 1;
            if (iy < 0 || iy >= H) continue;
            for (int kx = 0; kx < 3; ++kx) {
                const int ix = x + kx - 1;
                if (ix < 0 || ix >= W) continue;
                const T* src = in + ((s * H + iy) * W + ix) * ldi;
                dv = fmaf(to_f(src[c]), w[c * 9 + ky * 3 + kx], dv);
                gv = fmaf(to_f(src[half + c]), w[(half + c) * 9 + ky * 3 + kx], gv);
            }
        }
        dv += b[c];
        gv += b[half + c];
        out[pix * ldo + c] = from_f<T>(dv * silu(gv));
    }
}

__global__ void depthwise_plain_kernel(const float* __restrict__ in, int S, int H, int W, int C,
                                       const float* __restrict__ w, const float* __restrict__ b,
                                       float* __restrict__ out) {
    const long long total = static_cast<long long>(S) * H * W * C;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(i % C);
        const long long pix = i / C;
        const int x = static_cast<int>(pix % W);
        const int y = static_cast<int>((pix / W) % H);
        const long long s = pix / (static_cast<long long>(W) * H);
        float acc = 0.f;
        for (int ky = 0; ky < 3; ++ky) {
            const int iy = y + ky - 1;
            if (iy < 0 || iy >= H) continue;
            for (int kx = 0; kx < 3; ++kx) {
                const int ix = x + kx - 1;
                if (ix < 0 || ix >= W) continue;
                acc = fmaf(in[((s * H + iy) * W + ix) * C + c], w[c * 9 + ky * 3 + kx], acc);
            }
        }
        if (b) acc += b[c];
        out[i] = acc;
    }
}

int grid_for(long long n) {
    long long g = (n + 255) / 256;
    if (g > 148LL * 16) g = 148LL * 16;
    return static_cast<int>(g < 1 ? 1 : g);
}

}  // namespace

template <class T>
void depthwise_glu(const T* in, long long ldi, int S, int H, int W, int E, const float* w, const float* b, T* out,
                   long long ldo, int* err, cudaStream_t st) {
    SANA_REQUIRE(E % 2 == 0, "channel count must be even");
    const int half = E / 2;
    const long long pixels = static_cast<long long>(S) * H * W;
    if (pixels == 0 || half == 0) return;
    bool vec = sizeof(T) == 2 && half % 8 == 0 && ldi % 8 == 0 && ldo % 2 == 0 &&
               (reinterpret_cast<uintptr_t>(in) & 15) == 0 && (reinterpret_cast<uintptr_t>(out) & 3) == 0;
    // bf16 channel counts the stream kernel tiles (half % 8 == 0) must take it: a refusal for
    // pointers or row strides alone is an error, not a slow fallback. The scalar kernel is
    // the fp32 check mode's path and that of odd channel counts (small test models).
    SANA_REQUIRE(vec || sizeof(T) != 2 || half % 8 != 0,
                 "depthwise_glu: bf16 rows must be 16-byte aligned (input) and 4-byte aligned (output)");
    if (vec) {
        // the kernel copies each work item's taps and biases with bulk copies from 16-byte boundaries
        SANA_REQUIRE((reinterpret_cast<uintptr_t>(w) & 15) == 0 && (reinterpret_cast<uintptr_t>(b) & 15) == 0,
                     "depthwise_glu: the bf16 path needs 16-byte aligned tap and bias arrays");
        static int device_sms[64] = {0};
        static PerDeviceOnce attr;
        int dev = 0;
        SANA_CUDA(cudaGetDevice(&dev));
        if (attr.pending()) {
            SANA_CUDA(cudaFuncSetAttribute(dwglu_stream_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(dwglu_stream_smem())));
            attr.mark();
        }
        int& sms = device_sms[dev & 63];
        if (sms == 0) SANA_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        const int slices = ceil_div(half, kSliceCh), stripes = ceil_div(W, kStripe);
        // Split the image rows into bands (each re-reading a one-row halo) only when the
        // sequences, stripes and channel slices alone give fewer than two items per SM.
        const long long base = static_cast<long long>(S) * stripes * slices;
        int bands = static_cast<int>(std::min<long long>((2LL * sms + base - 1) / base, (H + 7) / 8));
        if (bands < 1) bands = 1;
        const int band_rows = ceil_div(H, bands);
        bands = ceil_div(H, band_rows);
        const long long items = base * bands;
        SANA_REQUIRE(items < (1LL << 31), "depthwise_glu: too many work items");
        // [S, H, W, 2 halves, half channels]; box = 64 channels x 2 halves x (32 + 2) pixels x rows
        CUtensorMap map;
        const cuuint64_t dims[5] = {static_cast<cuuint64_t>(half), 2, static_cast<cuuint64_t>(W),
                                    static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(S)};
        const cuuint64_t strides[4] = {static_cast<cuuint64_t>(half) * 2, static_cast<cuuint64_t>(ldi) * 2,
                                       static_cast<cuuint64_t>(ldi) * 2 * W,
                                       static_cast<cuuint64_t>(ldi) * 2 * W * H};
        const cuuint32_t box[5] = {kSliceCh, 2, kStripePx, kSlotRows, 1};
        tma_encode_tiled(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, in, dims, strides, box,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
        const int grid = static_cast<int>(std::min<long long>(items, sms));
        dwglu_stream_kernel<<<grid, kDwThreads, dwglu_stream_smem(), st>>>(
            map, S, H, W, half, band_rows, bands, stripes, w, b, reinterpret_cast<bf16*>(out), ldo, err);
    } else {
        dwglu_scalar_kernel<T><<<grid_for(pixels * half), 256, 0, st>>>(in, ldi, S, H, W, half, w, b, out, ldo);
    }
    SANA_CUDA(cudaGetLastError());
}

void depthwise3x3(const float* in, int S, int H, int W, int C, const float* w, const float* b, float* out,
                  cudaStream_t st) {
    const long long n = static_cast<long long>(S) * H * W * C;
    if (n == 0) return;
    depthwise_plain_kernel<<<grid_for(n), 256, 0, st>>>(in, S, H, W, C, w, b, out);
    SANA_CUDA(cudaGetLastError());
}

template void depthwise_glu<float>(const float*, long long, int, int, int, int, const float*, const float*, float*,
                                   long long, int*, cudaStream_t);
template void depthwise_glu<bf16>(const bf16*, long long, int, int, int, int, const float*, const float*, bf16*,
                                  long long, int*, cudaStream_t);

}  // namespace sana
