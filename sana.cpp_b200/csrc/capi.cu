// The C ABI of include/sana_cuda.h over the Engine and the kernels.
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <new>
#include <random>
#include <string>
#include <vector>

#include <algorithm>
#include <set>
#include <stdexcept>

#include <cuda.h>

#include "engine.h"
#include "gguf.h"
#include "sana_cuda.h"
#include "vae.h"

struct sana_cuda_ctx {
    std::unique_ptr<sana::Engine> eng;
    std::string err;
    std::unique_ptr<sana::VaeDecoder> vae;  // after eng: destroyed first
};

namespace {

using sana::bf16;
using sana::DevBuf;

// The stream of the handle the current entry point works on: every transfer of the
// single-op entry points is ordered on it (set by engine()).
thread_local cudaStream_t tl_stream = nullptr;

template <class F>
int guard(sana_cuda_ctx* ctx, F&& f) {
    if (!ctx) return SANA_ERR_INVALID;
    try {
        f();
        return SANA_OK;
    } catch (const std::invalid_argument& e) {
        ctx->err = e.what();
        return SANA_ERR_INVALID;
    } catch (const sana::TimeoutError& e) {
        ctx->err = e.what();
        return SANA_ERR_TIMEOUT;
    } catch (const sana::CudaError& e) {
        ctx->err = e.what();
        return SANA_ERR_CUDA;
    } catch (const std::bad_alloc&) {
        ctx->err = "out of host memory";
        return SANA_ERR_NOMEM;
    } catch (const std::exception& e) {
        ctx->err = e.what();
        return SANA_ERR_STATE;
    }
}

// The reference's default scheduler config with `flow_shift`.
sana::SchedConfig default_sched(float flow_shift) {
    sana::SchedConfig c;
    c.flow_shift = flow_shift;
    return c;
}

// A C-ABI scheduler config (NULL = the defaults), checked as validate_scheduler_config
// checks its numeric fields (scheduler.cpp:8-24).
sana::SchedConfig sched_of(const sana_scheduler_config* p) {
    sana::SchedConfig c;
    if (p) {
        c.num_train_timesteps = p->num_train_timesteps;
        c.flow_shift = p->flow_shift;
        c.flow_sigmas = p->use_flow_sigmas != 0;
        c.solver_order = p->solver_order;
        c.lower_order_final = p->lower_order_final != 0;
        c.final_sigmas_zero = p->final_sigmas_zero != 0;
        c.heun = p->solver_heun != 0;
    }
    sana::scheduler_validate(c);
    return c;
}

// --- host-side layout / precision helpers for the single-op entry points ----------------
uint16_t f32_to_bf16_bits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((u >> 16) | 0x40);  // NaN
    const uint32_t rounding = 0x7fffu + ((u >> 16) & 1u);
    return static_cast<uint16_t>((u + rounding) >> 16);
}
float bf16_bits_to_f32(uint16_t h) {
    const uint32_t u = static_cast<uint32_t>(h) << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// A device copy of host fp32 data in the activation type of the handle's mode.
struct ActBuf {
    DevBuf buf;
    bool bf = false;
    size_t n = 0;
    void upload(const float* host, size_t count, bool as_bf16) {
        bf = as_bf16;
        n = count;
        buf.ensure(std::max<size_t>(count, 1) * (bf ? 2 : 4));
        if (count == 0) return;
        if (bf) {
            std::vector<uint16_t> h(count);
            for (size_t i = 0; i < count; ++i) h[i] = f32_to_bf16_bits(host[i]);
            SANA_CUDA(cudaMemcpyAsync(buf.get(), h.data(), count * 2, cudaMemcpyHostToDevice, tl_stream));
        } else {
            SANA_CUDA(cudaMemcpyAsync(buf.get(), host, count * 4, cudaMemcpyHostToDevice, tl_stream));
        }
    }
    void alloc(size_t count, bool as_bf16) {
        bf = as_bf16;
        n = count;
        buf.ensure(std::max<size_t>(count, 1) * (bf ? 2 : 4));
    }
    void download(float* host) const {
        if (n == 0) return;
        if (bf) {
            std::vector<uint16_t> h(n);
            SANA_CUDA(cudaMemcpyAsync(h.data(), buf.get(), n * 2, cudaMemcpyDeviceToHost, tl_stream));
            SANA_CUDA(cudaStreamSynchronize(tl_stream));
            for (size_t i = 0; i < n; ++i) host[i] = bf16_bits_to_f32(h[i]);
        } else {
            SANA_CUDA(cudaMemcpyAsync(host, buf.get(), n * 4, cudaMemcpyDeviceToHost, tl_stream));
            SANA_CUDA(cudaStreamSynchronize(tl_stream));
        }
    }
    void* get() const { return buf.get(); }
};

DevBuf f32_upload(const float* host, size_t n) {
    DevBuf b;
    b.ensure(std::max<size_t>(n, 1) * 4);
    if (n) SANA_CUDA(cudaMemcpyAsync(b.get(), host, n * 4, cudaMemcpyHostToDevice, tl_stream));
    return b;
}

// [rows, cols] -> [cols, rows]
std::vector<float> transpose(const float* src, size_t rows, size_t cols) {
    std::vector<float> out(rows * cols);
    for (size_t r = 0; r < rows; ++r)
        for (size_t c = 0; c < cols; ++c) out[c * rows + r] = src[r * cols + c];
    return out;
}

// [B, H, T, D] -> token rows [B*T, H*D] (split_heads_3d inverse, transformer_ops.cpp:133)
std::vector<float> heads_to_tokens(const float* x, int B, int H, int T, int D) {
    std::vector<float> out(static_cast<size_t>(B) * T * H * D);
    for (int b = 0; b < B; ++b)
        for (int h = 0; h < H; ++h)
            for (int t = 0; t < T; ++t)
                std::memcpy(&out[(static_cast<size_t>(b) * T + t) * H * D + static_cast<size_t>(h) * D],
                            x + ((static_cast<size_t>(b) * H + h) * T + t) * D, D * sizeof(float));
    return out;
}

void tokens_to_heads(const float* x, int B, int H, int T, int D, float* out) {
    for (int b = 0; b < B; ++b)
        for (int h = 0; h < H; ++h)
            for (int t = 0; t < T; ++t)
                std::memcpy(out + ((static_cast<size_t>(b) * H + h) * T + t) * D,
                            &x[(static_cast<size_t>(b) * T + t) * H * D + static_cast<size_t>(h) * D],
                            D * sizeof(float));
}

// NCHW [B, C, HW] <-> NHWC token rows [B*HW, C]
std::vector<float> nchw_to_tokens(const float* x, int B, int C, int HW) {
    std::vector<float> out(static_cast<size_t>(B) * C * HW);
    for (int b = 0; b < B; ++b)
        for (int c = 0; c < C; ++c)
            for (int t = 0; t < HW; ++t)
                out[(static_cast<size_t>(b) * HW + t) * C + c] = x[(static_cast<size_t>(b) * C + c) * HW + t];
    return out;
}

void tokens_to_nchw(const float* x, int B, int C, int HW, float* out) {
    for (int b = 0; b < B; ++b)
        for (int c = 0; c < C; ++c)
            for (int t = 0; t < HW; ++t)
                out[(static_cast<size_t>(b) * C + c) * HW + t] = x[(static_cast<size_t>(b) * HW + t) * C + c];
}

sana::Epilogue epi(void* out, bool bf, long long ldo, const float* bias = nullptr, int act = sana::kActNone) {
    sana::Epilogue e;
    e.out = out;
    e.out_bf16 = bf ? 1 : 0;
    e.ldo = ldo;
    e.bias = bias;
    e.act = act;
    return e;
}

void run_gemm(sana::Engine& eng, const ActBuf& A, long long lda, const ActBuf& B, long long ldb, int M, int N, int K,
              const sana::Epilogue& e) {
    sana::GemmProblem p;
    p.A = A.get();
    p.a_bf16 = A.bf;
    p.lda = lda;
    p.B = B.get();
    p.b_bf16 = B.bf;
    p.ldb = ldb;
    p.M = M;
    p.N = N;
    p.K = K;
    p.ep = e;
    sana::gemm(p, eng.err(), eng.stream(), eng.num_sms());
}

void finish(sana::Engine& eng) {
    SANA_CUDA(cudaStreamSynchronize(eng.stream()));
    eng.check_device_error();
}

sana::Engine& engine(sana_cuda_ctx* ctx) {
    if (!ctx->eng) throw std::runtime_error("handle has no engine");
    tl_stream = ctx->eng->stream();
    return *ctx->eng;
}

// Device -> host copy ordered after the handle's work.
void d2h(void* host, const void* dev, size_t bytes) {
    if (!bytes) return;
    SANA_CUDA(cudaMemcpyAsync(host, dev, bytes, cudaMemcpyDeviceToHost, tl_stream));
    SANA_CUDA(cudaStreamSynchronize(tl_stream));
}

}  // namespace

// --- fixed scratch of sana_op_linear_attention_noalloc ----------------------------------
// One array per device, part of this library's device image: it holds 8 MiB of a device's
// memory from the time the CUDA runtime loads this library's device code there. Every
// handle, stream and host thread on a device shares it.
static __device__ __align__(256) float g_linattn_scratch[SANA_NOALLOC_SCRATCH_BYTES / sizeof(float)];

namespace {

constexpr int kScratchMaxDevices = 64;
std::mutex g_scratch_mu;
float* g_scratch_addr[kScratchMaxDevices] = {};
unsigned long long g_scratch_ctx[kScratchMaxDevices] = {};  // context id the address belongs to

// The unique id of the calling thread's current CUDA context (cuCtxGetId: never reused within
// a process, so a context re-created by cudaDeviceReset gets a new one).
unsigned long long current_context_id() {
    using GetCurrent = CUresult (*)(CUcontext*);
    using GetId = CUresult (*)(CUcontext, unsigned long long*);
    static GetCurrent get_current = nullptr;
    static GetId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<GetCurrent>(p);
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<GetId>(p);
    });
    if (!get_current || !get_id) throw sana::CudaError("cuCtxGetCurrent / cuCtxGetId are not available");
    CUcontext c = nullptr;
    unsigned long long id = 0;
    if (get_current(&c) != CUDA_SUCCESS || !c || get_id(c, &id) != CUDA_SUCCESS)
        throw sana::CudaError("no current CUDA context for the fixed scratch");
    return id;
}

// The device address of g_linattn_scratch on `device`, which the caller has made current.
// Looked up with cudaGetSymbolAddress on the first call per device and remembered together
// with the id of the context it belongs to; a call in a different context of that device
// (the primary context re-created after cudaDeviceReset) looks it up again.
float* linattn_scratch(int device) {
    SANA_REQUIRE(device >= 0 && device < kScratchMaxDevices, "device ordinal out of range for the fixed scratch");
    const unsigned long long ctx = current_context_id();
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_addr[device] || g_scratch_ctx[device] != ctx) {
        void* p = nullptr;
        SANA_CUDA(cudaGetSymbolAddress(&p, g_linattn_scratch));
        g_scratch_addr[device] = static_cast<float*>(p);
        g_scratch_ctx[device] = ctx;
    }
    return g_scratch_addr[device];
}

// Makes `device` current for the lifetime of the guard and restores the previous one.
struct CurrentDevice {
    int prev = -1;
    explicit CurrentDevice(int device) {
        SANA_CUDA(cudaGetDevice(&prev));
        if (prev != device) SANA_CUDA(cudaSetDevice(device));
    }
    ~CurrentDevice() {
        int now = -1;
        if (cudaGetDevice(&now) == cudaSuccess && now != prev) cudaSetDevice(prev);
    }
};

}  // namespace

extern "C" {

int sana_cuda_create(int device, int mode, sana_cuda_ctx** out) {
    if (!out) return SANA_ERR_INVALID;
    *out = nullptr;
    auto* ctx = new (std::nothrow) sana_cuda_ctx();
    if (!ctx) return SANA_ERR_NOMEM;
    int rc = guard(ctx, [&] { ctx->eng = std::make_unique<sana::Engine>(device, mode); });
    if (rc != SANA_OK) {
        // keep the handle so the caller can read the message; it has no engine
        *out = ctx;
        return rc;
    }
    *out = ctx;
    return SANA_OK;
}

void sana_cuda_destroy(sana_cuda_ctx* ctx) { delete ctx; }

const char* sana_cuda_last_error(const sana_cuda_ctx* ctx) { return ctx ? ctx->err.c_str() : "null handle"; }

void* sana_cuda_stream(sana_cuda_ctx* ctx) { return (ctx && ctx->eng) ? ctx->eng->stream() : nullptr; }

int sana_cuda_set_stream(sana_cuda_ctx* ctx, void* stream) {
    return guard(ctx, [&] { engine(ctx).set_stream(static_cast<cudaStream_t>(stream)); });
}

int sana_cuda_synchronize(sana_cuda_ctx* ctx) { return guard(ctx, [&] { finish(engine(ctx)); }); }

int sana_cuda_set_wait_limit(sana_cuda_ctx* ctx, unsigned long long ns) {
    return guard(ctx, [&] { engine(ctx).set_wait_limit_ns(ns); });
}

unsigned long long sana_cuda_wait_limit(const sana_cuda_ctx* ctx) {
    return (ctx && ctx->eng) ? ctx->eng->wait_limit_ns() : 0;
}

int sana_cuda_selftest_wait(sana_cuda_ctx* ctx, const int* flag, int expect) {
    return guard(ctx, [&] {
        SANA_REQUIRE(flag != nullptr, "flag must be a device address");
        sana::Engine& eng = engine(ctx);
        sana::wait_flag(flag, expect, eng.err(), eng.stream());
        finish(eng);
    });
}

int sana_cuda_last_launch_count(const sana_cuda_ctx* ctx) {
    return (ctx && ctx->eng) ? ctx->eng->last_launches() : 0;
}

void sana_cuda_gemm_counts(long long* tensor_core, long long* cuda_core) { sana::gemm_counts(tensor_core, cuda_core); }

int sana_cuda_upload_weights(sana_cuda_ctx* ctx, const sana_dims* dims, const float* const* model,
                             const float* const* blocks, int layout) {
    return guard(ctx, [&] {
        SANA_REQUIRE(dims != nullptr, "dims must not be null");
        sana::Dims d;
        d.n_blocks = dims->n_blocks;
        d.C = dims->hidden;
        d.Cl = dims->latent_channels;
        d.Din = dims->caption_dim;
        d.E = dims->ff_expanded;
        d.Hs = dims->self_heads;
        d.Hc = dims->cross_heads;
        engine(ctx).upload(d, model, blocks, layout);
    });
}

// --- GGUF weight files ---------------------------------------------------------------------
namespace {

// The reference's tensor names (load_caption_weights / load_block_weights /
// load_denoiser_weights, transformer.cpp:166-488); every tensor is required, as there.
const char* const kCaptionNames[4] = {"caption_projection.linear_1.weight", "caption_projection.linear_1.bias",
                                      "caption_projection.linear_2.weight", "caption_projection.linear_2.bias"};
const char* const kDenoiserNames[12] = {
    "patch_embed.proj.weight", "patch_embed.proj.bias",
    "time_embed.emb.timestep_embedder.linear_1.weight", "time_embed.emb.timestep_embedder.linear_1.bias",
    "time_embed.emb.timestep_embedder.linear_2.weight", "time_embed.emb.timestep_embedder.linear_2.bias",
    "time_embed.linear.weight", "time_embed.linear.bias", "caption_norm.weight", "scale_shift_table",
    "proj_out.weight", "proj_out.bias"};
// SanaBlockWeights field -> tensor suffix (nullptr: the loader's default, a zero bias or an
// identity norm, transformer.cpp:361-398)
const char* const kBlockNames[26] = {
    "scale_shift_table", nullptr, nullptr, "attn1.to_q.weight", nullptr, "attn1.to_k.weight", nullptr,
    "attn1.to_v.weight", nullptr, "attn1.to_out.0.weight", "attn1.to_out.0.bias", "attn2.to_q.weight",
    "attn2.to_q.bias", "attn2.to_k.weight", "attn2.to_k.bias", "attn2.to_v.weight", "attn2.to_v.bias",
    "attn2.to_out.0.weight", "attn2.to_out.0.bias", nullptr, nullptr, "ff.conv_inverted.weight",
    "ff.conv_inverted.bias", "ff.conv_depth.weight", "ff.conv_depth.bias", "ff.conv_point.weight"};

// block_weight_name / parse_trailing_index / find_block_prefixes (transformer.cpp:26-55, 401-430):
// the prefixes of every "<prefix>.scale_shift_table", numerically ordered on a trailing index.
bool trailing_index(const std::string& p, std::string* stem, size_t* idx) {
    const size_t dot = p.rfind('.');
    if (dot == std::string::npos || dot + 1 >= p.size()) return false;
    const std::string tail = p.substr(dot + 1);
    for (char ch : tail)
        if (ch < '0' || ch > '9') return false;
    *stem = p.substr(0, dot);
    *idx = static_cast<size_t>(std::stoull(tail));
    return true;
}

std::vector<std::string> block_prefixes(const sana::GgufFile& f) {
    const std::string suffix = ".scale_shift_table";
    std::set<std::string> uniq;
    for (const auto& t : f.tensors())
        if (t.name.size() > suffix.size() && t.name.compare(t.name.size() - suffix.size(), suffix.size(), suffix) == 0)
            uniq.insert(t.name.substr(0, t.name.size() - suffix.size()));
    std::vector<std::string> v(uniq.begin(), uniq.end());
    std::sort(v.begin(), v.end(), [](const std::string& a, const std::string& b) {
        std::string sa, sb;
        size_t ia = 0, ib = 0;
        if (trailing_index(a, &sa, &ia) && trailing_index(b, &sb, &ib) && sa == sb) return ia < ib;
        return a < b;
    });
    return v;
}

// An fp32 tensor of the file with the given rank; the reference reads GGUF payloads as
// float32 only (weights_io.cpp:331-351).
const float* tensor_f32(const sana::GgufFile& f, const std::string& name, size_t rank,
                        std::vector<int64_t>* shape_out) {
    const sana::GgufTensor* t = f.find(name);
    if (!t) throw std::invalid_argument("weight name not found in weight index: " + name);
    if (t->type != sana::kGgufF32) throw std::runtime_error("only float32 saved weights are supported: " + name);
    if (t->shape.size() != rank)
        throw std::runtime_error(name + " must be rank " + std::to_string(rank) + " in " + f.path());
    if (shape_out) *shape_out = t->shape;
    return reinterpret_cast<const float*>(t->data);
}

void require_shape(const std::string& name, const std::vector<int64_t>& got, const std::vector<int64_t>& want) {
    if (got != want) {
        std::string g, w;
        for (auto v : got) g += std::to_string(v) + ",";
        for (auto v : want) w += std::to_string(v) + ",";
        throw std::runtime_error(name + " has shape {" + g + "}, expected {" + w + "}");
    }
}

// Expected shape of SanaBlockWeights field i ([out, in] linear weights, conv [out, in, kh, kw]).
std::vector<int64_t> block_shape(int i, int64_t C, int64_t E) {
    switch (i) {
        case 0: return {6, C};
        case 10: case 12: case 14: case 16: case 18: return {C};
        case 21: return {E, C, 1, 1};
        case 22: case 24: return {E};
        case 23: return {E, 1, 3, 3};
        case 25: return {C, E / 2, 1, 1};
        default: return {C, C};  // the eight attention projections
    }
}

}  // namespace

struct sana_gguf {
    std::unique_ptr<sana::GgufFile> file;
};

int sana_gguf_open(const char* path, sana_gguf** out, char* err, size_t err_len) {
    if (!path || !out) return SANA_ERR_INVALID;
    *out = nullptr;
    try {
        auto h = std::make_unique<sana_gguf>();
        h->file = std::make_unique<sana::GgufFile>(path);
        *out = h.release();
        return SANA_OK;
    } catch (const std::exception& e) {
        if (err && err_len) std::snprintf(err, err_len, "%s", e.what());
        return SANA_ERR_STATE;
    }
}

void sana_gguf_close(sana_gguf* f) { delete f; }

int sana_gguf_tensor_count(const sana_gguf* f) { return f ? static_cast<int>(f->file->tensors().size()) : -1; }

int sana_gguf_find(const sana_gguf* f, const char* name) {
    if (!f || !name) return -1;
    const sana::GgufTensor* t = f->file->find(name);
    return t ? static_cast<int>(t - f->file->tensors().data()) : -1;
}

int sana_gguf_tensor_info(const sana_gguf* f, int i, const char** name, int* type, int* rank, int64_t* shape,
                          int max_rank, const void** data, uint64_t* nbytes) {
    if (!f || i < 0 || i >= static_cast<int>(f->file->tensors().size())) return SANA_ERR_INVALID;
    const sana::GgufTensor& t = f->file->tensors()[static_cast<size_t>(i)];
    if (name) *name = t.name.c_str();
    if (type) *type = static_cast<int>(t.type);
    if (rank) *rank = static_cast<int>(t.shape.size());
    if (shape)
        for (int d = 0; d < max_rank && d < static_cast<int>(t.shape.size()); ++d) shape[d] = t.shape[static_cast<size_t>(d)];
    if (data) *data = t.data;
    if (nbytes) *nbytes = t.nbytes;
    return SANA_OK;
}

int sana_gguf_tensor_offset(const sana_gguf* f, int i, uint64_t* offset) {
    if (!f || !offset || i < 0 || i >= static_cast<int>(f->file->tensors().size())) return SANA_ERR_INVALID;
    *offset = f->file->tensors()[static_cast<size_t>(i)].file_offset;
    return SANA_OK;
}

int sana_cuda_upload_gguf(sana_cuda_ctx* ctx, const char* model_path, const char* caption_path,
                          const char* denoiser_path, int self_heads, int cross_heads, sana_dims* dims_out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(model_path && caption_path && denoiser_path, "weight file paths must not be null");
        if (self_heads <= 0) throw std::invalid_argument("self_num_heads must be greater than 0");
        if (cross_heads <= 0) throw std::invalid_argument("cross_num_heads must be greater than 0");
        const sana::GgufFile mf(model_path), cf(caption_path), df(denoiser_path);
        std::vector<int64_t> sh;
        // dimensions from the caption, patch and first block tensors ([out, in] linear weights)
        const float* model[16];
        model[0] = tensor_f32(cf, kCaptionNames[0], 2, &sh);
        const int64_t C = sh[0], Din = sh[1];
        model[1] = tensor_f32(cf, kCaptionNames[1], 1, &sh);
        require_shape(kCaptionNames[1], sh, {C});
        model[2] = tensor_f32(cf, kCaptionNames[2], 2, &sh);
        require_shape(kCaptionNames[2], sh, {C, C});
        model[3] = tensor_f32(cf, kCaptionNames[3], 1, &sh);
        require_shape(kCaptionNames[3], sh, {C});
        model[4] = tensor_f32(df, kDenoiserNames[0], 4, &sh);
        const int64_t Cl = sh[1];
        require_shape(kDenoiserNames[0], sh, {C, Cl, 1, 1});
        const std::vector<std::vector<int64_t>> dshape = {
            {C, Cl, 1, 1}, {C}, {C, 256}, {C}, {C, C}, {C}, {6 * C, C}, {6 * C}, {C}, {2, C}, {Cl, C}, {Cl}};
        for (int i = 1; i < 12; ++i) {
            model[4 + i] = tensor_f32(df, kDenoiserNames[i], dshape[static_cast<size_t>(i)].size(), &sh);
            require_shape(kDenoiserNames[i], sh, dshape[static_cast<size_t>(i)]);
        }
        const std::vector<std::string> prefixes = block_prefixes(mf);
        if (prefixes.empty()) throw std::invalid_argument("weight index does not contain any prefixed model blocks");
        std::vector<const float*> blocks(26 * prefixes.size(), nullptr);
        int64_t E = 0;
        for (size_t b = 0; b < prefixes.size(); ++b) {
            const float** w = blocks.data() + 26 * b;
            for (int i = 0; i < 26; ++i) {
                if (!kBlockNames[i]) continue;
                const std::string name = prefixes[b] + "." + kBlockNames[i];
                const sana::GgufTensor* t = mf.find(name);
                if (!t) throw std::invalid_argument("weight name not found in weight index: " + name);
                w[i] = tensor_f32(mf, name, t->shape.size(), &sh);
                if (i == 21 && b == 0) E = sh.size() == 4 ? sh[0] : 0;
                // load_block_weights' checks (transformer.cpp:310-359), with the model's sizes
                require_shape(name, sh, block_shape(i, C, E));
            }
        }
        if (E <= 0 || E % 2 != 0) throw std::runtime_error("ff point conv input channels must match split GLUMB width");
        if (C % self_heads != 0)
            throw std::runtime_error("self attention hidden size must be divisible by self_num_heads");
        if (C % cross_heads != 0)
            throw std::runtime_error("cross attention hidden size must be divisible by cross_num_heads");
        sana::Dims d;
        d.n_blocks = static_cast<int>(prefixes.size());
        d.C = static_cast<int>(C);
        d.Cl = static_cast<int>(Cl);
        d.Din = static_cast<int>(Din);
        d.E = static_cast<int>(E);
        d.Hs = self_heads;
        d.Hc = cross_heads;
        engine(ctx).upload(d, model, blocks.data(), sana::kLayoutTorch);
        if (dims_out) {
            dims_out->n_blocks = d.n_blocks;
            dims_out->hidden = d.C;
            dims_out->latent_channels = d.Cl;
            dims_out->caption_dim = d.Din;
            dims_out->ff_expanded = d.E;
            dims_out->self_heads = d.Hs;
            dims_out->cross_heads = d.Hc;
        }
    });
}

int sana_cuda_set_cross_qk_norm(sana_cuda_ctx* ctx, int enable, const float* const* q_weights,
                                const float* const* k_weights, float eps) {
    return guard(ctx, [&] { engine(ctx).set_cross_qk_norm(enable != 0, q_weights, k_weights, eps); });
}

int sana_cuda_denoise_loop(sana_cuda_ctx* ctx, const float* latents, int B, int H, int W, const float* enc, int L,
                           int enc_dim, const float* bias, float guidance, int num_steps, float flow_shift,
                           float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(latents && enc && out, "latents, encoder states and output must not be null");
        engine(ctx).denoise_loop(latents, B, H, W, enc, L, enc_dim, bias, guidance, num_steps,
                                 default_sched(flow_shift), out);
    });
}

int sana_cuda_denoise_loop_config(sana_cuda_ctx* ctx, const sana_scheduler_config* config, const float* latents,
                                  int B, int H, int W, const float* enc, int L, int enc_dim, const float* bias,
                                  float guidance, int num_steps, float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(latents && enc && out, "latents, encoder states and output must not be null");
        engine(ctx).denoise_loop(latents, B, H, W, enc, L, enc_dim, bias, guidance, num_steps, sched_of(config),
                                 out);
    });
}

int sana_cuda_denoise_loop_device(sana_cuda_ctx* ctx, const float* latents, int B, int H, int W, const float* enc,
                                  int L, int enc_dim, const float* bias, float guidance, int num_steps,
                                  float flow_shift, float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(latents && enc && out, "latents, encoder states and output must not be null");
        engine(ctx).denoise_loop_device(latents, B, H, W, enc, L, enc_dim, bias, guidance, num_steps,
                                        default_sched(flow_shift), out);
    });
}

int sana_cuda_cfg_pair_export(sana_cuda_ctx* ctx, size_t max_latent_elems, void* handle) {
    return guard(ctx, [&] {
        SANA_REQUIRE(handle, "handle must not be null");
        engine(ctx).pair_export(max_latent_elems, handle);
    });
}

int sana_cuda_cfg_pair_connect(sana_cuda_ctx* ctx, int branch, const void* peer_handle) {
    return guard(ctx, [&] {
        SANA_REQUIRE(peer_handle, "peer handle must not be null");
        engine(ctx).pair_connect(branch, peer_handle);
    });
}

int sana_cuda_cfg_pair_close(sana_cuda_ctx* ctx) {
    return guard(ctx, [&] { engine(ctx).pair_close(); });
}

int sana_cuda_denoise_loop_pair_device(sana_cuda_ctx* ctx, const float* latents, int B, int H, int W,
                                       const float* enc, int L, int enc_dim, const float* bias, float guidance,
                                       int num_steps, float flow_shift, float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(latents && enc && out, "latents, encoder states and output must not be null");
        engine(ctx).denoise_loop_pair_device(latents, B, H, W, enc, L, enc_dim, bias, guidance, num_steps,
                                             default_sched(flow_shift), out);
    });
}

int sana_cuda_time_embed(sana_cuda_ctx* ctx, const float* timesteps, int S, float* emb, float* tmod) {
    return guard(ctx, [&] {
        SANA_REQUIRE(timesteps, "timesteps must not be null");
        sana::Engine& eng = engine(ctx);
        eng.time_embed(timesteps, S, emb, tmod);
        eng.check_device_error();
    });
}

int sana_cuda_denoise_step(sana_cuda_ctx* ctx, float* latents, int B, int H, int W, const float* context, int L,
                           const float* bias, float guidance, float timestep, const float* sigmas, int n_sigmas,
                           int* step_index, int* lower_order_count, float* history, int* n_history) {
    return sana_cuda_denoise_step_config(ctx, nullptr, latents, B, H, W, context, L, bias, guidance, timestep, sigmas,
                                         n_sigmas, step_index, lower_order_count, history, n_history);
}

int sana_cuda_denoise_step_config(sana_cuda_ctx* ctx, const sana_scheduler_config* config, float* latents, int B,
                                  int H, int W, const float* context, int L, const float* bias, float guidance,
                                  float timestep, const float* sigmas, int n_sigmas, int* step_index,
                                  int* lower_order_count, float* history, int* n_history) {
    return guard(ctx, [&] {
        SANA_REQUIRE(latents && context && sigmas && step_index && lower_order_count && n_history,
                     "null argument to denoise_step");
        const sana::SchedConfig sc = sched_of(config);
        SANA_REQUIRE(*n_history >= 0 && *n_history <= 2, "history holds at most two converted outputs");
        SANA_REQUIRE(*n_history == 0 || history, "history buffer missing");
        sana::Engine& eng = engine(ctx);
        const size_t numel = static_cast<size_t>(B) * eng.dims().Cl * H * W;
        sana::SchedulerHostState st;
        st.sigmas.assign(sigmas, sigmas + n_sigmas);
        st.step_index = *step_index;
        st.lower_order_count = *lower_order_count;
        for (int i = 0; i < *n_history; ++i) st.history.emplace_back(history + i * numel, history + (i + 1) * numel);
        eng.denoise_step(latents, B, H, W, context, L, bias, guidance, st, timestep, sc);
        *step_index = st.step_index;
        *lower_order_count = st.lower_order_count;
        *n_history = static_cast<int>(st.history.size());
        SANA_REQUIRE(history != nullptr, "history buffer missing");
        for (size_t i = 0; i < st.history.size(); ++i) std::memcpy(history + i * numel, st.history[i].data(), numel * 4);
    });
}

int sana_cuda_forward(sana_cuda_ctx* ctx, const float* latents, int S, int H, int W, float t, const float* context,
                      int L, const float* bias, float* noise_pred) {
    return guard(ctx, [&] {
        SANA_REQUIRE(latents && context && noise_pred, "null argument to forward");
        engine(ctx).forward_nocfg(latents, S, H, W, t, context, L, bias, noise_pred);
    });
}

int sana_cuda_block_forward(sana_cuda_ctx* ctx, int block, const float* x, int S, int T, const float* context, int L,
                            const float* tmod, const float* bias, float* after_self, float* after_cross,
                            float* after_ff) {
    return guard(ctx, [&] {
        SANA_REQUIRE(x && context && tmod, "null argument to block_forward");
        engine(ctx).block_forward(block, x, S, T, context, L, tmod, bias, after_self, after_cross, after_ff);
    });
}

int sana_cuda_run_model_blocks(sana_cuda_ctx* ctx, const float* x, int S, int T, const float* context, int L,
                               const float* tmod, const float* bias, int begin, int end, float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(x && context && tmod && out, "null argument to run_model_blocks");
        engine(ctx).run_blocks(x, S, T, context, L, tmod, bias, begin, end, out);
    });
}

int sana_cuda_project_caption(sana_cuda_ctx* ctx, const float* enc, int S, int L, int enc_dim, float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(enc && out, "null argument to project_caption");
        engine(ctx).project_caption(enc, S, L, enc_dim, out);
    });
}

int sana_cuda_profile_loop(sana_cuda_ctx* ctx, const float* latents, int B, int H, int W, const float* enc, int L,
                           int enc_dim, const float* bias, float guidance, int num_steps, float flow_shift, float* out,
                           char* report, size_t report_len) {
    return guard(ctx, [&] {
        SANA_REQUIRE(latents && enc && out && report && report_len > 0, "null argument to profile_loop");
        sana::Engine& eng = engine(ctx);
        eng.profile_loop_device(latents, B, H, W, enc, L, enc_dim, bias, guidance, num_steps,
                                default_sched(flow_shift), out);
        const std::string r = eng.profile_report();
        eng.profile_enable(false);
        std::snprintf(report, report_len, "%s", r.c_str());
    });
}

int sana_cuda_debug_read(sana_cuda_ctx* ctx, const char* name, size_t offset, size_t bytes, void* host,
                         size_t* size_out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(name != nullptr, "buffer name must not be null");
        const size_t n = engine(ctx).debug_read(name, offset, bytes, host);
        if (size_out) *size_out = n;
    });
}

// --- single operations -------------------------------------------------------------------

int sana_op_linear(sana_cuda_ctx* ctx, const float* x, int rows, int K, const float* w, const float* bias, int N,
                   float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(x && w && out && rows >= 0 && K >= 1 && N >= 1, "invalid linear arguments");
        sana::Engine& eng = engine(ctx);
        const bool bf = eng.mode() == sana::kModeBf16;
        ActBuf A, Bw;
        A.upload(x, static_cast<size_t>(rows) * K, bf);
        std::vector<float> wt = transpose(w, K, N);
        Bw.upload(wt.data(), wt.size(), bf);
        DevBuf bd = bias ? f32_upload(bias, N) : DevBuf();
        DevBuf o;
        o.ensure(std::max<size_t>(static_cast<size_t>(rows) * N, 1) * 4);
        run_gemm(eng, A, K, Bw, K, rows, N, K, epi(o.get(), false, N, bias ? bd.as<float>() : nullptr));
        finish(eng);
        if (rows) d2h(out, o.get(), static_cast<size_t>(rows) * N * 4);
    });
}

int sana_op_layer_norm(sana_cuda_ctx* ctx, const float* x, int rows, int C, float eps, const float* gamma,
                       const float* beta, float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(x && out && rows >= 0 && C >= 1, "invalid layer_norm arguments");
        sana::Engine& eng = engine(ctx);
        const size_t n = static_cast<size_t>(rows) * C;
        DevBuf xd = f32_upload(x, n), o, g, b;
        o.ensure(std::max<size_t>(n, 1) * 4);
        if (gamma) g = f32_upload(gamma, C);
        if (beta) b = f32_upload(beta, C);
        sana::ln_modulate<float>(xd.as<float>(), rows, C, std::max(rows, 1), g.as<float>(), b.as<float>(), nullptr, 0, 0,
                                 0, eps, o.as<float>(), eng.stream());
        finish(eng);
        if (n) d2h(out, o.get(), n * 4);
    });
}

int sana_op_rms_norm(sana_cuda_ctx* ctx, const float* x, int rows, int C, float eps, const float* weight, float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(x && out && rows >= 0 && C >= 1, "invalid rms_norm arguments");
        sana::Engine& eng = engine(ctx);
        const size_t n = static_cast<size_t>(rows) * C;
        DevBuf xd = f32_upload(x, n), o, w;
        o.ensure(std::max<size_t>(n, 1) * 4);
        if (weight) w = f32_upload(weight, C);
        sana::rms_norm<float>(xd.as<float>(), rows, C, eps, w.as<float>(), o.as<float>(), eng.stream());
        finish(eng);
        if (n) d2h(out, o.get(), n * 4);
    });
}

int sana_op_modulate(sana_cuda_ctx* ctx, const float* x, int B, int T, int C, const float* shift, const float* scale,
                     float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(x && shift && scale && out && B >= 1 && T >= 1 && C >= 1, "invalid modulate arguments");
        sana::Engine& eng = engine(ctx);
        const size_t n = static_cast<size_t>(B) * T * C;
        std::vector<float> mod(static_cast<size_t>(B) * 2 * C);
        for (int b = 0; b < B; ++b) {
            std::memcpy(&mod[static_cast<size_t>(b) * 2 * C], shift + static_cast<size_t>(b) * C, C * 4);
            std::memcpy(&mod[static_cast<size_t>(b) * 2 * C + C], scale + static_cast<size_t>(b) * C, C * 4);
        }
        DevBuf xd = f32_upload(x, n), md = f32_upload(mod.data(), mod.size()), o;
        o.ensure(n * 4);
        sana::modulate(xd.as<float>(), static_cast<long long>(B) * T, C, T, md.as<float>(), 2LL * C, 0, 1,
                       o.as<float>(), eng.stream());
        finish(eng);
        d2h(out, o.get(), n * 4);
    });
}

int sana_op_linear_attention(sana_cuda_ctx* ctx, const float* q, const float* k, const float* v, int B, int H, int Tq,
                             int Tk, int D, float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(q && k && v && out && B >= 1 && H >= 1 && Tq >= 1 && Tk >= 1 && D >= 1,
                     "invalid linear attention arguments");
        sana::Engine& eng = engine(ctx);
        const bool bf = eng.mode() == sana::kModeBf16;
        const int HD = H * D;
        std::vector<float> qt = heads_to_tokens(q, B, H, Tq, D);
        std::vector<float> kt = heads_to_tokens(k, B, H, Tk, D), vt = heads_to_tokens(v, B, H, Tk, D);
        std::vector<float> kv(static_cast<size_t>(B) * Tk * 2 * HD);
        for (size_t r = 0; r < static_cast<size_t>(B) * Tk; ++r) {
            std::memcpy(&kv[r * 2 * HD], &kt[r * HD], HD * 4);
            std::memcpy(&kv[r * 2 * HD + HD], &vt[r * HD], HD * 4);
        }
        ActBuf Q, KV, O;
        Q.upload(qt.data(), qt.size(), bf);
        KV.upload(kv.data(), kv.size(), bf);
        O.alloc(qt.size(), bf);
        DevBuf part;
        part.ensure(static_cast<size_t>(B) * H * (sana::linattn_chunks(Tk) + 1) * (D + 1) * D * 4);
        if (bf) {
            sana::linear_attention<bf16>(static_cast<const bf16*>(Q.get()), HD, 0, static_cast<const bf16*>(KV.get()),
                                         2LL * HD, 0, HD, B, Tq, Tk, H, D, part.as<float>(),
                                         static_cast<bf16*>(O.get()), HD, eng.stream());
        } else {
            sana::linear_attention<float>(static_cast<const float*>(Q.get()), HD, 0,
                                          static_cast<const float*>(KV.get()), 2LL * HD, 0, HD, B, Tq, Tk, H, D,
                                          part.as<float>(), static_cast<float*>(O.get()), HD, eng.stream());
        }
        finish(eng);
        std::vector<float> ot(qt.size());
        O.download(ot.data());
        tokens_to_heads(ot.data(), B, H, Tq, D, out);
    });
}

int sana_op_attention(sana_cuda_ctx* ctx, const float* q, const float* k, const float* v, int B, int H, int Tq,
                      int Tk, int D, const float* bias, float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(q && k && v && out && B >= 1 && H >= 1 && Tq >= 1 && Tk >= 1 && D >= 1,
                     "invalid attention arguments");
        sana::Engine& eng = engine(ctx);
        const bool bf = eng.mode() == sana::kModeBf16;
        const int HD = H * D;
        std::vector<float> qt = heads_to_tokens(q, B, H, Tq, D);
        std::vector<float> kt = heads_to_tokens(k, B, H, Tk, D), vt = heads_to_tokens(v, B, H, Tk, D);
        std::vector<float> kv(static_cast<size_t>(B) * Tk * 2 * HD);
        for (size_t r = 0; r < static_cast<size_t>(B) * Tk; ++r) {
            std::memcpy(&kv[r * 2 * HD], &kt[r * HD], HD * 4);
            std::memcpy(&kv[r * 2 * HD + HD], &vt[r * HD], HD * 4);
        }
        ActBuf Q, KV, O;
        Q.upload(qt.data(), qt.size(), bf);
        KV.upload(kv.data(), kv.size(), bf);
        O.alloc(qt.size(), bf);
        DevBuf bd, kl;
        if (bias) {
            bd = f32_upload(bias, static_cast<size_t>(B) * Tk);
            kl.ensure(static_cast<size_t>(B) * 4);
            sana::caption_kv_len(bd.as<float>(), B, Tk, kl.as<int>(), eng.stream());
        }
        const float scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(D)));
        if (bf) {
            sana::cross_attention<bf16>(static_cast<const bf16*>(Q.get()), HD, static_cast<const bf16*>(KV.get()),
                                        2LL * HD, 0, HD, bd.as<float>(), kl.as<int>(), B, Tq, Tk, H, D, scale,
                                        static_cast<bf16*>(O.get()), HD, eng.err(), eng.stream());
        } else {
            sana::cross_attention<float>(static_cast<const float*>(Q.get()), HD, static_cast<const float*>(KV.get()),
                                         2LL * HD, 0, HD, bd.as<float>(), kl.as<int>(), B, Tq, Tk, H, D, scale,
                                         static_cast<float*>(O.get()), HD, eng.err(), eng.stream());
        }
        finish(eng);
        std::vector<float> ot(qt.size());
        O.download(ot.data());
        tokens_to_heads(ot.data(), B, H, Tq, D, out);
    });
}

int sana_op_conv1x1(sana_cuda_ctx* ctx, const float* x, int B, int Cin, int H, int W, const float* w,
                    const float* bias, int Cout, float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(x && w && out && B >= 1 && Cin >= 1 && H >= 1 && W >= 1 && Cout >= 1, "invalid conv1x1 arguments");
        sana::Engine& eng = engine(ctx);
        const bool bf = eng.mode() == sana::kModeBf16;
        const int HW = H * W;
        std::vector<float> xt = nchw_to_tokens(x, B, Cin, HW);
        ActBuf A, Wt;
        A.upload(xt.data(), xt.size(), bf);
        Wt.upload(w, static_cast<size_t>(Cout) * Cin, bf);
        DevBuf bd = bias ? f32_upload(bias, Cout) : DevBuf(), o;
        o.ensure(static_cast<size_t>(B) * HW * Cout * 4);
        run_gemm(eng, A, Cin, Wt, Cin, B * HW, Cout, Cin, epi(o.get(), false, Cout, bd.as<float>()));
        finish(eng);
        std::vector<float> ot(static_cast<size_t>(B) * HW * Cout);
        d2h(ot.data(), o.get(), ot.size() * 4);
        tokens_to_nchw(ot.data(), B, Cout, HW, out);
    });
}

int sana_op_depthwise3x3(sana_cuda_ctx* ctx, const float* x, int B, int C, int H, int W, const float* w,
                         const float* bias, float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(x && w && out && B >= 1 && C >= 1 && H >= 1 && W >= 1, "invalid depthwise arguments");
        sana::Engine& eng = engine(ctx);
        const int HW = H * W;
        std::vector<float> xt = nchw_to_tokens(x, B, C, HW);
        DevBuf xd = f32_upload(xt.data(), xt.size()), wd = f32_upload(w, static_cast<size_t>(C) * 9), bd, o;
        if (bias) bd = f32_upload(bias, C);
        o.ensure(xt.size() * 4);
        sana::depthwise3x3(xd.as<float>(), B, H, W, C, wd.as<float>(), bd.as<float>(), o.as<float>(), eng.stream());
        finish(eng);
        std::vector<float> ot(xt.size());
        d2h(ot.data(), o.get(), ot.size() * 4);
        tokens_to_nchw(ot.data(), B, C, HW, out);
    });
}

int sana_op_glumb_conv(sana_cuda_ctx* ctx, const float* x, int B, int Cin, int H, int W, const float* w_inv,
                       const float* b_inv, int E, const float* w_dw, const float* b_dw, const float* w_pt, int Cout,
                       float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(x && w_inv && w_dw && w_pt && out && E >= 2 && E % 2 == 0, "invalid glumb_conv arguments");
        sana::Engine& eng = engine(ctx);
        const bool bf = eng.mode() == sana::kModeBf16;
        const int HW = H * W, M = B * HW;
        std::vector<float> xt = nchw_to_tokens(x, B, Cin, HW);
        ActBuf A, Wi, Wp, Hb, G;
        A.upload(xt.data(), xt.size(), bf);
        Wi.upload(w_inv, static_cast<size_t>(E) * Cin, bf);
        Wp.upload(w_pt, static_cast<size_t>(Cout) * (E / 2), bf);
        Hb.alloc(static_cast<size_t>(M) * E, bf);
        G.alloc(static_cast<size_t>(M) * (E / 2), bf);
        DevBuf bi, bd, wd = f32_upload(w_dw, static_cast<size_t>(E) * 9), o;
        if (b_inv) bi = f32_upload(b_inv, E);
        std::vector<float> zeros(E, 0.f);
        bd = f32_upload(b_dw ? b_dw : zeros.data(), E);
        o.ensure(static_cast<size_t>(M) * Cout * 4);
        run_gemm(eng, A, Cin, Wi, Cin, M, E, Cin, epi(Hb.get(), bf, E, bi.as<float>(), sana::kActSilu));
        if (bf) {
            sana::depthwise_glu<bf16>(static_cast<const bf16*>(Hb.get()), E, B, H, W, E, wd.as<float>(),
                                      bd.as<float>(), static_cast<bf16*>(G.get()), E / 2, eng.err(), eng.stream());
        } else {
            sana::depthwise_glu<float>(static_cast<const float*>(Hb.get()), E, B, H, W, E, wd.as<float>(),
                                       bd.as<float>(), static_cast<float*>(G.get()), E / 2, eng.err(), eng.stream());
        }
        run_gemm(eng, G, E / 2, Wp, E / 2, M, Cout, E / 2, epi(o.get(), false, Cout));
        finish(eng);
        std::vector<float> ot(static_cast<size_t>(M) * Cout);
        d2h(ot.data(), o.get(), ot.size() * 4);
        tokens_to_nchw(ot.data(), B, Cout, HW, out);
    });
}

int sana_op_project_caption(sana_cuda_ctx* ctx, const float* enc, int B, int L, int Din, const float* w1,
                            const float* b1, int C, const float* w2, const float* b2, const float* norm_w, float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(enc && w1 && w2 && norm_w && out && B >= 1 && L >= 1 && Din >= 1 && C >= 1,
                     "invalid project_caption arguments");
        sana::Engine& eng = engine(ctx);
        const bool bf = eng.mode() == sana::kModeBf16;
        const int M = B * L;
        ActBuf A, W1, W2, Hh;
        A.upload(enc, static_cast<size_t>(M) * Din, bf);
        std::vector<float> w1t = transpose(w1, Din, C), w2t = transpose(w2, C, C);
        W1.upload(w1t.data(), w1t.size(), bf);
        W2.upload(w2t.data(), w2t.size(), bf);
        Hh.alloc(static_cast<size_t>(M) * C, bf);
        DevBuf bd1, bd2, nd = f32_upload(norm_w, C), p, o;
        if (b1) bd1 = f32_upload(b1, C);
        if (b2) bd2 = f32_upload(b2, C);
        p.ensure(static_cast<size_t>(M) * C * 4);
        o.ensure(static_cast<size_t>(M) * C * 4);
        run_gemm(eng, A, Din, W1, Din, M, C, Din, epi(Hh.get(), bf, C, bd1.as<float>(), sana::kActGelu));
        run_gemm(eng, Hh, C, W2, C, M, C, C, epi(p.get(), false, C, bd2.as<float>()));
        sana::rms_norm<float>(p.as<float>(), M, C, 1e-5f, nd.as<float>(), o.as<float>(), eng.stream());
        finish(eng);
        d2h(out, o.get(), static_cast<size_t>(M) * C * 4);
    });
}

int sana_op_attention_block(sana_cuda_ctx* ctx, const float* x, int B, int T, int C, const float* wq, const float* bq,
                            const float* wk, const float* bk, const float* wv, const float* bv, const float* wo,
                            const float* bo, int heads, float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(x && wq && wk && wv && wo && out && B >= 1 && T >= 1 && C >= 1, "invalid attention_block arguments");
        SANA_REQUIRE(heads >= 1 && C % heads == 0, "hidden size must be divisible by num_heads");
        sana::Engine& eng = engine(ctx);
        const bool bf = eng.mode() == sana::kModeBf16;
        const int M = B * T, D = C / heads;
        std::vector<float> wqkv(static_cast<size_t>(3) * C * C), bqkv(3 * static_cast<size_t>(C), 0.f);
        const float* ws[3] = {wq, wk, wv};
        const float* bs[3] = {bq, bk, bv};
        for (int j = 0; j < 3; ++j) {
            std::vector<float> t = transpose(ws[j], C, C);
            std::memcpy(&wqkv[static_cast<size_t>(j) * C * C], t.data(), t.size() * 4);
            if (bs[j]) std::memcpy(&bqkv[static_cast<size_t>(j) * C], bs[j], C * 4);
        }
        std::vector<float> wot = transpose(wo, C, C);
        ActBuf X, Wqkv, Wo, QKV, AO;
        X.upload(x, static_cast<size_t>(M) * C, bf);
        Wqkv.upload(wqkv.data(), wqkv.size(), bf);
        Wo.upload(wot.data(), wot.size(), bf);
        QKV.alloc(static_cast<size_t>(M) * 3 * C, bf);
        AO.alloc(static_cast<size_t>(M) * C, bf);
        DevBuf bqd = f32_upload(bqkv.data(), bqkv.size()), bod, part, o;
        if (bo) bod = f32_upload(bo, C);
        part.ensure(static_cast<size_t>(B) * heads * (sana::linattn_chunks(T) + 1) * (D + 1) * D * 4);
        o.ensure(static_cast<size_t>(M) * C * 4);
        run_gemm(eng, X, C, Wqkv, C, M, 3 * C, C, epi(QKV.get(), bf, 3 * C, bqd.as<float>()));
        if (bf) {
            const bf16* qkv = static_cast<const bf16*>(QKV.get());
            sana::linear_attention<bf16>(qkv, 3LL * C, 0, qkv, 3LL * C, C, 2 * C, B, T, T, heads, D, part.as<float>(),
                                         static_cast<bf16*>(AO.get()), C, eng.stream());
        } else {
            const float* qkv = static_cast<const float*>(QKV.get());
            sana::linear_attention<float>(qkv, 3LL * C, 0, qkv, 3LL * C, C, 2 * C, B, T, T, heads, D,
                                          part.as<float>(), static_cast<float*>(AO.get()), C, eng.stream());
        }
        run_gemm(eng, AO, C, Wo, C, M, C, C, epi(o.get(), false, C, bod.as<float>()));
        finish(eng);
        d2h(out, o.get(), static_cast<size_t>(M) * C * 4);
    });
}

int sana_op_cross_attention_block(sana_cuda_ctx* ctx, const float* x, int B, int T, int C, const float* context,
                                  int L, const float* bias, const float* wq, const float* bq, const float* wk,
                                  const float* bk, const float* wv, const float* bv, const float* wo, const float* bo,
                                  int heads, float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(x && context && wq && wk && wv && wo && out && B >= 1 && T >= 1 && C >= 1 && L >= 1,
                     "invalid cross_attention_block arguments");
        SANA_REQUIRE(heads >= 1 && C % heads == 0, "hidden size must be divisible by num_heads");
        sana::Engine& eng = engine(ctx);
        const bool bf = eng.mode() == sana::kModeBf16;
        const int M = B * T, D = C / heads;
        std::vector<float> wkv(static_cast<size_t>(2) * C * C), bkv(2 * static_cast<size_t>(C), 0.f);
        {
            std::vector<float> tk = transpose(wk, C, C), tv = transpose(wv, C, C);
            std::memcpy(wkv.data(), tk.data(), tk.size() * 4);
            std::memcpy(wkv.data() + static_cast<size_t>(C) * C, tv.data(), tv.size() * 4);
            if (bk) std::memcpy(bkv.data(), bk, C * 4);
            if (bv) std::memcpy(bkv.data() + C, bv, C * 4);
        }
        std::vector<float> wqt = transpose(wq, C, C), wot = transpose(wo, C, C);
        ActBuf X, Cx, Wq, Wkv, Wo, Q, KV, AO;
        X.upload(x, static_cast<size_t>(M) * C, bf);
        Cx.upload(context, static_cast<size_t>(B) * L * C, bf);
        Wq.upload(wqt.data(), wqt.size(), bf);
        Wkv.upload(wkv.data(), wkv.size(), bf);
        Wo.upload(wot.data(), wot.size(), bf);
        Q.alloc(static_cast<size_t>(M) * C, bf);
        KV.alloc(static_cast<size_t>(B) * L * 2 * C, bf);
        AO.alloc(static_cast<size_t>(M) * C, bf);
        DevBuf bqd, bkvd = f32_upload(bkv.data(), bkv.size()), bod, bd, kl, o;
        if (bq) bqd = f32_upload(bq, C);
        if (bo) bod = f32_upload(bo, C);
        if (bias) {
            bd = f32_upload(bias, static_cast<size_t>(B) * L);
            kl.ensure(static_cast<size_t>(B) * 4);
            sana::caption_kv_len(bd.as<float>(), B, L, kl.as<int>(), eng.stream());
        }
        o.ensure(static_cast<size_t>(M) * C * 4);
        run_gemm(eng, X, C, Wq, C, M, C, C, epi(Q.get(), bf, C, bqd.as<float>()));
        run_gemm(eng, Cx, C, Wkv, C, B * L, 2 * C, C, epi(KV.get(), bf, 2 * C, bkvd.as<float>()));
        const float scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(D)));
        if (bf) {
            sana::cross_attention<bf16>(static_cast<const bf16*>(Q.get()), C, static_cast<const bf16*>(KV.get()), 2LL * C,
                                        0, C, bd.as<float>(), kl.as<int>(), B, T, L, heads, D, scale,
                                        static_cast<bf16*>(AO.get()), C, eng.err(), eng.stream());
        } else {
            sana::cross_attention<float>(static_cast<const float*>(Q.get()), C, static_cast<const float*>(KV.get()),
                                         2LL * C, 0, C, bd.as<float>(), kl.as<int>(), B, T, L, heads, D, scale,
                                         static_cast<float*>(AO.get()), C, eng.err(), eng.stream());
        }
        run_gemm(eng, AO, C, Wo, C, M, C, C, epi(o.get(), false, C, bod.as<float>()));
        finish(eng);
        d2h(out, o.get(), static_cast<size_t>(M) * C * 4);
    });
}

int sana_op_cfg(sana_cuda_ctx* ctx, const float* noise, int B, int Cl, int H, int W, float guidance, float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(noise && out && B >= 1 && Cl >= 1 && H >= 1 && W >= 1, "invalid cfg arguments");
        sana::Engine& eng = engine(ctx);
        const int HW = H * W;
        const size_t n = static_cast<size_t>(B) * Cl * HW;
        std::vector<float> rows = nchw_to_tokens(noise, 2 * B, Cl, HW);
        DevBuf nd = f32_upload(rows.data(), rows.size()), lat, h0, h1;
        lat.ensure(n * 4);
        h0.ensure(n * 4);
        h1.ensure(n * 4);
        SANA_CUDA(cudaMemsetAsync(lat.get(), 0, n * 4, eng.stream()));
        sana::SchedCoef k{};
        k.guidance = guidance;
        k.sigma_s = -1.0f;  // x0 = 0 - (-1) * guided = guided
        k.a = 0.0f;
        k.b = 1.0f;
        sana::cfg_scheduler_step(nd.as<float>(), B, Cl, HW, lat.as<float>(), h0.as<float>(), h1.as<float>(), k,
                                 eng.stream());
        finish(eng);
        d2h(out, lat.get(), n * 4);
    });
}

// --- the remaining transformer_ops.h / transformer.h pieces --------------------------------

int sana_op_split_heads(sana_cuda_ctx* ctx, const float* in, int B, int T, int hidden, int heads, float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(in && out && B >= 0 && T >= 0 && hidden >= 1, "invalid split_heads arguments");
        SANA_REQUIRE(heads >= 1, "num_heads must be greater than 0");
        SANA_REQUIRE(hidden % heads == 0, "hidden size must be divisible by num_heads");
        sana::Engine& eng = engine(ctx);
        const size_t n = static_cast<size_t>(B) * T * hidden;
        DevBuf a = f32_upload(in, n), o;
        o.ensure(std::max<size_t>(n, 1) * 4);
        sana::permute_heads(a.as<float>(), o.as<float>(), B, T, heads, hidden / heads, true, eng.stream());
        finish(eng);
        d2h(out, o.get(), n * 4);
    });
}

int sana_op_merge_heads(sana_cuda_ctx* ctx, const float* in, int B, int H, int T, int D, float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(in && out && B >= 0 && H >= 0 && T >= 0 && D >= 0, "invalid merge_heads arguments");
        sana::Engine& eng = engine(ctx);
        const size_t n = static_cast<size_t>(B) * H * T * D;
        DevBuf a = f32_upload(in, n), o;
        o.ensure(std::max<size_t>(n, 1) * 4);
        sana::permute_heads(a.as<float>(), o.as<float>(), B, T, H, D, false, eng.stream());
        finish(eng);
        d2h(out, o.get(), n * 4);
    });
}

namespace {
// Per (batch, head) products C_bh[M, N] = A_bh[M, K] . B_bh[N, K]^T on the handle's GEMM path
// (tensor cores in bf16 mode where the shape allows, CUDA cores otherwise), fp32 output.
void batched_gemm_nt(sana::Engine& eng, const ActBuf& A, const ActBuf& Bm, int batches, int M, int N, int K, float* C) {
    const size_t es = A.bf ? 2 : 4;
    for (int i = 0; i < batches; ++i) {
        sana::GemmProblem p;
        p.A = static_cast<const uint8_t*>(A.get()) + static_cast<size_t>(i) * M * K * es;
        p.a_bf16 = A.bf;
        p.lda = K;
        p.B = static_cast<const uint8_t*>(Bm.get()) + static_cast<size_t>(i) * N * K * es;
        p.b_bf16 = Bm.bf;
        p.ldb = K;
        p.M = M;
        p.N = N;
        p.K = K;
        p.ep = epi(C + static_cast<size_t>(i) * M * N, false, N);
        sana::gemm(p, eng.err(), eng.stream(), eng.num_sms());
    }
}
}  // namespace

int sana_op_attention_scores(sana_cuda_ctx* ctx, const float* q, const float* k, int B, int H, int Tq, int Tk, int D,
                             float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(q && k && out && B >= 1 && H >= 1 && Tq >= 1 && Tk >= 1 && D >= 1,
                     "invalid attention_scores arguments");
        sana::Engine& eng = engine(ctx);
        const bool bf = eng.mode() == sana::kModeBf16;
        ActBuf Q, K;
        Q.upload(q, static_cast<size_t>(B) * H * Tq * D, bf);
        K.upload(k, static_cast<size_t>(B) * H * Tk * D, bf);
        DevBuf o;
        o.ensure(static_cast<size_t>(B) * H * Tq * Tk * 4);
        batched_gemm_nt(eng, Q, K, B * H, Tq, Tk, D, o.as<float>());
        finish(eng);
        d2h(out, o.get(), static_cast<size_t>(B) * H * Tq * Tk * 4);
    });
}

int sana_op_softmax_lastdim(sana_cuda_ctx* ctx, const float* in, long long rows, int n, float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(in && out && rows >= 0 && n >= 1, "invalid softmax arguments");
        sana::Engine& eng = engine(ctx);
        const size_t count = static_cast<size_t>(rows) * n;
        DevBuf a = f32_upload(in, count), o;
        o.ensure(std::max<size_t>(count, 1) * 4);
        sana::softmax_rows(a.as<float>(), rows, n, o.as<float>(), eng.stream());
        finish(eng);
        d2h(out, o.get(), count * 4);
    });
}

int sana_op_attention_values(sana_cuda_ctx* ctx, const float* probs, const float* v, int B, int H, int Tq, int Tk,
                             int D, float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(probs && v && out && B >= 1 && H >= 1 && Tq >= 1 && Tk >= 1 && D >= 1,
                     "invalid attention_values arguments");
        sana::Engine& eng = engine(ctx);
        const bool bf = eng.mode() == sana::kModeBf16;
        const int BH = B * H;
        ActBuf P, Vt;
        P.upload(probs, static_cast<size_t>(BH) * Tq * Tk, bf);
        DevBuf vd = f32_upload(v, static_cast<size_t>(BH) * Tk * D);
        Vt.alloc(static_cast<size_t>(BH) * D * Tk, bf);  // per (b, h): v^T [D, Tk]
        for (int i = 0; i < BH; ++i) {
            const float* src = vd.as<float>() + static_cast<size_t>(i) * Tk * D;
            if (bf) {
                sana::repack<bf16>(src, Tk, D, true, static_cast<bf16*>(Vt.get()) + static_cast<size_t>(i) * D * Tk,
                                   eng.stream());
            } else {
                sana::repack<float>(src, Tk, D, true, static_cast<float*>(Vt.get()) + static_cast<size_t>(i) * D * Tk,
                                    eng.stream());
            }
        }
        DevBuf o;
        o.ensure(static_cast<size_t>(BH) * Tq * D * 4);
        batched_gemm_nt(eng, P, Vt, BH, Tq, D, Tk, o.as<float>());
        finish(eng);
        d2h(out, o.get(), static_cast<size_t>(BH) * Tq * D * 4);
    });
}

int sana_op_block_modulation(sana_cuda_ctx* ctx, const float* tmod, const float* table, int B, int C, float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(tmod && table && out && B >= 1 && C >= 1, "invalid block modulation arguments");
        sana::Engine& eng = engine(ctx);
        DevBuf t = f32_upload(tmod, static_cast<size_t>(B) * 6 * C), tb = f32_upload(table, static_cast<size_t>(6) * C),
               o;
        o.ensure(static_cast<size_t>(B) * 6 * C * 4);
        sana::block_modulation(t.as<float>(), B, C, tb.as<float>(), 1, o.as<float>(), eng.stream());
        finish(eng);
        d2h(out, o.get(), static_cast<size_t>(B) * 6 * C * 4);
    });
}


// --- device-pointer kernels (microbenchmarks) ---------------------------------------------

int sana_op_gemm_device(sana_cuda_ctx* ctx, const void* A, const void* B, int M, int N, int K, const float* bias,
                        int act, void* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(A && B && out && M >= 1 && N >= 1 && K >= 1, "invalid gemm arguments");
        sana::Engine& eng = engine(ctx);
        sana::GemmProblem p;
        p.A = A;
        p.lda = K;
        p.B = B;
        p.ldb = K;
        p.M = M;
        p.N = N;
        p.K = K;
        p.ep = epi(out, true, N, bias, act);
        sana::gemm(p, eng.err(), eng.stream(), eng.num_sms());
    });
}

int sana_op_gemm_f32out_device(sana_cuda_ctx* ctx, const void* A, const void* B, int M, int N, int K,
                               const float* bias, int act, float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(A && B && out && M >= 1 && N >= 1 && K >= 1, "invalid gemm arguments");
        sana::Engine& eng = engine(ctx);
        sana::GemmProblem p;
        p.A = A;
        p.lda = K;
        p.B = B;
        p.ldb = K;
        p.M = M;
        p.N = N;
        p.K = K;
        p.ep = epi(out, false, N, bias, act);
        sana::gemm(p, eng.err(), eng.stream(), eng.num_sms());
    });
}

int sana_op_gemm_residual_device(sana_cuda_ctx* ctx, const void* A, const void* B, int M, int N, int K,
                                 const float* bias, const float* resid, const float* gate, int rows_per_gate,
                                 float* out, void* out_bf16) {
    return guard(ctx, [&] {
        SANA_REQUIRE(A && B && resid && out && M >= 1 && N >= 1 && K >= 1, "invalid gemm arguments");
        SANA_REQUIRE(!gate || rows_per_gate >= 1, "rows_per_gate must be positive with a gate");
        sana::Engine& eng = engine(ctx);
        sana::GemmProblem p;
        p.A = A;
        p.lda = K;
        p.B = B;
        p.ldb = K;
        p.M = M;
        p.N = N;
        p.K = K;
        p.ep = epi(out, false, N, bias);
        p.ep.resid = resid;
        p.ep.ldr = N;
        p.ep.gate = gate;
        p.ep.gate_ld = N;
        p.ep.rows_per_gate = gate ? rows_per_gate : 1;
        p.ep.out2 = out_bf16;
        p.ep.out2_bf16 = 1;
        p.ep.ldo2 = N;
        sana::gemm(p, eng.err(), eng.stream(), eng.num_sms());
    });
}

int sana_op_linear_attention_device(sana_cuda_ctx* ctx, const void* qkv, int S, int T, int heads, int D,
                                    float* partial, void* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(qkv && partial && out && S >= 1 && T >= 1 && heads >= 1 && D >= 1, "invalid arguments");
        sana::Engine& eng = engine(ctx);
        const int C = heads * D;
        const bf16* q = static_cast<const bf16*>(qkv);
        sana::linear_attention<bf16>(q, 3LL * C, 0, q, 3LL * C, C, 2 * C, S, T, T, heads, D, partial,
                                     static_cast<bf16*>(out), C, eng.stream());
    });
}

size_t sana_op_linear_attention_workspace(int S, int T, int heads, int D) {
    return static_cast<size_t>(S) * heads * (sana::linattn_chunks(T) + 1) * (D + 1) * D * sizeof(float);
}

int sana_op_linear_attention_noalloc(sana_cuda_ctx* ctx, const void* qkv, int S, int T, int heads, int D,
                                     void* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(qkv && out && S >= 1 && T >= 1 && heads >= 1 && D >= 1 && D <= 128, "invalid arguments");
        // in double: the product of the four factors can overflow size_t for absurd inputs
        const double need = static_cast<double>(S) * heads * (sana::linattn_chunks(T) + 1) * (D + 1) * D * 4.0;
        if (need > static_cast<double>(SANA_NOALLOC_SCRATCH_BYTES))
            throw sana::InvalidArg("linear attention scratch of " + std::to_string(static_cast<long long>(need)) +
                                   " bytes exceeds the fixed " + std::to_string(SANA_NOALLOC_SCRATCH_BYTES) +
                                   "-byte scratch of sana_op_linear_attention_noalloc; pass a workspace to "
                                   "sana_op_linear_attention_device instead");
        sana::Engine& eng = engine(ctx);
        CurrentDevice on(eng.device());
        float* scratch = linattn_scratch(eng.device());
        const int C = heads * D;
        const bf16* q = static_cast<const bf16*>(qkv);
        sana::linear_attention<bf16>(q, 3LL * C, 0, q, 3LL * C, C, 2 * C, S, T, T, heads, D, scratch,
                                     static_cast<bf16*>(out), C, eng.stream());
    });
}

int sana_op_depthwise_glu_device(sana_cuda_ctx* ctx, const void* in, int S, int H, int W, int E, const float* w,
                                 const float* b, void* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(in && w && b && out && S >= 1 && H >= 1 && W >= 1 && E >= 2, "invalid arguments");
        sana::Engine& eng = engine(ctx);
        sana::depthwise_glu<bf16>(static_cast<const bf16*>(in), E, S, H, W, E, w, b, static_cast<bf16*>(out), E / 2,
                                  eng.err(), eng.stream());
    });
}

int sana_op_ln_modulate_device(sana_cuda_ctx* ctx, const float* x, long long rows, int C, int rows_per_seq,
                               const float* mod, long long mod_ld, int shift_idx, int scale_idx, float eps,
                               void* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(x && out && rows >= 0 && C >= 1 && rows_per_seq >= 1 && eps >= 0.f, "invalid arguments");
        SANA_REQUIRE(!mod || (shift_idx >= 0 && scale_idx >= 0 && mod_ld >= C), "invalid modulation layout");
        sana::Engine& eng = engine(ctx);
        sana::ln_modulate<bf16>(x, rows, C, rows_per_seq, nullptr, nullptr, mod, mod_ld, shift_idx, scale_idx, eps,
                                static_cast<bf16*>(out), eng.stream());
    });
}

int sana_op_cross_attention_device(sana_cuda_ctx* ctx, const void* q, const void* kv, const float* bias,
                                   int* kv_len, int S, int T, int L, int heads, int D, void* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(q && kv && out && S >= 1 && T >= 1 && L >= 1 && heads >= 1 && D >= 1, "invalid arguments");
        sana::Engine& eng = engine(ctx);
        const int C = heads * D;
        if (bias && kv_len) sana::caption_kv_len(bias, S, L, kv_len, eng.stream());
        const float scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(D)));
        sana::cross_attention<bf16>(static_cast<const bf16*>(q), C, static_cast<const bf16*>(kv), 2LL * C, 0, C, bias,
                                    bias ? kv_len : nullptr, S, T, L, heads, D, scale, static_cast<bf16*>(out), C,
                                    eng.err(), eng.stream());
    });
}

// --- scheduler -------------------------------------------------------------------------------

void sana_scheduler_config_default(sana_scheduler_config* c) {
    if (!c) return;
    const sana::SchedConfig d;
    c->num_train_timesteps = d.num_train_timesteps;
    c->flow_shift = d.flow_shift;
    c->use_flow_sigmas = d.flow_sigmas ? 1 : 0;
    c->solver_order = d.solver_order;
    c->lower_order_final = d.lower_order_final ? 1 : 0;
    c->final_sigmas_zero = d.final_sigmas_zero ? 1 : 0;
    c->solver_heun = d.heun ? 1 : 0;
}

int sana_scheduler_schedule_config(const sana_scheduler_config* config, int n, float* timesteps, float* sigmas) {
    if (!timesteps || !sigmas) return SANA_ERR_INVALID;
    try {
        std::vector<float> ts, sg;
        sana::scheduler_schedule(n, sched_of(config), ts, sg);
        std::memcpy(timesteps, ts.data(), ts.size() * 4);
        std::memcpy(sigmas, sg.data(), sg.size() * 4);
        return SANA_OK;
    } catch (...) {
        return SANA_ERR_INVALID;
    }
}

int sana_scheduler_schedule(int n, float flow_shift, float* timesteps, float* sigmas) {
    sana_scheduler_config c;
    sana_scheduler_config_default(&c);
    c.flow_shift = flow_shift;
    return sana_scheduler_schedule_config(&c, n, timesteps, sigmas);
}

int sana_scheduler_convert(sana_cuda_ctx* ctx, const float* sigmas, int n_sigmas, int step_index,
                           const float* model_output, const float* sample, int numel, float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(sigmas && model_output && sample && out && numel >= 1, "invalid convert arguments");
        SANA_REQUIRE(n_sigmas >= 2 && step_index >= 0 && step_index < n_sigmas - 1,
                     "scheduler step_index is out of range");
        sana::Engine& eng = engine(ctx);
        std::vector<float> rows(2 * static_cast<size_t>(numel));
        std::memcpy(rows.data(), model_output, numel * 4);
        std::memcpy(rows.data() + numel, model_output, numel * 4);
        DevBuf nd = f32_upload(rows.data(), rows.size()), lat = f32_upload(sample, numel), h0, h1;
        h0.ensure(numel * 4);
        h1.ensure(numel * 4);
        sana::SchedCoef k{};
        k.guidance = 1.0f;
        k.sigma_s = sigmas[step_index];
        sana::cfg_scheduler_step(nd.as<float>(), 1, 1, numel, lat.as<float>(), h0.as<float>(), h1.as<float>(), k,
                                 eng.stream());
        finish(eng);
        d2h(out, h0.get(), numel * 4);
    });
}

int sana_scheduler_update(sana_cuda_ctx* ctx, int order, const float* sigmas, int n_sigmas, int step_index,
                          const float* m0, const float* m1, const float* sample, int numel, float* out) {
    return sana_scheduler_update_config(ctx, nullptr, order, sigmas, n_sigmas, step_index, m0, m1, sample, numel,
                                        out);
}

int sana_scheduler_update_config(sana_cuda_ctx* ctx, const sana_scheduler_config* config, int order,
                                 const float* sigmas, int n_sigmas, int step_index, const float* m0, const float* m1,
                                 const float* sample, int numel, float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(sigmas && m0 && sample && out && numel >= 1, "invalid update arguments");
        SANA_REQUIRE(order == 1 || order == 2, "order must be 1 or 2");
        SANA_REQUIRE(order == 1 || m1, "second-order update requires two model outputs");
        const sana::SchedConfig sc = sched_of(config);
        sana::Engine& eng = engine(ctx);
        std::vector<float> sg(sigmas, sigmas + n_sigmas);
        const sana::SchedCoef k = sana::scheduler_coefficients_order(sg, step_index, order, 1.0f, sc);
        DevBuf a = f32_upload(m0, numel), b = f32_upload(m1 ? m1 : m0, numel), x = f32_upload(sample, numel), o;
        o.ensure(numel * 4);
        sana::scheduler_update(a.as<float>(), b.as<float>(), x.as<float>(), numel, k, o.as<float>(), eng.stream());
        finish(eng);
        d2h(out, o.get(), numel * 4);
    });
}

int sana_scheduler_step(sana_cuda_ctx* ctx, const float* sigmas, int n_sigmas, int* step_index,
                        int* lower_order_count, float* history, int* n_history, const float* model_output,
                        const float* sample, int numel, float* out) {
    return sana_scheduler_step_config(ctx, nullptr, sigmas, n_sigmas, step_index, lower_order_count, history,
                                      n_history, model_output, sample, numel, out);
}

int sana_scheduler_step_config(sana_cuda_ctx* ctx, const sana_scheduler_config* config, const float* sigmas,
                               int n_sigmas, int* step_index, int* lower_order_count, float* history, int* n_history,
                               const float* model_output, const float* sample, int numel, float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(sigmas && step_index && lower_order_count && n_history && model_output && sample && out &&
                         numel >= 1,
                     "invalid step arguments");
        SANA_REQUIRE(*n_history >= 0 && *n_history <= 2 && (*n_history == 0 || history), "invalid history");
        SANA_REQUIRE(history != nullptr, "history buffer (2 x numel) required");
        const sana::SchedConfig sc = sched_of(config);
        sana::Engine& eng = engine(ctx);
        std::vector<float> sg(sigmas, sigmas + n_sigmas);
        const sana::SchedCoef k = sana::scheduler_coefficients(sg, *step_index, *lower_order_count, 1.0f, sc);
        // the history after this step's push, capped at solver_order (step_sana_scheduler,
        // scheduler.cpp:286-289), must hold two outputs for the second-order update
        const int kept = std::min(*n_history + 1, sc.solver_order);
        if (k.second_order) {
            SANA_REQUIRE(kept >= 2, "second-order update requires two model outputs");
        }
        std::vector<float> rows(2 * static_cast<size_t>(numel));
        std::memcpy(rows.data(), model_output, numel * 4);
        std::memcpy(rows.data() + numel, model_output, numel * 4);
        DevBuf nd = f32_upload(rows.data(), rows.size()), lat = f32_upload(sample, numel), h0, h1;
        h0.ensure(numel * 4);
        if (*n_history >= 1) h1 = f32_upload(history + static_cast<size_t>(*n_history - 1) * numel, numel);
        else h1.ensure(numel * 4);
        sana::cfg_scheduler_step(nd.as<float>(), 1, 1, numel, lat.as<float>(), h0.as<float>(), h1.as<float>(), k,
                                 eng.stream());
        finish(eng);
        d2h(out, lat.get(), numel * 4);
        std::vector<float> conv(numel);
        d2h(conv.data(), h0.get(), numel * 4);
        // push, then keep the newest `kept` outputs, oldest first
        const int drop = *n_history + 1 - kept;
        if (drop > 0 && *n_history > drop)
            std::memmove(history, history + static_cast<size_t>(drop) * numel,
                         static_cast<size_t>(*n_history - drop) * numel * 4);
        std::memcpy(history + static_cast<size_t>(kept - 1) * numel, conv.data(), numel * 4);
        *n_history = kept;
        if (*lower_order_count < sc.solver_order) ++*lower_order_count;
        ++*step_index;
    });
}

// --- synthetic inputs ---------------------------------------------------------------------

// torch.randn on a CPU generator for n >= 16 (the algorithm restated by torch_rng.cpp:9-68):
// MT19937 draws, uniforms u = (draw & (2^24 - 1)) / 2^24, Box-Muller on complete blocks of
// 16 (radius from the first 8, angle from the last 8), and a final re-drawn block of 16
// over the last 16 elements when n is not a multiple of 16.
int sana_randn_torch_cpu(float* out, size_t n, uint64_t seed) {
    if (!out || n < 16) return SANA_ERR_INVALID;
    std::mt19937 gen(static_cast<std::mt19937::result_type>(seed & 0xffffffffULL));
    auto uniform = [&gen]() { return static_cast<float>(gen() & 0xffffffu) * (1.0f / 16777216.0f); };
    auto block16 = [](float* d) {
        const double two_pi = 2.0 * 3.14159265358979323846;
        for (int j = 0; j < 8; ++j) {
            const float radius = std::sqrt(-2.0f * std::log(1.0f - d[j]));
            const float angle = static_cast<float>(two_pi * static_cast<double>(d[j + 8]));
            d[j] = radius * std::cos(angle);
            d[j + 8] = radius * std::sin(angle);
        }
    };
    for (size_t i = 0; i < n; ++i) out[i] = uniform();
    for (size_t i = 0; i + 16 <= n; i += 16) block16(out + i);
    if (n % 16 != 0) {
        float* tail = out + n - 16;
        for (int j = 0; j < 16; ++j) tail[j] = uniform();
        block16(tail);
    }
    return SANA_OK;
}

/* --- the text-encoder output contract (gemma_encoder.cpp:51-77,177-244) ---------------- */

namespace {

void write_err(char* err, size_t err_len, const char* msg) {
    if (err && err_len) std::snprintf(err, err_len, "%s", msg);
}

// Real tokens the positive branch keeps after the row-0 + tail slice: row 0 when the branch
// has any real token, plus every kept tail row below the real count (gemma_encoder.cpp:205-215).
size_t kept_real_tokens(size_t positive_rows, size_t positive_real, size_t L) {
    size_t kept = positive_real > 0 ? 1 : 0;
    for (size_t pos = positive_rows - (L - 1); pos < positive_rows; ++pos)
        if (pos < positive_real) ++kept;
    return kept;
}

void check_prompt_pair(size_t negative_rows, size_t negative_real, size_t positive_rows, size_t positive_real,
                       size_t hidden, size_t L) {
    if (L == 0 || hidden == 0) throw std::invalid_argument("max_sequence_length and hidden must be positive");
    if (negative_rows != L) throw std::invalid_argument("negative branch must be padded to max_sequence_length");
    if (negative_real > negative_rows || positive_real > positive_rows)
        throw std::invalid_argument("tokenized text exceeds padded_length; truncation not implemented");
    if (L > positive_rows) throw std::invalid_argument("select_rows_first_and_last: keep must be in (0, rows]");
}

void attention_bias_row(float* row, size_t real, size_t L) {
    for (size_t t = 0; t < L; ++t) {
        const float mask = t < real ? 1.0f : 0.0f;
        row[t] = (1.0f - mask) * -10000.0f;
    }
}

}  // namespace

int sana_select_rows_first_and_last(const float* in, size_t rows, size_t cols, size_t keep, float* out, char* err,
                                    size_t err_len) {
    if (!in || !out) return SANA_ERR_INVALID;
    if (keep == 0 || keep > rows) {
        write_err(err, err_len, "select_rows_first_and_last: keep must be in (0, rows]");
        return SANA_ERR_INVALID;
    }
    std::memcpy(out, in, cols * sizeof(float));
    std::memcpy(out + cols, in + (rows - (keep - 1)) * cols, (keep - 1) * cols * sizeof(float));
    return SANA_OK;
}

int sana_prompt_pair_assemble(const float* negative, size_t negative_rows, size_t negative_real,
                              const float* positive, size_t positive_rows, size_t positive_real, size_t hidden,
                              size_t max_sequence_length, float* embeddings, float* bias, char* err,
                              size_t err_len) {
    if (!negative || !positive || !embeddings || !bias) return SANA_ERR_INVALID;
    const size_t L = max_sequence_length;
    try {
        check_prompt_pair(negative_rows, negative_real, positive_rows, positive_real, hidden, L);
    } catch (const std::invalid_argument& e) {
        write_err(err, err_len, e.what());
        return SANA_ERR_INVALID;
    }
    std::memcpy(embeddings, negative, L * hidden * sizeof(float));
    sana_select_rows_first_and_last(positive, positive_rows, hidden, L, embeddings + L * hidden, nullptr, 0);
    attention_bias_row(bias, negative_real, L);
    attention_bias_row(bias + L, kept_real_tokens(positive_rows, positive_real, L), L);
    return SANA_OK;
}

int sana_cuda_prompt_pairs_device(sana_cuda_ctx* ctx, int pairs, const float* negative, const int* negative_real,
                                  const float* positive, int positive_rows, const int* positive_real, int hidden,
                                  int L, float* enc, float* bias) {
    return guard(ctx, [&] {
        SANA_REQUIRE(negative && positive && negative_real && positive_real && enc && bias, "invalid arguments");
        SANA_REQUIRE(pairs >= 1 && pairs <= sana::kMaxPromptPairs, "prompt pair count must be in [1, 64]");
        SANA_REQUIRE(positive_rows >= 0 && hidden >= 0 && L >= 0, "invalid arguments");
        sana::PromptPairCounts counts{};
        for (int p = 0; p < pairs; ++p) {
            SANA_REQUIRE(negative_real[p] >= 0 && positive_real[p] >= 0, "invalid arguments");
            check_prompt_pair(static_cast<size_t>(L), static_cast<size_t>(negative_real[p]),
                              static_cast<size_t>(positive_rows), static_cast<size_t>(positive_real[p]),
                              static_cast<size_t>(hidden), static_cast<size_t>(L));
            counts.real[p] = negative_real[p];
            counts.real[pairs + p] = static_cast<int>(
                kept_real_tokens(static_cast<size_t>(positive_rows), static_cast<size_t>(positive_real[p]),
                                 static_cast<size_t>(L)));
        }
        sana::Engine& eng = engine(ctx);
        sana::prompt_pairs(negative, positive, pairs, positive_rows, hidden, L, counts, enc, bias, eng.stream());
    });
}

/* --- the VAE decoder (vae.h, vae.cpp:243-325) ------------------------------------------- */

namespace {

sana::VaeDecoder& vae_of(sana_cuda_ctx* ctx) {
    sana::Engine& eng = engine(ctx);
    if (!ctx->vae) ctx->vae = std::make_unique<sana::VaeDecoder>(eng);
    return *ctx->vae;
}

sana::VaeDims vae_dims_from(const sana_vae_dims* d) {
    sana::VaeDims v;
    v.latent_channels = d->latent_channels;
    v.out_channels = d->out_channels;
    v.n_blocks = d->n_blocks;
    v.head_dim = d->head_dim;
    v.ms_kernel = d->ms_kernel;
    v.scaling_factor = d->scaling_factor;
    SANA_REQUIRE(d->n_blocks >= 1 && d->n_blocks <= 8, "vae decoder must contain at least one up block");
    for (int i = 0; i < d->n_blocks; ++i) {
        v.blocks[i].channels = d->blocks[i].channels;
        v.blocks[i].has_upsample = d->blocks[i].has_upsample;
        v.blocks[i].is_res_block = d->blocks[i].is_res_block;
        v.blocks[i].layers = d->blocks[i].layers;
    }
    return v;
}

}  // namespace

int sana_cuda_vae_upload(sana_cuda_ctx* ctx, const sana_vae_dims* dims, const float* const* tensors) {
    return guard(ctx, [&] {
        SANA_REQUIRE(dims && tensors, "invalid arguments");
        vae_of(ctx).upload(vae_dims_from(dims), tensors);
    });
}

namespace {

// Up block prefixes "decoder.up_blocks.<n>" of the file in numeric order
// (find_vae_decoder_up_block_prefixes, vae.cpp:103-145).
std::vector<std::string> vae_block_prefixes(const sana::GgufFile& f) {
    static const std::string head = "decoder.up_blocks.";
    std::set<std::pair<size_t, std::string>> ordered;
    for (const sana::GgufTensor& t : f.tensors()) {
        if (t.name.compare(0, head.size(), head) != 0) continue;
        const size_t dot = t.name.find('.', head.size());
        if (dot == std::string::npos || dot == head.size()) continue;
        const std::string num = t.name.substr(head.size(), dot - head.size());
        if (num.find_first_not_of("0123456789") != std::string::npos) continue;
        ordered.insert({static_cast<size_t>(std::stoull(num)), head + num});
    }
    std::vector<std::string> v;
    for (const auto& e : ordered) v.push_back(e.second);
    return v;
}

}  // namespace

int sana_cuda_vae_upload_gguf(sana_cuda_ctx* ctx, const char* path, float scaling_factor, sana_vae_dims* dims_out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(path, "invalid arguments");
        const sana::GgufFile f(path);
        std::vector<int64_t> sh;
        std::vector<const float*> table;
        auto take = [&](const std::string& name, const std::vector<int64_t>& want) {
            table.push_back(tensor_f32(f, name, want.size(), &sh));
            require_shape(name, sh, want);
        };
        auto shape_of = [&](const std::string& name, size_t rank) {
            tensor_f32(f, name, rank, &sh);
            return sh;
        };
        const std::vector<std::string> prefixes = vae_block_prefixes(f);
        if (prefixes.empty()) throw std::invalid_argument("vae decoder must contain at least one up block");
        if (prefixes.size() > 8) throw std::invalid_argument("vae decoder has more than 8 up blocks");
        // load_vae_up_block_weights (vae.cpp:64-99): an upsample conv at layer 0 when present,
        // ResBlocks only after one, three layers
        sana::VaeDims d;
        d.n_blocks = static_cast<int>(prefixes.size());
        d.head_dim = 32;
        d.ms_kernel = 5;
        d.scaling_factor = scaling_factor;
        std::vector<int> base(prefixes.size());
        for (size_t i = 0; i < prefixes.size(); ++i) {
            const std::string& pre = prefixes[i];
            sana::VaeBlockDims& b = d.blocks[i];
            b.has_upsample = f.find(pre + ".0.conv.weight") ? 1 : 0;
            base[i] = b.has_upsample;
            b.is_res_block = (b.has_upsample && f.find(pre + "." + std::to_string(base[i]) + ".conv1.weight")) ? 1 : 0;
            b.layers = 3;
            const std::string l0 = pre + "." + std::to_string(base[i]);
            b.channels = static_cast<int>(
                b.has_upsample ? shape_of(pre + ".0.conv.weight", 4)[0]
                               : (b.is_res_block ? shape_of(l0 + ".conv1.weight", 4)[0] : shape_of(l0 + ".attn.to_q.weight", 2)[0]));
            if (!b.is_res_block) d.ms_kernel = static_cast<int>(shape_of(l0 + ".attn.to_qkv_multiscale.0.proj_in.weight", 4)[2]);
        }
        const std::vector<int64_t> cin = shape_of("decoder.conv_in.weight", 4);
        const std::vector<int64_t> cout = shape_of("decoder.conv_out.weight", 4);
        d.latent_channels = static_cast<int>(cin[1]);
        d.out_channels = static_cast<int>(cout[0]);
        const int64_t n = d.n_blocks, Cn = d.blocks[n - 1].channels, C0 = d.blocks[0].channels;
        const int64_t k = d.ms_kernel;
        take("decoder.conv_in.weight", {Cn, cin[1], 3, 3});
        take("decoder.conv_in.bias", {Cn});
        take("decoder.norm_out.weight", {C0});
        take("decoder.norm_out.bias", {C0});
        take("decoder.conv_out.weight", {cout[0], C0, 3, 3});
        take("decoder.conv_out.bias", {cout[0]});
        for (int64_t i = 0; i < n; ++i) {
            const sana::VaeBlockDims& b = d.blocks[i];
            const std::string& pre = prefixes[static_cast<size_t>(i)];
            const int64_t C = b.channels;
            if (b.has_upsample) {
                if (i + 1 >= n) throw std::invalid_argument("the innermost vae up block has no upsample");
                take(pre + ".0.conv.weight", {C, d.blocks[i + 1].channels, 3, 3});
                take(pre + ".0.conv.bias", {C});
            }
            for (int l = 0; l < b.layers; ++l) {
                const std::string lp = pre + "." + std::to_string(base[static_cast<size_t>(i)] + l);
                if (b.is_res_block) {
                    take(lp + ".conv1.weight", {C, C, 3, 3});
                    take(lp + ".conv1.bias", {C});
                    take(lp + ".conv2.weight", {C, C, 3, 3});
                    take(lp + ".norm.weight", {C});
                    take(lp + ".norm.bias", {C});
                } else {
                    take(lp + ".attn.to_q.weight", {C, C});
                    take(lp + ".attn.to_k.weight", {C, C});
                    take(lp + ".attn.to_v.weight", {C, C});
                    take(lp + ".attn.to_qkv_multiscale.0.proj_in.weight", {3 * C, 1, k, k});
                    take(lp + ".attn.to_qkv_multiscale.0.proj_out.weight", {3 * C, 32, 1, 1});
                    take(lp + ".attn.to_out.weight", {C, 2 * C});
                    take(lp + ".attn.norm_out.weight", {C});
                    take(lp + ".attn.norm_out.bias", {C});
                    take(lp + ".conv_out.conv_inverted.weight", {8 * C, C, 1, 1});
                    take(lp + ".conv_out.conv_inverted.bias", {8 * C});
                    take(lp + ".conv_out.conv_depth.weight", {8 * C, 1, 3, 3});
                    take(lp + ".conv_out.conv_depth.bias", {8 * C});
                    take(lp + ".conv_out.conv_point.weight", {C, 4 * C, 1, 1});
                    take(lp + ".conv_out.norm.weight", {C});
                    take(lp + ".conv_out.norm.bias", {C});
                }
            }
        }
        vae_of(ctx).upload(d, table.data());
        if (dims_out) {
            dims_out->latent_channels = d.latent_channels;
            dims_out->out_channels = d.out_channels;
            dims_out->n_blocks = d.n_blocks;
            dims_out->head_dim = d.head_dim;
            dims_out->ms_kernel = d.ms_kernel;
            dims_out->scaling_factor = d.scaling_factor;
            for (int i = 0; i < d.n_blocks; ++i)
                dims_out->blocks[i] = {d.blocks[i].channels, d.blocks[i].has_upsample, d.blocks[i].is_res_block,
                                       d.blocks[i].layers};
        }
    });
}

int sana_cuda_vae_decode(sana_cuda_ctx* ctx, const float* latents, int B, int h, int w, float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(latents && out, "invalid arguments");
        vae_of(ctx).decode_host(latents, B, h, w, out);
    });
}

int sana_cuda_vae_decode_device(sana_cuda_ctx* ctx, const float* latents, int B, int h, int w, float* out) {
    return guard(ctx, [&] {
        SANA_REQUIRE(latents && out, "invalid arguments");
        vae_of(ctx).decode(latents, B, h, w, out);
    });
}

int sana_cuda_vae_last_launch_count(const sana_cuda_ctx* ctx) {
    return (ctx && ctx->vae) ? ctx->vae->last_launches() : 0;
}

}  // extern "C"
