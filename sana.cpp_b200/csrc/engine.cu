// Denoiser engine: weight cache, workspace, block / step / loop orchestration and
// CUDA-graph capture of the whole denoising loop. See engine.h.
#include "engine.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <sstream>
#include <type_traits>

namespace sana {

// ---------------------------------------------------------------------------------------
// DevBuf
// ---------------------------------------------------------------------------------------
void DevBuf::ensure(size_t bytes) {
    if (bytes <= n_ && p_) return;
    release();
    if (bytes == 0) return;
    cudaError_t e = cudaMalloc(&p_, bytes);
    if (e != cudaSuccess) {
        p_ = nullptr;
        throw CudaError(std::string("cudaMalloc(") + std::to_string(bytes) + "): " + cudaGetErrorString(e));
    }
    n_ = bytes;
}

void DevBuf::release() {
    if (p_) cudaFree(p_);
    p_ = nullptr;
    n_ = 0;
}

// ---------------------------------------------------------------------------------------
// Host-side scheduler and timestep arithmetic (the reference's fp32 expressions)
// ---------------------------------------------------------------------------------------
void scheduler_validate(const SchedConfig& c) {
    SANA_REQUIRE(c.solver_order >= 1, "solver_order must be positive");
    SANA_REQUIRE(c.solver_order <= 2, "only solver_order <= 2 is supported");
}

void scheduler_schedule(int n, const SchedConfig& c, std::vector<float>& timesteps, std::vector<float>& sigmas) {
    scheduler_validate(c);
    SANA_REQUIRE(n > 0, "num_inference_steps must be positive");
    SANA_REQUIRE(c.flow_sigmas, "only use_flow_sigmas=true is supported");
    SANA_REQUIRE(c.final_sigmas_zero, "only zero final_sigmas_type is supported");
    SANA_REQUIRE(c.num_train_timesteps > 0, "num_train_timesteps must be positive");
    const float denom = static_cast<float>(c.num_train_timesteps);
    const float flow_shift = c.flow_shift;
    std::vector<float> shifted(static_cast<size_t>(n) + 1);
    // alpha = 1 + (1/denom - 1) * i/n; sigma = 1 - alpha; shifted = shift*sigma / (1 + (shift-1)*sigma)
    // (scheduler.cpp:124-131). The reference as compiled (g++ -O3 with FMA available)
    // fuses the two multiply-adds; writing them as fma keeps the schedule bit-identical to
    // it whatever this file is compiled with.
    for (int i = 0; i <= n; ++i) {
        const float alpha = std::fma(1.0f / denom - 1.0f, static_cast<float>(i) / static_cast<float>(n), 1.0f);
        const float sigma = 1.0f - alpha;
        shifted[i] = flow_shift * sigma / std::fma(flow_shift - 1.0f, sigma, 1.0f);
    }
    timesteps.clear();
    sigmas.clear();
    for (int i = 0; i < n; ++i) {
        const float s = shifted[n - i];
        sigmas.push_back(s);
        timesteps.push_back(static_cast<float>(static_cast<int>(s * denom)));
    }
    sigmas.push_back(0.0f);
}

void scheduler_schedule(int n, float flow_shift, std::vector<float>& timesteps, std::vector<float>& sigmas) {
    SchedConfig c;
    c.flow_shift = flow_shift;
    scheduler_schedule(n, c, timesteps, sigmas);
}

// sigma_to_alpha_sigma_t (scheduler.cpp:71-77): flow sigmas give (1 - sigma, sigma), the
// variance-preserving form (1 / sqrt(sigma^2 + 1), sigma / sqrt(sigma^2 + 1)); the square
// term is a fused multiply-add as in the reference build.
static void alpha_sigma(float sigma, const SchedConfig& c, float& alpha, float& sig) {
    if (c.flow_sigmas) {
        alpha = 1.0f - sigma;
        sig = sigma;
    } else {
        alpha = 1.0f / std::sqrt(std::fma(sigma, sigma, 1.0f));
        sig = sigma * alpha;
    }
}

// compute_lambda (scheduler.cpp:79-81).
static float lambda_of(float alpha, float sigma) { return std::log(alpha) - std::log(sigma); }

int scheduler_step_order(const SchedConfig& c, int n, int i, int lower) {
    const bool lower_final = (i == n - 1) && (c.lower_order_final || c.final_sigmas_zero);
    return (c.solver_order == 1 || lower < 1 || lower_final) ? 1 : 2;
}

SchedCoef scheduler_coefficients(const std::vector<float>& sg, int i, int lower, float guidance,
                                 const SchedConfig& c) {
    SANA_REQUIRE(sg.size() >= 2 && i >= 0 && i < static_cast<int>(sg.size()) - 1,
                 "scheduler step_index is out of range");
    const int n = static_cast<int>(sg.size()) - 1;
    return scheduler_coefficients_order(sg, i, scheduler_step_order(c, n, i, lower), guidance, c);
}

SchedCoef scheduler_coefficients_order(const std::vector<float>& sg, int i, int order, float guidance,
                                       const SchedConfig& c) {
    SANA_REQUIRE(sg.size() >= 2 && i >= 0 && i < static_cast<int>(sg.size()) - 1,
                 "scheduler step_index is out of range");
    SANA_REQUIRE(order == 1 || i >= 1, "second-order update requires at least one previous step");
    SchedCoef k{};
    k.guidance = guidance;
    k.sigma_s = sg[i];  // convert_sana_scheduler_model_output uses the schedule's sigma as is
    float alpha_t, sigma_t, alpha_s0, sigma_s0;
    alpha_sigma(sg[i + 1], c, alpha_t, sigma_t);
    alpha_sigma(sg[i], c, alpha_s0, sigma_s0);
    const float lambda_t = lambda_of(alpha_t, sigma_t), lambda_s0 = lambda_of(alpha_s0, sigma_s0);
    const float h = lambda_t - lambda_s0;
    k.a = sigma_t / sigma_s0;
    k.b = -alpha_t * (std::exp(-h) - 1.0f);
    if (order == 1) {  // sana_scheduler_first_order_update (scheduler.cpp:175-205)
        k.c = 0.0f;
        k.inv_r0 = 0.0f;
        k.second_order = 0;
    } else {  // sana_scheduler_second_order_update (scheduler.cpp:207-270)
        float alpha_s1, sigma_s1;
        alpha_sigma(sg[i - 1], c, alpha_s1, sigma_s1);
        const float h0 = lambda_s0 - lambda_of(alpha_s1, sigma_s1);
        const float r0 = h0 / h;
        k.c = c.heun ? alpha_t * ((std::exp(-h) - 1.0f) / h + 1.0f) : -0.5f * alpha_t * (std::exp(-h) - 1.0f);
        k.inv_r0 = 1.0f / r0;
        k.second_order = 1;
    }
    return k;
}

std::vector<SchedCoef> scheduler_loop_coefficients(const SchedConfig& c, const std::vector<float>& sg, float guidance) {
    scheduler_validate(c);
    const int n = static_cast<int>(sg.size()) - 1;
    std::vector<SchedCoef> coefs;
    int lower = 0;
    for (int i = 0; i < n; ++i) {
        coefs.push_back(scheduler_coefficients(sg, i, lower, guidance, c));
        if (lower < c.solver_order) ++lower;
    }
    return coefs;
}

void timestep_features(float t, float* out) {
    const int half = 128;
    const float log_scale = -std::log(10000.0f) / static_cast<float>(half);
    for (int i = 0; i < half; ++i) {
        const float freq = std::exp(static_cast<float>(i) * log_scale);
        const float v = t * freq;
        out[i] = std::cos(v);
        out[half + i] = std::sin(v);
    }
}

// ---------------------------------------------------------------------------------------
// Engine basics
// ---------------------------------------------------------------------------------------
Engine::Engine(int device, int mode) : device_(device), mode_(mode) {
    SANA_REQUIRE(mode == kModeBf16 || mode == kModeF32, "mode must be SANA_MODE_BF16 or SANA_MODE_F32");
    SANA_CUDA(cudaSetDevice(device));
    SANA_CUDA(cudaDeviceGetAttribute(&num_sms_, cudaDevAttrMultiProcessorCount, device));
    SANA_CUDA(cudaStreamCreateWithFlags(&own_st_, cudaStreamNonBlocking));
    st_ = own_st_;
    err_.ensure(kErrWordBytes);
    SANA_CUDA(cudaMemsetAsync(err_.get(), 0, kErrWordBytes, st_));
    set_wait_limit_ns(kWaitLimitNs);
    SANA_CUDA(cudaStreamSynchronize(st_));
    tproj_table_.ensure(static_cast<size_t>(1024) * 256 * sizeof(float));
}

void Engine::set_wait_limit_ns(unsigned long long ns) {
    SANA_REQUIRE(ns >= 1000, "the wait limit must be at least 1 microsecond");
    wait_limit_host_ = ns;
    SANA_CUDA(cudaMemcpyAsync(static_cast<char*>(err_.get()) + 8, &wait_limit_host_, sizeof(wait_limit_host_),
                              cudaMemcpyHostToDevice, st_));
    SANA_CUDA(cudaStreamSynchronize(st_));
}



Engine::~Engine() {
    cudaSetDevice(device_);
    for (auto& g : graphs_)
        if (g.second.exec) cudaGraphExecDestroy(g.second.exec);
    if (pair_peer_) cudaIpcCloseMemHandle(pair_peer_);
    if (pair_region_) cudaFree(pair_region_);
    if (own_st_) cudaStreamDestroy(own_st_);
}

// Region layout: kPairBlocks flags, kPairBlocks exchange counts and the buffer capacity
// (a 1 KB header), then two receive buffers of pair_cap_ floats.
constexpr size_t kPairHeader = 1024;
constexpr size_t kPairCapOffset = 2 * kPairBlocks * sizeof(int);

PairLink Engine::pair_link() const {
    PairLink l;
    l.flags = static_cast<int*>(pair_region_);
    l.count = l.flags + kPairBlocks;
    l.recv = reinterpret_cast<float*>(static_cast<char*>(pair_region_) + kPairHeader);
    l.peer_flags = static_cast<int*>(pair_peer_);
    l.peer_recv = reinterpret_cast<float*>(static_cast<char*>(pair_peer_) + kPairHeader);
    l.capacity = pair_cap_;
    return l;
}

void Engine::pair_close() {
    SANA_CUDA(cudaSetDevice(device_));
    SANA_CUDA(cudaStreamSynchronize(st_));
    // recorded loops hold the peer's addresses
    for (auto it = graphs_.begin(); it != graphs_.end();) {
        if (it->first.find(",pair") != std::string::npos) {
            if (it->second.exec) cudaGraphExecDestroy(it->second.exec);
            it = graphs_.erase(it);
        } else {
            ++it;
        }
    }
    if (pair_peer_) SANA_CUDA(cudaIpcCloseMemHandle(pair_peer_));
    pair_peer_ = nullptr;
    pair_branch_ = -1;
}

void Engine::pair_export(size_t capacity, void* handle) {
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
    SANA_REQUIRE(capacity >= 4 && capacity <= (1ull << 32), "exchange capacity must be 4 .. 2^32 latent elements");
    static_assert(kPairCapOffset + sizeof(long long) <= kPairHeader, "pair header too small");
    pair_close();
    if (pair_region_) SANA_CUDA(cudaFree(pair_region_));
    pair_region_ = nullptr;
    pair_cap_ = static_cast<long long>((capacity + 3) / 4 * 4);
    const size_t bytes = kPairHeader + 2 * static_cast<size_t>(pair_cap_) * sizeof(float);
    SANA_CUDA(cudaMalloc(&pair_region_, bytes));
    SANA_CUDA(cudaMemsetAsync(pair_region_, 0, bytes, st_));
    SANA_CUDA(cudaMemcpyAsync(static_cast<char*>(pair_region_) + kPairCapOffset, &pair_cap_, sizeof pair_cap_,
                              cudaMemcpyHostToDevice, st_));
    SANA_CUDA(cudaStreamSynchronize(st_));
    cudaIpcMemHandle_t h;
    SANA_CUDA(cudaIpcGetMemHandle(&h, pair_region_));
    std::memcpy(handle, &h, sizeof h);
}

void Engine::pair_connect(int branch, const void* peer_handle) {
    SANA_REQUIRE(pair_region_, "export this GPU's exchange region before connecting");
    SANA_REQUIRE(branch == 0 || branch == 1, "branch must be 0 (unconditional) or 1 (conditional)");
    pair_close();
    cudaIpcMemHandle_t h;
    std::memcpy(&h, peer_handle, sizeof h);
    SANA_CUDA(cudaIpcOpenMemHandle(&pair_peer_, h, cudaIpcMemLazyEnablePeerAccess));
    // the kernel addresses the peer's buffers with this GPU's capacity: they must agree
    long long peer_cap = 0;
    SANA_CUDA(cudaMemcpy(&peer_cap, static_cast<char*>(pair_peer_) + kPairCapOffset, sizeof peer_cap,
                         cudaMemcpyDeviceToHost));
    if (peer_cap != pair_cap_) {
        cudaIpcCloseMemHandle(pair_peer_);
        pair_peer_ = nullptr;
        throw std::invalid_argument("the peer exported a different exchange capacity");
    }
    pair_branch_ = branch;
}

void Engine::denoise_loop_pair_device(const float* lat, int B, int H, int W, const float* enc, int L, int Din,
                                      const float* bias, float guidance, int num_steps, const SchedConfig& sc,
                                      float* out) {
    SANA_REQUIRE(have_w_, "weights have not been uploaded");
    SANA_REQUIRE(pair_peer_, "connect to the peer GPU before running a two-GPU loop");
    SANA_REQUIRE(B >= 1 && H >= 1 && W >= 1 && L >= 1, "invalid loop shapes");
    SANA_REQUIRE(Din == d_.Din, "encoder hidden size must match caption projection input");
    SANA_REQUIRE(static_cast<long long>(B) * d_.Cl * H * W <= pair_cap_, "latents exceed the exchange capacity");
    ensure_workspace(B, H * W, L);
    pair_run_ = true;
    try {
        run_loop(lat, B, H, W, enc, L, Din, bias, guidance, num_steps, sc, out,
                 "dev,pair" + std::to_string(pair_branch_));
    } catch (...) {
        pair_run_ = false;
        throw;
    }
    pair_run_ = false;
}

void Engine::check_device_error() {
    int h = 0;
    SANA_CUDA(cudaMemcpyAsync(&h, err_.get(), sizeof(int), cudaMemcpyDeviceToHost, st_));
    SANA_CUDA(cudaStreamSynchronize(st_));
    if (h != 0) {
        SANA_CUDA(cudaMemsetAsync(err_.get(), 0, sizeof(int), st_));
        SANA_CUDA(cudaStreamSynchronize(st_));
        throw TimeoutError("a device-side wait exceeded its time limit (code " + std::to_string(h) + ")");
    }
}

void Engine::gemm_act(const void* A, long long lda, const void* Bw, long long ldb, int M, int N, int K,
                      const Epilogue& ep, bool f32_operands) {
    GemmProblem p;
    p.A = A;
    p.lda = lda;
    p.B = Bw;
    p.ldb = ldb;
    p.M = M;
    p.N = N;
    p.K = K;
    p.a_bf16 = (!f32_operands && mode_ == kModeBf16) ? 1 : 0;
    p.b_bf16 = p.a_bf16;
    p.ep = ep;
    p.require_tc = 1;
    gemm(p, err(), st_, num_sms_);
}

static Epilogue epi_out(void* out, bool bf16_out, long long ldo, const float* bias = nullptr, int act = kActNone) {
    Epilogue e;
    e.out = out;
    e.out_bf16 = bf16_out ? 1 : 0;
    e.ldo = ldo;
    e.bias = bias;
    e.act = act;
    return e;
}

// ---------------------------------------------------------------------------------------
// Weight upload
// ---------------------------------------------------------------------------------------
void Engine::upload(const Dims& d, const float* const* model, const float* const* blocks, int layout) {
    SANA_REQUIRE(d.n_blocks >= 1, "model must contain at least one block");
    SANA_REQUIRE(d.C >= 1 && d.Cl >= 1 && d.Din >= 1 && d.E >= 2, "invalid model dimensions");
    SANA_REQUIRE(d.E % 2 == 0, "ff point conv input channels must match split GLUMB width");
    SANA_REQUIRE(d.Hs >= 1 && d.C % d.Hs == 0, "self attention hidden size must be divisible by self_num_heads");
    SANA_REQUIRE(d.Hc >= 1 && d.C % d.Hc == 0, "cross attention hidden size must be divisible by cross_num_heads");
    SANA_REQUIRE(d.C / d.Hs <= 128 && d.C / d.Hc <= 128, "head_dim above 128 is not supported");
    SANA_REQUIRE(layout == kLayoutReference || layout == kLayoutTorch, "unknown weight layout");
    SANA_REQUIRE(model != nullptr && blocks != nullptr, "weight tables must not be null");
    const int required_model[] = {0, 2, 4, 6, 8, 10, 12, 13, 14};
    for (int i : required_model) SANA_REQUIRE(model[i] != nullptr, "missing model weight tensor " + std::to_string(i));
    for (int b = 0; b < d.n_blocks; ++b) {
        const float* const* w = blocks + 26 * b;
        const int required[] = {0, 3, 5, 7, 9, 11, 13, 15, 17, 21, 23, 25};
        for (int i : required)
            SANA_REQUIRE(w[i] != nullptr, "missing block weight " + std::to_string(i) + " of block " + std::to_string(b));
    }
    for (auto& g : graphs_)
        if (g.second.exec) cudaGraphExecDestroy(g.second.exec);
    graphs_.clear();
    d_ = d;
    ws_S_ = ws_T_ = ws_L_ = 0;
    cross_qk_norm_ = false;  // new weights: the option's weights are gone with the old ones
    if (mode_ == kModeBf16) upload_impl<bf16>(model, blocks, layout);
    else upload_impl<float>(model, blocks, layout);
    SANA_CUDA(cudaStreamSynchronize(st_));
    have_w_ = true;
}

template <class T>
void Engine::upload_impl(const float* const* model, const float* const* blocks, int layout) {
    const int C = d_.C, Cl = d_.Cl, Din = d_.Din, E = d_.E, nb = d_.n_blocks;
    DevBuf staging;
    // Copies a [rows, cols] fp32 host matrix into dst (type TO at element offset) as the
    // K-major [out, in] operand. `linear` tensors arrive [in, out] in the reference layout.
    auto put = [&](auto* dst, const float* host, int out_f, int in_f, bool linear) {
        using TO = std::remove_pointer_t<decltype(dst)>;
        const size_t n = static_cast<size_t>(out_f) * in_f;
        staging.ensure(n * sizeof(float));
        SANA_CUDA(cudaMemcpyAsync(staging.get(), host, n * sizeof(float), cudaMemcpyHostToDevice, st_));
        if (linear && layout == kLayoutReference) {
            repack<TO>(staging.as<float>(), in_f, out_f, true, dst, st_);
        } else {
            repack<TO>(staging.as<float>(), out_f, in_f, false, dst, st_);
        }
        SANA_CUDA(cudaStreamSynchronize(st_));
    };
    auto vec = [&](DevBuf& dst, const float* host, size_t n, float fill_if_null, bool keep_null) {
        if (!host && keep_null) {
            dst.release();
            return;
        }
        dst.ensure(n * sizeof(float));
        if (host) {
            SANA_CUDA(cudaMemcpyAsync(dst.get(), host, n * sizeof(float), cudaMemcpyHostToDevice, st_));
        } else {
            std::vector<float> f(n, fill_if_null);
            SANA_CUDA(cudaMemcpyAsync(dst.get(), f.data(), n * sizeof(float), cudaMemcpyHostToDevice, st_));
        }
    };
    const size_t as = sizeof(T);

    // model-level tensors (SanaDenoiserWeights order)
    cap_w1_.ensure(static_cast<size_t>(C) * Din * as);
    put(cap_w1_.as<T>(), model[0], C, Din, true);
    vec(cap_b1_, model[1], C, 0.f, true);
    cap_w2_.ensure(static_cast<size_t>(C) * C * as);
    put(cap_w2_.as<T>(), model[2], C, C, true);
    vec(cap_b2_, model[3], C, 0.f, true);
    patch_w_.ensure(static_cast<size_t>(C) * Cl * as);
    put(patch_w_.as<T>(), model[4], C, Cl, false);
    vec(patch_b_, model[5], C, 0.f, true);
    te_w1_.ensure(static_cast<size_t>(C) * 256 * as);
    put(te_w1_.as<T>(), model[6], C, 256, true);
    vec(te_b1_, model[7], C, 0.f, true);
    te_w2_.ensure(static_cast<size_t>(C) * C * as);
    put(te_w2_.as<T>(), model[8], C, C, true);
    vec(te_b2_, model[9], C, 0.f, true);
    tp_w_.ensure(static_cast<size_t>(6) * C * C * as);
    put(tp_w_.as<T>(), model[10], 6 * C, C, true);
    vec(tp_b_, model[11], 6 * static_cast<size_t>(C), 0.f, true);
    vec(cap_norm_, model[12], C, 1.f, false);
    vec(ftable_, model[13], 2 * static_cast<size_t>(C), 0.f, false);
    out_w_.ensure(static_cast<size_t>(Cl) * C * as);
    put(out_w_.as<T>(), model[14], Cl, C, true);
    vec(out_b_, model[15], Cl, 0.f, true);

    // blocks (SanaBlockWeights field order)
    blk_.clear();
    blk_.resize(nb);
    tables_.ensure(static_cast<size_t>(nb) * 6 * C * 4);
    for (int b = 0; b < nb; ++b) {
        const float* const* w = blocks + 26 * b;
        BlockWeights& k = blk_[b];
        SANA_CUDA(cudaMemcpyAsync(tables_.as<float>() + static_cast<size_t>(b) * 6 * C, w[0],
                                  6 * static_cast<size_t>(C) * 4, cudaMemcpyHostToDevice, st_));
        vec(k.ln1g, w[1], C, 1.f, true);
        vec(k.ln1b, w[2], C, 0.f, true);
        k.wqkv.ensure(static_cast<size_t>(3) * C * C * as);
        put(k.wqkv.as<T>(), w[3], C, C, true);
        put(k.wqkv.as<T>() + static_cast<size_t>(C) * C, w[5], C, C, true);
        put(k.wqkv.as<T>() + static_cast<size_t>(2) * C * C, w[7], C, C, true);
        if (w[4] || w[6] || w[8]) {
            std::vector<float> bq(3 * static_cast<size_t>(C), 0.f);
            for (int j = 0; j < 3; ++j)
                if (w[4 + 2 * j]) std::memcpy(bq.data() + static_cast<size_t>(j) * C, w[4 + 2 * j], C * sizeof(float));
            vec(k.bqkv, bq.data(), bq.size(), 0.f, false);
        } else {
            k.bqkv.release();
        }
        k.wo.ensure(static_cast<size_t>(C) * C * as);
        put(k.wo.as<T>(), w[9], C, C, true);
        vec(k.bo, w[10], C, 0.f, true);
        k.wcq.ensure(static_cast<size_t>(C) * C * as);
        put(k.wcq.as<T>(), w[11], C, C, true);
        vec(k.bcq, w[12], C, 0.f, true);
        k.wckv.ensure(static_cast<size_t>(2) * C * C * as);
        put(k.wckv.as<T>(), w[13], C, C, true);
        put(k.wckv.as<T>() + static_cast<size_t>(C) * C, w[15], C, C, true);
        if (w[14] || w[16]) {
            std::vector<float> bkv(2 * static_cast<size_t>(C), 0.f);
            if (w[14]) std::memcpy(bkv.data(), w[14], C * sizeof(float));
            if (w[16]) std::memcpy(bkv.data() + C, w[16], C * sizeof(float));
            vec(k.bckv, bkv.data(), bkv.size(), 0.f, false);
        } else {
            k.bckv.release();
        }
        k.wco.ensure(static_cast<size_t>(C) * C * as);
        put(k.wco.as<T>(), w[17], C, C, true);
        vec(k.bco, w[18], C, 0.f, true);
        vec(k.ln2g, w[19], C, 1.f, true);
        vec(k.ln2b, w[20], C, 0.f, true);
        k.winv.ensure(static_cast<size_t>(E) * C * as);
        put(k.winv.as<T>(), w[21], E, C, false);
        vec(k.binv, w[22], E, 0.f, true);
        vec(k.wdw, w[23], static_cast<size_t>(E) * 9, 0.f, false);
        vec(k.bdw, w[24], E, 0.f, false);
        k.wpt.ensure(static_cast<size_t>(C) * (E / 2) * as);
        put(k.wpt.as<T>(), w[25], C, E / 2, false);
    }
}

// ---------------------------------------------------------------------------------------
// Workspace
// ---------------------------------------------------------------------------------------
void Engine::ensure_workspace(int S, int T, int L) {
    SANA_REQUIRE(have_w_, "weights have not been uploaded");
    if (S <= ws_S_ && T <= ws_T_ && L <= ws_L_) return;
    S = std::max(S, ws_S_);
    T = std::max(T, ws_T_);
    L = std::max(L, ws_L_);
    for (auto& g : graphs_)
        if (g.second.exec) cudaGraphExecDestroy(g.second.exec);
    graphs_.clear();
    const size_t C = d_.C, E = d_.E, Cl = d_.Cl, Din = d_.Din, nb = d_.n_blocks;
    const size_t M = static_cast<size_t>(S) * T, SL = static_cast<size_t>(S) * std::max(L, 1);
    const size_t as = act_size();
    const size_t Ds = C / d_.Hs;
    const size_t chunks = static_cast<size_t>(linattn_chunks(T));
    x_.ensure(M * C * 4);
    x1_.ensure(M * C * 4);
    x2_.ensure(M * C * 4);
    x3_.ensure(M * C * 4);
    xb_.ensure(M * C * as);
    a_.ensure(M * C * as);
    qkv_.ensure(M * 3 * C * as);
    ao_.ensure(M * C * as);
    cq_.ensure(M * C * as);
    ffh_.ensure(M * E * as);
    glu_.ensure(M * (E / 2) * as);
    part_.ensure(static_cast<size_t>(S) * d_.Hs * (chunks + 1) * (Ds + 1) * Ds * 4);
    y_.ensure(M * C * 4);
    noise_.ensure(M * Cl * 4);
    pt_.ensure(M * Cl * 4);
    ctx_.ensure(SL * C * as);
    ctx_f32_.ensure(SL * C * 4);
    caph_.ensure(SL * C * as);
    capp_.ensure(SL * C * 4);
    enc_t_.ensure(SL * Din * as);
    ckv_.ensure(nb * SL * 2 * C * as);
    ckv1_.ensure(SL * 2 * C * as);
    tproj_.ensure(static_cast<size_t>(S) * 256 * 4);
    teh_.ensure(static_cast<size_t>(S) * C * 4);
    emb_.ensure(static_cast<size_t>(S) * C * 4);
    embs_.ensure(static_cast<size_t>(S) * C * 4);
    tmod_.ensure(static_cast<size_t>(S) * 6 * C * 4);
    mods_.ensure(nb * S * 6 * C * 4);
    fmod_.ensure(static_cast<size_t>(S) * 2 * C * 4);
    bias_d_.ensure(SL * 4);
    kvlen_.ensure(static_cast<size_t>(S) * 4);
    lat_.ensure(static_cast<size_t>(S) * Cl * T * 4);
    hist_.ensure(2 * static_cast<size_t>(S) * Cl * T * 4);
    in_lat_.ensure(static_cast<size_t>(S) * Cl * T * 4);
    in_enc_.ensure(SL * Din * 4);
    in_bias_.ensure(SL * 4);
    in_x_.ensure(M * C * 4);
    in_tmod_.ensure(static_cast<size_t>(S) * 6 * C * 4);
    out_buf_.ensure(std::max(M * C, static_cast<size_t>(S) * Cl * T) * 4);
    ws_S_ = S;
    ws_T_ = T;
    ws_L_ = L;
}

// ---------------------------------------------------------------------------------------
// Pieces of the forward pass (templated on the activation type)
// ---------------------------------------------------------------------------------------
template <class T>
void Engine::caption_impl(const float* enc_d, int S, int L) {
    const int C = d_.C, Din = d_.Din;
    const long long rows = static_cast<long long>(S) * L;
    const bool bf = mode_ == kModeBf16;
    const void* A = enc_d;
    if (bf) {
        convert<T>(enc_d, rows * Din, enc_t_.as<T>(), st_);
        A = enc_t_.get();
    }
    // project_caption_context (transformer_ops.cpp:64-76)
    gemm_act(A, Din, cap_w1_.get(), Din, static_cast<int>(rows), C, Din,
             epi_out(caph_.get(), bf, C, cap_b1_.as<float>(), kActGelu));
    gemm_act(caph_.get(), C, cap_w2_.get(), C, static_cast<int>(rows), C, C,
             epi_out(capp_.get(), false, C, cap_b2_.as<float>()));
    rms_norm<T>(capp_.as<float>(), rows, C, 1e-5f, cap_norm_.as<float>(), ctx_.as<T>(), st_);
}

template <class T>
void Engine::kv_impl(int b, int S, int L, void* dst) {
    const int C = d_.C;
    const long long rows = static_cast<long long>(S) * L;
    gemm_act(ctx_.get(), C, blk_[b].wckv.get(), C, static_cast<int>(rows), 2 * C, C,
             epi_out(dst, mode_ == kModeBf16, 2 * C, blk_[b].bckv.as<float>()));
    if (cross_qk_norm_)  // the K half of each [k | v] row
        rms_norm_rows<T>(static_cast<T*>(dst), rows, C, 2LL * C, cross_qk_eps_, blk_[b].ckn.as<float>(), st_);
}

void Engine::set_cross_qk_norm(bool enable, const float* const* q_w, const float* const* k_w, float eps) {
    SANA_REQUIRE(have_w_, "weights have not been uploaded");
    SANA_REQUIRE(!enable || eps >= 0.f, "eps must not be negative");
    for (int b = 0; b < d_.n_blocks; ++b) {
        BlockWeights& w = blk_[b];
        w.cqn.release();
        w.ckn.release();
        if (!enable) continue;
        const size_t bytes = static_cast<size_t>(d_.C) * 4;
        if (q_w && q_w[b]) {
            w.cqn.ensure(bytes);
            SANA_CUDA(cudaMemcpyAsync(w.cqn.get(), q_w[b], bytes, cudaMemcpyHostToDevice, st_));
        }
        if (k_w && k_w[b]) {
            w.ckn.ensure(bytes);
            SANA_CUDA(cudaMemcpyAsync(w.ckn.get(), k_w[b], bytes, cudaMemcpyHostToDevice, st_));
        }
    }
    SANA_CUDA(cudaStreamSynchronize(st_));
    cross_qk_norm_ = enable;
    cross_qk_eps_ = eps;
    for (auto& g : graphs_)  // captured loops hold the old choice
        if (g.second.exec) cudaGraphExecDestroy(g.second.exec);
    graphs_.clear();
}

template <class T>
void Engine::kv_all_impl(int S, int L) {
    const size_t stride = static_cast<size_t>(S) * L * 2 * d_.C;
    for (int b = 0; b < d_.n_blocks; ++b) kv_impl<T>(b, S, L, ckv_.as<T>() + b * stride);
}

// block_forward (transformer.cpp:726-778) on device buffers. x_in may alias the outputs.
template <class T>
void Engine::block_impl(int b, const float* x_in, float* x_self, float* x_cross, float* x_ff, int S, int Tn, int L,
                        const float* mod_b, const void* ckv_b, const float* bias_d, const int* kvlen_d) {
    const BlockWeights& w = blk_[b];
    const int C = d_.C, E = d_.E;
    const int M = S * Tn;
    const long long C6 = 6LL * C;
    const bool bf = mode_ == kModeBf16;
    T* a = a_.as<T>();
    T* qkv = qkv_.as<T>();
    T* ao = ao_.as<T>();

    // self attention: LN(eps 1e-6) + modulate(shift_msa, scale_msa) -> QKV -> linear attention
    {
        ProfScope p(this, "ln_modulate");
        ln_modulate<T>(x_in, M, C, Tn, w.ln1g.as<float>(), w.ln1b.as<float>(), mod_b, C6, 0, 1, 1e-6f, a, st_);
    }
    {
        ProfScope p(this, "gemm_qkv");
        gemm_act(a, C, w.wqkv.get(), C, M, 3 * C, C, epi_out(qkv, bf, 3 * C, w.bqkv.as<float>()));
    }
    const int Ds = C / d_.Hs;
    {
        ProfScope p(this, "linear_attention");
        linear_attention<T>(qkv, 3LL * C, 0, qkv, 3LL * C, C, 2 * C, S, Tn, Tn, d_.Hs, Ds, part_.as<float>(), ao, C,
                            st_);
    }
    // out projection + gate_msa + residual (after_self); bf16 mode also keeps a bf16 copy
    {
        Epilogue e = epi_out(x_self, false, C, w.bo.as<float>());
        e.resid = x_in;
        e.ldr = C;
        e.gate = mod_b + 2 * C;
        e.gate_ld = C6;
        e.rows_per_gate = Tn;
        if (bf) {
            e.out2 = xb_.get();
            e.out2_bf16 = 1;
            e.ldo2 = C;
        }
        ProfScope p(this, "gemm_out");
        gemm_act(ao, C, w.wo.get(), C, M, C, C, e);
    }
    // cross attention (no norm, no gate): q from the residual stream
    const void* xq = bf ? static_cast<const void*>(xb_.get()) : static_cast<const void*>(x_self);
    {
        ProfScope p(this, "gemm_cross_q");
        gemm_act(xq, C, w.wcq.get(), C, M, C, C, epi_out(cq_.get(), bf, C, w.bcq.as<float>()));
    }
    if (cross_qk_norm_) {
        ProfScope p(this, "cross_q_norm");
        rms_norm_rows<T>(cq_.as<T>(), M, C, C, cross_qk_eps_, w.cqn.as<float>(), st_);
    }
    const int Dc = C / d_.Hc;
    const float scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(Dc)));
    {
        ProfScope p(this, "cross_attention");
        cross_attention<T>(cq_.as<T>(), C, static_cast<const T*>(ckv_b), 2LL * C, 0, C, bias_d, kvlen_d, S, Tn, L,
                           d_.Hc, Dc, scale, ao, C, err(), st_);
    }
    {
        Epilogue e = epi_out(x_cross, false, C, w.bco.as<float>());
        e.resid = x_self;
        e.ldr = C;
        ProfScope p(this, "gemm_cross_out");
        gemm_act(ao, C, w.wco.get(), C, M, C, C, e);
    }
    // Mix-FFN: LN + modulate(shift_mlp, scale_mlp) -> inverted 1x1 + SiLU -> depthwise + GLU
    // -> point 1x1 + gate_mlp + residual (after_ff)
    {
        ProfScope p(this, "ln_modulate");
        ln_modulate<T>(x_cross, M, C, Tn, w.ln2g.as<float>(), w.ln2b.as<float>(), mod_b, C6, 3, 4, 1e-6f, a, st_);
    }
    {
        ProfScope p(this, "gemm_ff_inverted");
        gemm_act(a, C, w.winv.get(), C, M, E, C, epi_out(ffh_.get(), bf, E, w.binv.as<float>(), kActSilu));
    }
    const int side = static_cast<int>(std::lround(std::sqrt(static_cast<double>(Tn))));
    {
        ProfScope p(this, "depthwise_glu");
        depthwise_glu<T>(ffh_.as<T>(), E, S, side, side, E, w.wdw.as<float>(), w.bdw.as<float>(), glu_.as<T>(), E / 2,
                         err(), st_);
    }
    {
        Epilogue e = epi_out(x_ff, false, C);
        e.resid = x_cross;
        e.ldr = C;
        e.gate = mod_b + 5 * C;
        e.gate_ld = C6;
        e.rows_per_gate = Tn;
        ProfScope p(this, "gemm_ff_point");
        gemm_act(glu_.get(), E / 2, w.wpt.get(), E / 2, M, C, E / 2, e);
    }
}

// t-embedding MLP and t_block (transformer.cpp:638-656), fp32 weights and activations.
template <class T>
void Engine::time_embed_impl(const void* tproj_d, int S) {
    // timestep embedding MLP and t_block (transformer.cpp:639-652); in bf16 mode the three
    // projections run on the tensor cores with bf16 operands like every other dense
    // projection, emb itself (the final layer's modulation input) staying fp32
    const int C = d_.C;
    const bool b16 = sizeof(T) == 2;
    gemm_act(tproj_d, 256, te_w1_.get(), 256, S, C, 256, epi_out(teh_.get(), b16, C, te_b1_.as<float>(), kActSilu),
             false);
    Epilogue e = epi_out(emb_.get(), false, C, te_b2_.as<float>());
    e.out2 = embs_.get();
    e.out2_bf16 = b16 ? 1 : 0;
    e.ldo2 = C;
    e.act2 = kActSilu;
    gemm_act(teh_.get(), C, te_w2_.get(), C, S, C, C, e, false);
    gemm_act(embs_.get(), C, tp_w_.get(), C, S, 6 * C, C, epi_out(tmod_.get(), false, 6 * C, tp_b_.as<float>()), false);
}

// repeat_batch_4d_local + patch embed 1x1 conv + grid_to_tokens (transformer.cpp:627-636).
template <class T>
void Engine::prologue_impl(const float* lat_d, int images, int S, int H, int W) {
    const int C = d_.C, Cl = d_.Cl;
    const int M = S * H * W;
    patch_tokens<T>(lat_d, images, S, Cl, H * W, pt_.as<T>(), st_);
    gemm_act(pt_.get(), Cl, patch_w_.get(), Cl, M, C, Cl, epi_out(x_.get(), false, C, patch_b_.as<float>()), false);
}

// Final layer (transformer.cpp:668-678): LN (no affine) + modulate(emb + table) + proj_out.
template <class T>
void Engine::epilogue_impl(int S, int Tn) {
    const int C = d_.C, Cl = d_.Cl;
    const int M = S * Tn;
    final_modulation(emb_.as<float>(), S, C, ftable_.as<float>(), fmod_.as<float>(), st_);
    ln_modulate<T>(x_.as<float>(), M, C, Tn, nullptr, nullptr, fmod_.as<float>(), 2LL * C, 0, 1, 1e-6f, y_.as<T>(),
                   st_);
    gemm_act(y_.get(), C, out_w_.get(), C, M, Cl, C, epi_out(noise_.get(), false, Cl, out_b_.as<float>()), false);
}

template <class T>
void Engine::loop_body(const float* lat_in, int B, int H, int W, const float* enc_d, int L, int Din,
                       const float* bias_d, const std::vector<SchedCoef>& coefs, float* out_d) {
    (void)Din;
    // both branches (uncond then cond sequences), or this GPU's branch of a two-GPU pair
    const int S = pair_run_ ? B : 2 * B, Tn = H * W, C = d_.C, Cl = d_.Cl, nb = d_.n_blocks;
    const size_t n_lat = static_cast<size_t>(B) * Cl * Tn;
    {
        ProfScope p(this, "caption_projection");
        caption_impl<T>(enc_d, S, L);
    }
    {
        ProfScope p(this, "gemm_cross_kv");
        kv_all_impl<T>(S, L);
    }
    if (bias_d) caption_kv_len(bias_d, S, L, kvlen_.as<int>(), st_);
    SANA_CUDA(cudaMemcpyAsync(lat_.get(), lat_in, n_lat * 4, cudaMemcpyDeviceToDevice, st_));
    const size_t ckv_stride = static_cast<size_t>(S) * L * 2 * C;
    for (size_t step = 0; step < coefs.size(); ++step) {
        {
            ProfScope p(this, "timestep_embedding");
            broadcast_rows<T>(tproj_table_.as<float>() + step * 256, S, 256, tproj_.as<T>(), st_);
            time_embed_impl<T>(tproj_.get(), S);
            block_modulation(tmod_.as<float>(), S, C, tables_.as<float>(), nb, mods_.as<float>(), st_);
        }
        {
            ProfScope p(this, "patch_embed");
            prologue_impl<T>(lat_.as<float>(), B, S, H, W);
        }
        for (int b = 0; b < nb; ++b) {
            block_impl<T>(b, x_.as<float>(), x_.as<float>(), x_.as<float>(), x_.as<float>(), S, Tn, L,
                          mods_.as<float>() + static_cast<size_t>(b) * S * 6 * C, ckv_.as<T>() + b * ckv_stride, bias_d,
                          bias_d ? kvlen_.as<int>() : nullptr);
        }
        {
            ProfScope p(this, "final_layer");
            epilogue_impl<T>(S, Tn);
        }
        float* cur = hist_.as<float>() + (step % 2) * n_lat;
        const float* prev = hist_.as<float>() + ((step + 1) % 2) * n_lat;
        ProfScope p(this, "cfg_scheduler");
        if (pair_run_)
            cfg_pair_step(noise_.as<float>(), pair_link(), B, Cl, Tn, lat_.as<float>(), cur, prev, coefs[step],
                          pair_branch_, err(), st_);
        else
            cfg_scheduler_step(noise_.as<float>(), B, Cl, Tn, lat_.as<float>(), cur, prev, coefs[step], st_);
    }
    SANA_CUDA(cudaMemcpyAsync(out_d, lat_.get(), n_lat * 4, cudaMemcpyDeviceToDevice, st_));
}

// ---------------------------------------------------------------------------------------
// Loop driver with graph capture
// ---------------------------------------------------------------------------------------
void Engine::run_loop(const float* lat_d, int B, int H, int W, const float* enc_d, int L, int Din,
                      const float* bias_d, float guidance, int num_steps, const SchedConfig& sc, float* out_d,
                      const std::string& key_extra) {
    SANA_REQUIRE(num_steps >= 1 && num_steps <= 1024, "num_inference_steps must be in 1..1024");
    std::vector<float> ts, sg;
    scheduler_schedule(num_steps, sc, ts, sg);
    const std::vector<SchedCoef> coefs = scheduler_loop_coefficients(sc, sg, guidance);
    std::vector<float> table(static_cast<size_t>(num_steps) * 256);
    for (int i = 0; i < num_steps; ++i) timestep_features(ts[i], table.data() + static_cast<size_t>(i) * 256);
    SANA_CUDA(cudaMemcpyAsync(tproj_table_.get(), table.data(), table.size() * 4, cudaMemcpyHostToDevice, st_));

    std::ostringstream key;
    key << B << ',' << H << ',' << W << ',' << L << ',' << Din << ',' << num_steps << ',' << guidance << ','
        << sc.flow_shift << ',' << sc.num_train_timesteps << ',' << sc.flow_sigmas << sc.solver_order
        << sc.lower_order_final << sc.final_sigmas_zero << sc.heun << ',' << lat_d << ',' << enc_d << ',' << bias_d
        << ',' << out_d << ',' << key_extra;
    GraphEntry& g = graphs_[key.str()];
    auto body = [&] {
        if (mode_ == kModeBf16) loop_body<bf16>(lat_d, B, H, W, enc_d, L, Din, bias_d, coefs, out_d);
        else loop_body<float>(lat_d, B, H, W, enc_d, L, Din, bias_d, coefs, out_d);
    };
    if (g.calls == 0) {
        body();  // first call: eager (sets kernel attributes, warms up)
    } else {
        if (!g.exec) {
            cudaGraph_t graph;
            SANA_CUDA(cudaStreamBeginCapture(st_, cudaStreamCaptureModeThreadLocal));
            try {
                body();
            } catch (...) {
                cudaStreamEndCapture(st_, &graph);
                throw;
            }
            SANA_CUDA(cudaStreamEndCapture(st_, &graph));
            size_t n = 0;
            SANA_CUDA(cudaGraphGetNodes(graph, nullptr, &n));
            std::vector<cudaGraphNode_t> nodes(n);
            SANA_CUDA(cudaGraphGetNodes(graph, nodes.data(), &n));
            int kernels = 0;
            for (auto nd : nodes) {
                cudaGraphNodeType t;
                SANA_CUDA(cudaGraphNodeGetType(nd, &t));
                if (t == cudaGraphNodeTypeKernel) ++kernels;
            }
            g.launches = kernels;
            SANA_CUDA(cudaGraphInstantiate(&g.exec, graph, 0));
            SANA_CUDA(cudaGraphDestroy(graph));
        }
        SANA_CUDA(cudaGraphLaunch(g.exec, st_));
        last_launches_ = g.launches;
    }
    ++g.calls;
}

void Engine::denoise_loop_device(const float* lat, int B, int H, int W, const float* enc, int L, int Din,
                                 const float* bias, float guidance, int num_steps, const SchedConfig& sc, float* out) {
    SANA_REQUIRE(have_w_, "weights have not been uploaded");
    SANA_REQUIRE(B >= 1 && H >= 1 && W >= 1 && L >= 1, "invalid loop shapes");
    SANA_REQUIRE(Din == d_.Din, "encoder hidden size must match caption projection input");
    ensure_workspace(2 * B, H * W, L);
    run_loop(lat, B, H, W, enc, L, Din, bias, guidance, num_steps, sc, out, "dev");
}

void Engine::denoise_loop(const float* lat, int B, int H, int W, const float* enc, int L, int Din, const float* bias,
                          float guidance, int num_steps, const SchedConfig& sc, float* out) {
    SANA_REQUIRE(have_w_, "weights have not been uploaded");
    SANA_REQUIRE(B >= 1 && H >= 1 && W >= 1 && L >= 1, "invalid loop shapes");
    SANA_REQUIRE(Din == d_.Din, "encoder hidden size must match caption projection input");
    const int S = 2 * B;
    ensure_workspace(S, H * W, L);
    const size_t n_lat = static_cast<size_t>(B) * d_.Cl * H * W;
    SANA_CUDA(cudaMemcpyAsync(in_lat_.get(), lat, n_lat * 4, cudaMemcpyHostToDevice, st_));
    SANA_CUDA(cudaMemcpyAsync(in_enc_.get(), enc, static_cast<size_t>(S) * L * Din * 4, cudaMemcpyHostToDevice, st_));
    if (bias) {
        SANA_CUDA(cudaMemcpyAsync(in_bias_.get(), bias, static_cast<size_t>(S) * L * 4, cudaMemcpyHostToDevice, st_));
    }
    run_loop(in_lat_.as<float>(), B, H, W, in_enc_.as<float>(), L, Din, bias ? in_bias_.as<float>() : nullptr,
             guidance, num_steps, sc, out_buf_.as<float>(), "host");
    SANA_CUDA(cudaMemcpyAsync(out, out_buf_.get(), n_lat * 4, cudaMemcpyDeviceToHost, st_));
    SANA_CUDA(cudaStreamSynchronize(st_));
    check_device_error();
}

// ---------------------------------------------------------------------------------------
// Finer host-buffer entry points
// ---------------------------------------------------------------------------------------
void Engine::time_embed(const float* t, int S, float* emb, float* tmod) {
    SANA_REQUIRE(have_w_, "weights have not been uploaded");
    SANA_REQUIRE(S >= 1 && S <= 1024, "time_embed takes 1..1024 timesteps");
    ensure_workspace(S, 1, 1);
    std::vector<float> feats(static_cast<size_t>(S) * 256);
    for (int s = 0; s < S; ++s) timestep_features(t[s], feats.data() + static_cast<size_t>(s) * 256);
    SANA_CUDA(cudaMemcpyAsync(tproj_table_.get(), feats.data(), feats.size() * 4, cudaMemcpyHostToDevice, st_));
    const int C = d_.C;
    if (mode_ == kModeBf16) {
        convert<bf16>(tproj_table_.as<float>(), static_cast<long long>(S) * 256, tproj_.as<bf16>(), st_);
        time_embed_impl<bf16>(tproj_.get(), S);
    } else {
        convert<float>(tproj_table_.as<float>(), static_cast<long long>(S) * 256, tproj_.as<float>(), st_);
        time_embed_impl<float>(tproj_.get(), S);
    }
    if (emb)
        SANA_CUDA(cudaMemcpyAsync(emb, emb_.get(), static_cast<size_t>(S) * C * 4, cudaMemcpyDeviceToHost, st_));
    if (tmod)
        SANA_CUDA(cudaMemcpyAsync(tmod, tmod_.get(), static_cast<size_t>(S) * 6 * C * 4, cudaMemcpyDeviceToHost, st_));
    SANA_CUDA(cudaStreamSynchronize(st_));
}

void Engine::project_caption(const float* enc, int S, int L, int Din, float* out) {
    SANA_REQUIRE(have_w_, "weights have not been uploaded");
    SANA_REQUIRE(Din == d_.Din, "encoder hidden size must match caption projection input");
    ensure_workspace(S, 1, L);
    const size_t rows = static_cast<size_t>(S) * L;
    SANA_CUDA(cudaMemcpyAsync(in_enc_.get(), enc, rows * Din * 4, cudaMemcpyHostToDevice, st_));
    if (mode_ == kModeBf16) caption_impl<bf16>(in_enc_.as<float>(), S, L);
    else caption_impl<float>(in_enc_.as<float>(), S, L);
    // The caller receives the fp32 normalised context (ctx_ holds the activation type).
    rms_norm<float>(capp_.as<float>(), static_cast<long long>(rows), d_.C, 1e-5f, cap_norm_.as<float>(),
                    ctx_f32_.as<float>(), st_);
    SANA_CUDA(cudaMemcpyAsync(out, ctx_f32_.get(), rows * d_.C * 4, cudaMemcpyDeviceToHost, st_));
    SANA_CUDA(cudaStreamSynchronize(st_));
    check_device_error();
}

void Engine::block_forward(int b, const float* x, int S, int Tn, const float* ctx, int L, const float* tmod,
                           const float* bias, float* after_self, float* after_cross, float* after_ff) {
    SANA_REQUIRE(have_w_, "weights have not been uploaded");
    SANA_REQUIRE(b >= 0 && b < d_.n_blocks, "invalid model block range");
    SANA_REQUIRE(S >= 1 && Tn >= 1 && L >= 1, "invalid block shapes");
    const long long side = std::llround(std::sqrt(static_cast<double>(Tn)));
    SANA_REQUIRE(side * side == Tn, "token count must form a square grid");
    ensure_workspace(S, Tn, L);
    const int C = d_.C;
    const size_t M = static_cast<size_t>(S) * Tn;
    SANA_CUDA(cudaMemcpyAsync(in_x_.get(), x, M * C * 4, cudaMemcpyHostToDevice, st_));
    SANA_CUDA(cudaMemcpyAsync(ctx_f32_.get(), ctx, static_cast<size_t>(S) * L * C * 4, cudaMemcpyHostToDevice, st_));
    SANA_CUDA(cudaMemcpyAsync(in_tmod_.get(), tmod, static_cast<size_t>(S) * 6 * C * 4, cudaMemcpyHostToDevice, st_));
    if (bias) {
        SANA_CUDA(cudaMemcpyAsync(bias_d_.get(), bias, static_cast<size_t>(S) * L * 4, cudaMemcpyHostToDevice, st_));
        caption_kv_len(bias_d_.as<float>(), S, L, kvlen_.as<int>(), st_);
    }
    block_modulation(in_tmod_.as<float>(), S, C, tables_.as<float>() + static_cast<size_t>(b) * 6 * C, 1,
                     mods_.as<float>(), st_);
    auto run = [&](auto tag) {
        using T = decltype(tag);
        convert<T>(ctx_f32_.as<float>(), static_cast<long long>(S) * L * C, ctx_.as<T>(), st_);
        kv_impl<T>(b, S, L, ckv1_.get());
        block_impl<T>(b, in_x_.as<float>(), x1_.as<float>(), x2_.as<float>(), x3_.as<float>(), S, Tn, L,
                      mods_.as<float>(), ckv1_.get(), bias ? bias_d_.as<float>() : nullptr,
                      bias ? kvlen_.as<int>() : nullptr);
    };
    if (mode_ == kModeBf16) run(bf16{});
    else run(float{});
    if (after_self) SANA_CUDA(cudaMemcpyAsync(after_self, x1_.get(), M * C * 4, cudaMemcpyDeviceToHost, st_));
    if (after_cross) SANA_CUDA(cudaMemcpyAsync(after_cross, x2_.get(), M * C * 4, cudaMemcpyDeviceToHost, st_));
    if (after_ff) SANA_CUDA(cudaMemcpyAsync(after_ff, x3_.get(), M * C * 4, cudaMemcpyDeviceToHost, st_));
    SANA_CUDA(cudaStreamSynchronize(st_));
    check_device_error();
}

void Engine::run_blocks(const float* x, int S, int Tn, const float* ctx, int L, const float* tmod, const float* bias,
                        int begin, int end, float* out) {
    SANA_REQUIRE(have_w_, "weights have not been uploaded");
    SANA_REQUIRE(begin >= 0 && begin <= end && end <= d_.n_blocks, "invalid model block range");
    const long long side = std::llround(std::sqrt(static_cast<double>(Tn)));
    SANA_REQUIRE(side * side == Tn, "token count must form a square grid");
    ensure_workspace(S, Tn, L);
    const int C = d_.C;
    const size_t M = static_cast<size_t>(S) * Tn;
    SANA_CUDA(cudaMemcpyAsync(x_.get(), x, M * C * 4, cudaMemcpyHostToDevice, st_));
    SANA_CUDA(cudaMemcpyAsync(ctx_f32_.get(), ctx, static_cast<size_t>(S) * L * C * 4, cudaMemcpyHostToDevice, st_));
    SANA_CUDA(cudaMemcpyAsync(in_tmod_.get(), tmod, static_cast<size_t>(S) * 6 * C * 4, cudaMemcpyHostToDevice, st_));
    if (bias) {
        SANA_CUDA(cudaMemcpyAsync(bias_d_.get(), bias, static_cast<size_t>(S) * L * 4, cudaMemcpyHostToDevice, st_));
        caption_kv_len(bias_d_.as<float>(), S, L, kvlen_.as<int>(), st_);
    }
    block_modulation(in_tmod_.as<float>(), S, C, tables_.as<float>(), d_.n_blocks, mods_.as<float>(), st_);
    auto run = [&](auto tag) {
        using T = decltype(tag);
        convert<T>(ctx_f32_.as<float>(), static_cast<long long>(S) * L * C, ctx_.as<T>(), st_);
        for (int b = begin; b < end; ++b) {
            kv_impl<T>(b, S, L, ckv1_.get());
            block_impl<T>(b, x_.as<float>(), x_.as<float>(), x_.as<float>(), x_.as<float>(), S, Tn, L,
                          mods_.as<float>() + static_cast<size_t>(b) * S * 6 * C, ckv1_.get(),
                          bias ? bias_d_.as<float>() : nullptr, bias ? kvlen_.as<int>() : nullptr);
        }
    };
    if (mode_ == kModeBf16) run(bf16{});
    else run(float{});
    SANA_CUDA(cudaMemcpyAsync(out, x_.get(), M * C * 4, cudaMemcpyDeviceToHost, st_));
    SANA_CUDA(cudaStreamSynchronize(st_));
    check_device_error();
}

// tokens [S*T, Cl] (device) -> NCHW [S, Cl, T] (host)
static void tokens_to_nchw_host(const std::vector<float>& tok, int S, int T, int Cl, float* out) {
    for (int s = 0; s < S; ++s)
        for (int t = 0; t < T; ++t)
            for (int c = 0; c < Cl; ++c)
                out[(static_cast<size_t>(s) * Cl + c) * T + t] = tok[(static_cast<size_t>(s) * T + t) * Cl + c];
}

void Engine::forward_nocfg(const float* lat, int S, int H, int W, float t, const float* ctx, int L, const float* bias,
                           float* noise) {
    SANA_REQUIRE(have_w_, "weights have not been uploaded");
    SANA_REQUIRE(S >= 1 && H >= 1 && W >= 1 && L >= 1, "invalid forward shapes");
    const int Tn = H * W, C = d_.C, Cl = d_.Cl;
    ensure_workspace(S, Tn, L);
    SANA_CUDA(cudaMemcpyAsync(in_lat_.get(), lat, static_cast<size_t>(S) * Cl * Tn * 4, cudaMemcpyHostToDevice, st_));
    SANA_CUDA(cudaMemcpyAsync(ctx_f32_.get(), ctx, static_cast<size_t>(S) * L * C * 4, cudaMemcpyHostToDevice, st_));
    if (bias) {
        SANA_CUDA(cudaMemcpyAsync(bias_d_.get(), bias, static_cast<size_t>(S) * L * 4, cudaMemcpyHostToDevice, st_));
        caption_kv_len(bias_d_.as<float>(), S, L, kvlen_.as<int>(), st_);
    }
    std::vector<float> feat(256);
    timestep_features(t, feat.data());
    SANA_CUDA(cudaMemcpyAsync(tproj_table_.get(), feat.data(), 256 * 4, cudaMemcpyHostToDevice, st_));
    auto run = [&](auto tag) {
        using T = decltype(tag);
        convert<T>(ctx_f32_.as<float>(), static_cast<long long>(S) * L * C, ctx_.as<T>(), st_);
        kv_all_impl<T>(S, L);
        broadcast_rows<T>(tproj_table_.as<float>(), S, 256, tproj_.as<T>(), st_);
        time_embed_impl<T>(tproj_.get(), S);
        block_modulation(tmod_.as<float>(), S, C, tables_.as<float>(), d_.n_blocks, mods_.as<float>(), st_);
        prologue_impl<T>(in_lat_.as<float>(), S, S, H, W);
        const size_t ckv_stride = static_cast<size_t>(S) * L * 2 * C;
        for (int b = 0; b < d_.n_blocks; ++b) {
            block_impl<T>(b, x_.as<float>(), x_.as<float>(), x_.as<float>(), x_.as<float>(), S, Tn, L,
                          mods_.as<float>() + static_cast<size_t>(b) * S * 6 * C, ckv_.as<T>() + b * ckv_stride,
                          bias ? bias_d_.as<float>() : nullptr, bias ? kvlen_.as<int>() : nullptr);
        }
        epilogue_impl<T>(S, Tn);
    };
    if (mode_ == kModeBf16) run(bf16{});
    else run(float{});
    std::vector<float> tok(static_cast<size_t>(S) * Tn * Cl);
    SANA_CUDA(cudaMemcpyAsync(tok.data(), noise_.get(), tok.size() * 4, cudaMemcpyDeviceToHost, st_));
    SANA_CUDA(cudaStreamSynchronize(st_));
    check_device_error();
    tokens_to_nchw_host(tok, S, Tn, Cl, noise);
}

void Engine::denoise_step(float* lat, int B, int H, int W, const float* ctx, int L, const float* bias, float guidance,
                          SchedulerHostState& state, float timestep, const SchedConfig& sc) {
    scheduler_validate(sc);
    SANA_REQUIRE(have_w_, "weights have not been uploaded");
    SANA_REQUIRE(state.sigmas.size() >= 2, "scheduler sigmas must have one extra final entry");
    SANA_REQUIRE(state.step_index >= 0 && state.step_index < static_cast<int>(state.sigmas.size()) - 1,
                 "scheduler step_index is out of range");
    const int S = 2 * B, Tn = H * W, C = d_.C, Cl = d_.Cl;
    ensure_workspace(S, Tn, L);
    const size_t n_lat = static_cast<size_t>(B) * Cl * Tn;
    const SchedCoef k = scheduler_coefficients(state.sigmas, state.step_index, state.lower_order_count, guidance, sc);
    if (k.second_order) {
        // the converted output of this step joins the history, capped at solver_order (2)
        SANA_REQUIRE(!state.history.empty() && state.history.back().size() == n_lat,
                     "second-order update requires two model outputs");
    }
    SANA_CUDA(cudaMemcpyAsync(lat_.get(), lat, n_lat * 4, cudaMemcpyHostToDevice, st_));
    if (k.second_order) {
        SANA_CUDA(cudaMemcpyAsync(hist_.as<float>() + n_lat, state.history.back().data(), n_lat * 4,
                                  cudaMemcpyHostToDevice, st_));
    }
    SANA_CUDA(cudaMemcpyAsync(ctx_f32_.get(), ctx, static_cast<size_t>(S) * L * C * 4, cudaMemcpyHostToDevice, st_));
    if (bias) {
        SANA_CUDA(cudaMemcpyAsync(bias_d_.get(), bias, static_cast<size_t>(S) * L * 4, cudaMemcpyHostToDevice, st_));
        caption_kv_len(bias_d_.as<float>(), S, L, kvlen_.as<int>(), st_);
    }
    std::vector<float> feat(256);
    timestep_features(timestep, feat.data());
    SANA_CUDA(cudaMemcpyAsync(tproj_table_.get(), feat.data(), 256 * 4, cudaMemcpyHostToDevice, st_));
    auto run = [&](auto tag) {
        using T = decltype(tag);
        convert<T>(ctx_f32_.as<float>(), static_cast<long long>(S) * L * C, ctx_.as<T>(), st_);
        kv_all_impl<T>(S, L);
        broadcast_rows<T>(tproj_table_.as<float>(), S, 256, tproj_.as<T>(), st_);
        time_embed_impl<T>(tproj_.get(), S);
        block_modulation(tmod_.as<float>(), S, C, tables_.as<float>(), d_.n_blocks, mods_.as<float>(), st_);
        prologue_impl<T>(lat_.as<float>(), B, S, H, W);
        const size_t ckv_stride = static_cast<size_t>(S) * L * 2 * C;
        for (int b = 0; b < d_.n_blocks; ++b) {
            block_impl<T>(b, x_.as<float>(), x_.as<float>(), x_.as<float>(), x_.as<float>(), S, Tn, L,
                          mods_.as<float>() + static_cast<size_t>(b) * S * 6 * C, ckv_.as<T>() + b * ckv_stride,
                          bias ? bias_d_.as<float>() : nullptr, bias ? kvlen_.as<int>() : nullptr);
        }
        epilogue_impl<T>(S, Tn);
        cfg_scheduler_step(noise_.as<float>(), B, Cl, Tn, lat_.as<float>(), hist_.as<float>(), hist_.as<float>() + n_lat,
                           k, st_);
    };
    if (mode_ == kModeBf16) run(bf16{});
    else run(float{});
    std::vector<float> x0(n_lat);
    SANA_CUDA(cudaMemcpyAsync(lat, lat_.get(), n_lat * 4, cudaMemcpyDeviceToHost, st_));
    SANA_CUDA(cudaMemcpyAsync(x0.data(), hist_.get(), n_lat * 4, cudaMemcpyDeviceToHost, st_));
    SANA_CUDA(cudaStreamSynchronize(st_));
    check_device_error();
    state.history.push_back(std::move(x0));
    while (state.history.size() > static_cast<size_t>(sc.solver_order)) state.history.erase(state.history.begin());
    if (state.lower_order_count < sc.solver_order) ++state.lower_order_count;
    ++state.step_index;
}

size_t Engine::debug_read(const std::string& name, size_t offset, size_t bytes, void* host) {
    const std::map<std::string, const DevBuf*> bufs = {
        {"a", &a_},       {"qkv", &qkv_},   {"ao", &ao_},     {"cq", &cq_},     {"xb", &xb_},
        {"ffh", &ffh_},   {"glu", &glu_},   {"x", &x_},       {"x1", &x1_},     {"x2", &x2_},
        {"x3", &x3_},     {"mods", &mods_}, {"tmod", &tmod_}, {"emb", &emb_},   {"ckv1", &ckv1_},
        {"ctx", &ctx_},   {"kvlen", &kvlen_}, {"noise", &noise_}, {"lat", &lat_}, {"part", &part_}};
    auto it = bufs.find(name);
    SANA_REQUIRE(it != bufs.end(), "unknown buffer " + name);
    const DevBuf& b = *it->second;
    if (host && bytes) {
        SANA_REQUIRE(offset + bytes <= b.bytes(), "read past the end of " + name);
        SANA_CUDA(cudaMemcpyAsync(host, static_cast<const char*>(b.get()) + offset, bytes, cudaMemcpyDeviceToHost,
                                  st_));
        SANA_CUDA(cudaStreamSynchronize(st_));
    }
    return b.bytes();
}

cudaEvent_t Engine::prof_event() {
    cudaEvent_t e;
    SANA_CUDA(cudaEventCreate(&e));
    ev_pool_.push_back(e);
    return e;
}

void Engine::profile_enable(bool on) {
    SANA_CUDA(cudaStreamSynchronize(st_));
    for (auto e : ev_pool_) cudaEventDestroy(e);
    ev_pool_.clear();
    prof_.clear();
    prof_on_ = on;
}

std::string Engine::profile_report() {
    SANA_CUDA(cudaStreamSynchronize(st_));
    std::map<std::string, std::pair<int, double>> agg;
    for (const auto& r : prof_) {
        float ms = 0.f;
        SANA_CUDA(cudaEventElapsedTime(&ms, r.a, r.b));
        auto& a = agg[r.name];
        a.first += 1;
        a.second += ms;
    }
    std::ostringstream o;
    o << "{";
    bool first = true;
    for (const auto& kv : agg) {
        o << (first ? "" : ", ") << '"' << kv.first << "\": [" << kv.second.first << ", " << kv.second.second << "]";
        first = false;
    }
    o << "}";
    return o.str();
}

void Engine::profile_loop_device(const float* lat, int B, int H, int W, const float* enc, int L, int Din,
                                 const float* bias, float guidance, int num_steps, const SchedConfig& sc, float* out) {
    SANA_REQUIRE(have_w_, "weights have not been uploaded");
    ensure_workspace(2 * B, H * W, L);
    std::vector<float> ts, sg;
    scheduler_schedule(num_steps, sc, ts, sg);
    const std::vector<SchedCoef> coefs = scheduler_loop_coefficients(sc, sg, guidance);
    std::vector<float> table(static_cast<size_t>(num_steps) * 256);
    for (int i = 0; i < num_steps; ++i) timestep_features(ts[i], table.data() + static_cast<size_t>(i) * 256);
    SANA_CUDA(cudaMemcpyAsync(tproj_table_.get(), table.data(), table.size() * 4, cudaMemcpyHostToDevice, st_));
    profile_enable(true);
    if (mode_ == kModeBf16) loop_body<bf16>(lat, B, H, W, enc, L, Din, bias, coefs, out);
    else loop_body<float>(lat, B, H, W, enc, L, Din, bias, coefs, out);
    SANA_CUDA(cudaStreamSynchronize(st_));
    prof_on_ = false;
}

}  // namespace sana
