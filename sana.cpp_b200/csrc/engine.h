// The Sana denoiser engine behind the C ABI: device weight cache, workspace, and the
// orchestration of block_forward / run_model_blocks / the denoising step and loop
// (transformer.cpp:544-778) over the kernels of gemm.h and kernels.h.
#pragma once

#include <map>
#include <string>
#include <vector>

#include "common.cuh"
#include "gemm.h"
#include "kernels.h"

namespace sana {

struct Dims {
    int n_blocks = 0, C = 0, Cl = 0, Din = 0, E = 0, Hs = 0, Hc = 0;
};

enum Mode : int { kModeBf16 = 0, kModeF32 = 1 };
enum Layout : int { kLayoutReference = 0, kLayoutTorch = 1 };

// One cudaMalloc'd region, freed on destruction.
class DevBuf {
   public:
    DevBuf() = default;
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    DevBuf(DevBuf&& o) noexcept : p_(o.p_), n_(o.n_) {
        o.p_ = nullptr;
        o.n_ = 0;
    }
    DevBuf& operator=(DevBuf&& o) noexcept {
        if (this != &o) {
            release();
            p_ = o.p_;
            n_ = o.n_;
            o.p_ = nullptr;
            o.n_ = 0;
        }
        return *this;
    }
    ~DevBuf() { release(); }
    void ensure(size_t bytes);  // grows (contents are not kept)
    void release();
    void* get() const { return p_; }
    template <class T> T* as() const { return static_cast<T*>(p_); }
    size_t bytes() const { return n_; }

   private:
    void* p_ = nullptr;
    size_t n_ = 0;
};

struct BlockWeights {
    DevBuf cqn, ckn;            // optional cross-attention q / k RMSNorm weights [C] f32 (empty = ones)
    DevBuf wqkv, bqkv;          // [3C, C] act type, [3C] f32
    DevBuf wo, bo;              // [C, C], [C]
    DevBuf wcq, bcq;            // [C, C], [C]
    DevBuf wckv, bckv;          // [2C, C], [2C]
    DevBuf wco, bco;            // [C, C], [C]
    DevBuf ln1g, ln1b, ln2g, ln2b;  // [C] f32 (empty = identity)
    DevBuf winv, binv;          // [E, C], [E]
    DevBuf wdw, bdw;            // [E, 9] f32, [E]
    DevBuf wpt;                 // [C, E/2]
};

// Scheduler state as the reference keeps it (SanaSchedulerState, scheduler.h:27-32),
// with the converted outputs on the host.
struct SchedulerHostState {
    std::vector<float> sigmas;   // n_steps + 1
    int step_index = 0;
    int lower_order_count = 0;
    std::vector<std::vector<float>> history;  // oldest first, <= 2
};

// SanaSchedulerConfig (scheduler.h:9-20) as the device path uses it: the string-valued
// fields the reference only compares against one accepted value (timestep_spacing,
// prediction_type, algorithm_type) are checked by the callers.
struct SchedConfig {
    int num_train_timesteps = 1000;
    float flow_shift = 3.0f;
    bool flow_sigmas = true;        // use_flow_sigmas
    int solver_order = 2;           // 1 or 2
    bool lower_order_final = true;
    bool final_sigmas_zero = true;  // final_sigmas_type == "zero"
    bool heun = false;              // solver_type: midpoint (false) or heun (true)
};
// validate_scheduler_config (scheduler.cpp:8-24) for the numeric fields.
void scheduler_validate(const SchedConfig& c);
// The order step_sana_scheduler takes at step i of n with lower_order_step_count `lower`
// (scheduler.cpp:291-311): 1 or 2.
int scheduler_step_order(const SchedConfig& c, int n_steps, int step_index, int lower_order_count);
// Host-side DPM-Solver++ coefficients of one step, computed with the reference's fp32
// arithmetic (scheduler.cpp:71-81, 175-270, 291-311).
SchedCoef scheduler_coefficients(const std::vector<float>& sigmas, int step_index, int lower_order_count,
                                 float guidance, const SchedConfig& c = SchedConfig());
// The same for an explicit order (1 or 2).
SchedCoef scheduler_coefficients_order(const std::vector<float>& sigmas, int step_index, int order, float guidance,
                                       const SchedConfig& c = SchedConfig());
// The coefficients of every step of a fresh state (init_sana_scheduler_state) run to the end.
std::vector<SchedCoef> scheduler_loop_coefficients(const SchedConfig& c, const std::vector<float>& sigmas,
                                                   float guidance);
// build_sana_scheduler_timesteps (scheduler.cpp:89-141).
void scheduler_schedule(int n, const SchedConfig& c, std::vector<float>& timesteps, std::vector<float>& sigmas);
void scheduler_schedule(int n, float flow_shift, std::vector<float>& timesteps, std::vector<float>& sigmas);
// timestep_embedding_2d for one timestep (transformer.cpp:77-122): [cos | sin], 256 wide.
void timestep_features(float t, float* out256);

class Engine {
   public:
    Engine(int device, int mode);
    ~Engine();

    int mode() const { return mode_; }
    const Dims& dims() const { return d_; }
    bool has_weights() const { return have_w_; }
    int last_launches() const { return last_launches_; }
    cudaStream_t stream() const { return st_; }
    void set_stream(cudaStream_t s) { st_ = s ? s : own_st_; }

    // model: 16 tensors, blocks: n_blocks x 26 (SanaBlockWeights field order); see sana_cuda.h.
    void upload(const Dims& d, const float* const* model, const float* const* blocks, int layout);

    // --- host-buffer entry points (the reference-facing API) ---------------------------
    void project_caption(const float* enc, int S, int L, int Din, float* out);
    // Timestep embedding and t_block for S sequences at host timesteps t[S]: emb [S, C] (the
    // final layer's modulation input) and tmod [S, 6C] to host buffers (either may be null).
    void time_embed(const float* t, int S, float* emb, float* tmod);
    void block_forward(int b, const float* x, int S, int T, const float* ctx, int L, const float* tmod,
                       const float* bias, float* after_self, float* after_cross, float* after_ff);
    void run_blocks(const float* x, int S, int T, const float* ctx, int L, const float* tmod, const float* bias,
                    int begin, int end, float* out);
    void forward_nocfg(const float* lat, int S, int H, int W, float t, const float* ctx, int L, const float* bias,
                       float* noise);
    void denoise_step(float* lat, int B, int H, int W, const float* ctx, int L, const float* bias, float guidance,
                      SchedulerHostState& state, float timestep, const SchedConfig& sc = SchedConfig());
    void denoise_loop(const float* lat, int B, int H, int W, const float* enc, int L, int Din, const float* bias,
                      float guidance, int num_steps, const SchedConfig& sc, float* out);
    // Device-pointer variant of denoise_loop (inputs already in HBM, fp32).
    void denoise_loop_device(const float* lat, int B, int H, int W, const float* enc, int L, int Din,
                             const float* bias, float guidance, int num_steps, const SchedConfig& sc, float* out);

    // Per-kernel profiling of eager (uncaptured) work: CUDA events around every launch of the
    // loop, summed per kernel class. enable() clears previous records.
    void profile_enable(bool on);
    std::string profile_report();  // JSON: {"kernel": [launches, total_ms], ...}
    // Runs the denoising loop once eagerly with profiling on (device pointers).
    void profile_loop_device(const float* lat, int B, int H, int W, const float* enc, int L, int Din,
                             const float* bias, float guidance, int num_steps, const SchedConfig& sc, float* out);

    // Read-back of a named workspace buffer (diagnostics): a, qkv, ao, cq, xb, ffh, glu,
    // x, x1, x2, x3, mods, tmod, emb, ckv1, ctx, kvlen, noise, lat. Returns its size.
    size_t debug_read(const std::string& name, size_t offset, size_t bytes, void* host);

    // Device-side error word (timeouts); checked and cleared after every host API call.
    void check_device_error();
    int* err() const { return err_.as<int>(); }
    // Optional RMSNorm of the cross-attention q and k projections over each token's C channels,
    // not part of the reference's block (off by default). q_w / k_w: n_blocks pointers to [C]
    // weights (NULL array or entries = ones).
    void set_cross_qk_norm(bool enable, const float* const* q_w, const float* const* k_w, float eps);
    // Time limit of every bounded device-side wait of this handle (common.cuh).
    void set_wait_limit_ns(unsigned long long ns);
    unsigned long long wait_limit_ns() const { return wait_limit_host_; }
    int num_sms() const { return num_sms_; }
    int device() const { return device_; }

    // Guidance split across two GPUs (cfgpair.cu), one process and handle per GPU:
    // pair_export allocates this GPU's exchange region for up to `capacity` latent elements and
    // writes its CUDA IPC handle (64 bytes) to `handle`; pair_connect maps the peer's region and
    // takes branch 0 (unconditional) or 1 (conditional); denoise_loop_pair_device runs the loop
    // of that branch (enc / bias hold its B sequences), meeting the peer once per step. Both
    // GPUs must run the same loops in the same order; after a timeout both export again.
    void pair_export(size_t capacity, void* handle);
    void pair_connect(int branch, const void* peer_handle);
    void pair_close();
    void denoise_loop_pair_device(const float* lat, int B, int H, int W, const float* enc, int L, int Din,
                                  const float* bias, float guidance, int num_steps, const SchedConfig& sc,
                                  float* out);

   private:
    template <class T> void upload_impl(const float* const* model, const float* const* blocks, int layout);
    template <class T> void caption_impl(const float* enc_d, int S, int L);
    template <class T> void kv_impl(int b, int S, int L, void* ckv_dst);
    template <class T> void kv_all_impl(int S, int L);
    template <class T>
    void block_impl(int b, const float* x_in, float* x_self, float* x_cross, float* x_ff, int S, int Tn, int L,
                    const float* mod_b, const void* ckv_b, const float* bias_d, const int* kvlen_d);
    template <class T> void time_embed_impl(const void* tproj_d, int S);
    template <class T> void prologue_impl(const float* lat_d, int images, int S, int H, int W);
    template <class T> void epilogue_impl(int S, int Tn);
    template <class T>
    void loop_body(const float* lat_in, int B, int H, int W, const float* enc_d, int L, int Din, const float* bias_d,
                   const std::vector<SchedCoef>& coefs, float* out_d);

    void ensure_workspace(int S, int T, int L);
    void gemm_act(const void* A, long long lda, const void* Bw, long long ldb, int M, int N, int K,
                  const Epilogue& ep, bool b_is_f32 = false);
    void run_loop(const float* lat_d, int B, int H, int W, const float* enc_d, int L, int Din, const float* bias_d,
                  float guidance, int num_steps, const SchedConfig& sc, float* out_d, const std::string& key_extra);
    size_t act_size() const { return mode_ == kModeBf16 ? 2 : 4; }

    int device_ = 0, mode_ = 0, num_sms_ = 148;
    cudaStream_t own_st_ = nullptr, st_ = nullptr;
    Dims d_;
    bool have_w_ = false;
    int last_launches_ = 0;
    DevBuf err_;
    unsigned long long wait_limit_host_ = 0;  // host copy of the limit in err_ (pinned by value)
    bool cross_qk_norm_ = false;
    float cross_qk_eps_ = 1e-6f;

    // two-GPU guidance: this GPU's region [flags | counts | 2 receive buffers], the peer's
    // mapping, the branch, and whether the loop being recorded runs one branch
    void* pair_region_ = nullptr;
    long long pair_cap_ = 0;
    void* pair_peer_ = nullptr;
    int pair_branch_ = -1;
    bool pair_run_ = false;
    PairLink pair_link() const;

    // weights
    DevBuf cap_w1_, cap_b1_, cap_w2_, cap_b2_, cap_norm_;
    DevBuf patch_w_, patch_b_, te_w1_, te_b1_, te_w2_, te_b2_, tp_w_, tp_b_;
    DevBuf ftable_, out_w_, out_b_, tables_;
    std::vector<BlockWeights> blk_;

    // workspace (sized by ensure_workspace)
    int ws_S_ = 0, ws_T_ = 0, ws_L_ = 0;
    DevBuf x_, x1_, x2_, x3_, xb_, a_, qkv_, ao_, cq_, ffh_, glu_, part_, y_, noise_, pt_;
    DevBuf ctx_, ctx_f32_, caph_, capp_, enc_t_, ckv_, ckv1_;
    DevBuf tproj_, teh_, emb_, embs_, tmod_, mods_, fmod_;
    DevBuf bias_d_, kvlen_, lat_, hist_, in_lat_, in_enc_, in_bias_, in_x_, in_tmod_, out_buf_;
    DevBuf tproj_table_;

    // captured loops
    struct GraphEntry {
        cudaGraphExec_t exec = nullptr;
        int launches = 0;
        int calls = 0;
    };
    std::map<std::string, GraphEntry> graphs_;

    // profiling
    friend class ProfScope;
    bool prof_on_ = false;
    struct ProfRec {
        std::string name;
        cudaEvent_t a, b;
    };
    std::vector<ProfRec> prof_;
    std::vector<cudaEvent_t> ev_pool_;
    cudaEvent_t prof_event();
};

// Records CUDA events around the launches in its scope when the engine profiles.
class ProfScope {
   public:
    ProfScope(Engine* e, const char* name) : e_(e) {
        if (e_->prof_on_) {
            rec_.name = name;
            rec_.a = e_->prof_event();
            rec_.b = e_->prof_event();
            cudaEventRecord(rec_.a, e_->st_);
        }
    }
    ~ProfScope() {
        if (e_->prof_on_) {
            cudaEventRecord(rec_.b, e_->st_);
            e_->prof_.push_back(rec_);
        }
    }

   private:
    Engine* e_;
    Engine::ProfRec rec_{};
};

}  // namespace sana
