// C ABI of the engine: initialize / use_model and friends (include/rosenna.h).
//
// initialize() reads the three model files, builds the launch plan and uploads
// the packed weights to every selected GPU.  use_model splits the batch into
// contiguous sample ranges, one per GPU (one host thread each), and runs the
// plan on chunks of samples: host->device copies of a chunk's rows, the plan's
// kernels, device->host copies, with four streams taking chunks in turn so that
// the copies of some chunks overlap the kernels of others.  No collective is
// involved: samples are independent and weights are replicated.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/rosenna.h"
#include "conv_tc.cuh"
#include "kernels.cuh"
#include "mlp_tc.cuh"
#include "model_files.hpp"
#include "plan.hpp"

namespace rosenna {
namespace {

constexpr int kSlots = 4;  // chunk streams (four ran the small MLP 4.6 % faster end to end than three)
constexpr int kLegacyArgs = 16;  // arrays the fixed-shape use_model symbol takes

struct Slot {
    cudaStream_t stream = nullptr;
    cudaEvent_t done = nullptr;     // last device-path use of this slot's scratch
    int64_t cap = 0;                // samples the scratch buffers hold
    std::vector<float *> scratch;   // per plan buffer (intermediates only)
    std::vector<float *> io;        // per plan buffer: device copies of inputs/outputs (host path)
    int64_t io_cap = 0;
    float *mid = nullptr;           // conv_pair_tc_kernel's per-CTA buffer (fused conv pairs only)
    int64_t mid_cols = 0;
};

struct Device {
    int id = 0;
    int num_sms = 148;
    float *arena = nullptr;
    int *err = nullptr;       // tensor-core kernel status word (0 = ok)
    int *err_host = nullptr;  // pinned copy, refreshed at the end of each call that ran a tensor-core kernel
    std::vector<TcArgs> tc_args;  // per plan step (tensor-core MLP steps only)
    std::vector<TcLstmArgs> lstm_args;  // per plan step (tensor-core LSTM steps only)
    std::vector<TcLstm2Args> lstm2_args;  // per plan step (first step of a fused LSTM pair only)
    Slot slots[kSlots];
    // allocation-free entry point: device address of the fixed scratch array,
    // looked up at initialize (or why it could not be)
    void *noalloc_base = nullptr;
    std::string noalloc_err;
    // per-step timing (rosenna_step_timing_begin/end): event pairs, the plan
    // step each recorded pair belongs to, pairs used so far
    std::vector<cudaEvent_t> tev;
    std::vector<int> tev_step;
    int64_t tev_used = 0;
};

struct Context {
    bool ready = false;
    ModelFiles mf;
    Plan plan;
    std::string desc;
    std::vector<int> device_ids;  // selected by rosenna_set_devices (empty: all)
    std::vector<std::unique_ptr<Device>> devs;
    std::vector<MlpLayerDev> mlp_tables;       // host copies, concatenated
    std::vector<int64_t> mlp_table_off;        // per step: index into mlp_tables, device offset in arena
    std::vector<int64_t> mlp_table_arena_off;
    std::vector<bool> is_io_in, is_io_out;
    int conv_group = 4;  // tensor-core conv unit order: sample tiles per block group (ROSENNA_CONV_GROUP)
    int64_t mid_rows = 0;  // rows of the largest fused conv pair's intermediate (0: no fused pair)
    int64_t scratch_budget = 0;  // measure_scratch_budget() at initialize
};

Context g_ctx;
std::mutex g_mu;
int g_status = 0;
std::string g_error;
std::atomic<int64_t> g_launches{0};

int fail(int code, const std::string &msg) {
    g_status = code;
    g_error = msg;
    return code;
}
int ok() {
    g_status = 0;
    g_error.clear();
    return 0;
}

#define CUDA_TRY(expr)                                                                                         \
    do {                                                                                                       \
        cudaError_t e_ = (expr);                                                                               \
        if (e_ != cudaSuccess)                                                                                 \
            return Status::Err(ROSENNA_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(e_));          \
    } while (0)

// Bytes of intermediates a call may allocate: a quarter of the device memory
// free at initialize, at most 16 GB.  Measured once (cudaMemGetInfo is a call
// into the kernel driver, which can wait behind other processes' driver work
// on a shared machine: made on every call it left the GPU idle for
// milliseconds at a time).
int64_t measure_scratch_budget() {
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) return (int64_t)4 << 30;
    return (int64_t)std::min<size_t>(free_b / 4, (size_t)16 << 30);
}
int64_t scratch_budget_bytes() { return g_ctx.scratch_budget > 0 ? g_ctx.scratch_budget : (int64_t)4 << 30; }

void release_device(Device &d) {
    cudaSetDevice(d.id);
    for (auto &s : d.slots) {
        for (auto p : s.scratch) cudaFree(p);
        for (auto p : s.io) cudaFree(p);
        if (s.mid) cudaFree(s.mid);
        s.mid = nullptr;
        s.mid_cols = 0;
        s.scratch.clear();
        s.io.clear();
        s.cap = s.io_cap = 0;
        if (s.stream) cudaStreamDestroy(s.stream);
        if (s.done) cudaEventDestroy(s.done);
        s.stream = nullptr;
        s.done = nullptr;
    }
    for (auto e : d.tev) cudaEventDestroy(e);
    d.tev.clear();
    d.tev_step.clear();
    d.tev_used = 0;
    d.noalloc_base = nullptr;
    cudaFree(d.arena);
    cudaFree(d.err);
    if (d.err_host) cudaFreeHost(d.err_host);
    d.arena = nullptr;
    d.err = nullptr;
    d.err_host = nullptr;
}

void release_all() {
    int cur = 0;
    cudaGetDevice(&cur);
    for (auto &d : g_ctx.devs) release_device(*d);
    g_ctx.devs.clear();
    g_ctx.ready = false;
    cudaSetDevice(cur);
}

// intermediate buffers: used by a step and not a model input/output
bool is_scratch(int b) { return !g_ctx.is_io_in[(size_t)b] && !g_ctx.is_io_out[(size_t)b]; }

// Buffers the plan's launches touch.  A fused LSTM pair never writes the first
// layer's output sequence (the second layer reads it from shared memory).
std::vector<bool> used_buffers() {
    const Plan &P = g_ctx.plan;
    std::vector<bool> used(P.buf_rows.size(), false);
    for (size_t si = 0; si < P.steps.size(); si++) {
        const Step &st = P.steps[si];
        // (a fused conv pair keeps its intermediate: the two-kernel path takes
        // calls the pair kernel cannot)
        const bool skip_y = st.kind == Step::LSTM && st.fuse_next;
        const bool skip_in = si > 0 && P.steps[si - 1].kind == Step::LSTM && P.steps[si - 1].fuse_next;
        for (int b : {st.in, st.out, st.h0, st.c0, st.y, st.hn, st.cn}) {
            if (b < 0 || (skip_y && b == st.y) || (skip_in && b == st.in)) continue;
            used[(size_t)b] = true;
        }
    }
    return used;
}

Status ensure_scratch(Slot &s, int64_t cap) {
    if (s.cap >= cap) return Status::Ok();
    for (auto p : s.scratch) cudaFree(p);
    s.scratch.assign(g_ctx.plan.buf_rows.size(), nullptr);
    s.cap = 0;
    const std::vector<bool> used = used_buffers();
    for (size_t b = 0; b < used.size(); b++) {
        if (!used[b] || !is_scratch((int)b)) continue;
        CUDA_TRY(cudaMalloc(&s.scratch[b], sizeof(float) * (size_t)g_ctx.plan.buf_rows[b] * (size_t)cap));
    }
    s.cap = cap;
    return Status::Ok();
}

// conv_pair_tc_kernel's buffer: 256 sample columns per SM of the largest
// fused pair's intermediate rows.
Status ensure_mid(Slot &s, int num_sms) {
    const int64_t cols = (int64_t)num_sms * kConvPairMidPerCta;
    if (g_ctx.mid_rows <= 0 || s.mid_cols >= cols) return Status::Ok();
    if (s.mid) cudaFree(s.mid);
    s.mid = nullptr;
    s.mid_cols = 0;
    CUDA_TRY(cudaMalloc(&s.mid, sizeof(float) * (size_t)g_ctx.mid_rows * (size_t)cols));
    s.mid_cols = cols;
    return Status::Ok();
}

Status ensure_io(Slot &s, int64_t cap) {
    if (s.io_cap >= cap) return Status::Ok();
    for (auto p : s.io) cudaFree(p);
    s.io.assign(g_ctx.plan.buf_rows.size(), nullptr);
    s.io_cap = 0;
    for (auto *v : {&g_ctx.plan.inputs, &g_ctx.plan.outputs})
        for (auto &io : *v)
            CUDA_TRY(cudaMalloc(&s.io[(size_t)io.buf], sizeof(float) * (size_t)io.rows * (size_t)cap));
    s.io_cap = cap;
    return Status::Ok();
}

// Largest chunk whose intermediates fit the scratch budget.
int64_t max_chunk(int64_t n) {
    int64_t rows = 0;
    const std::vector<bool> used = used_buffers();
    for (size_t b = 0; b < g_ctx.plan.buf_rows.size(); b++)
        if (used[b] && is_scratch((int)b)) rows += g_ctx.plan.buf_rows[b];
    int64_t cap = n;
    if (rows > 0) cap = std::max<int64_t>(1024, scratch_budget_bytes() / (int64_t)(sizeof(float) * rows));
    return std::max<int64_t>(1, std::min(cap, n));
}

// Runs the plan on `cnt` samples.  ptr[b]/ld[b] address buffer b (row r of
// sample s at ptr[b][r*ld[b] + s]).
// `mid`: the slot's conv_pair_tc_kernel buffer, or null (fused conv pairs then
// run as two kernels).
Status run_plan(Device &d, const std::vector<float *> &ptr, const std::vector<int64_t> &ld, int64_t cnt,
                cudaStream_t stream, const Slot *mid) {
    const Plan &P = g_ctx.plan;
    const float *arena = d.arena;
    int64_t launches = 0;
    bool tc_ran = false;  // a tensor-core kernel ran: refresh the pinned status copy once, after the last step
    for (size_t si = 0; si < P.steps.size(); si++) {
        const Step &s = P.steps[si];
        cudaError_t e = cudaSuccess;
        bool pair_ran = false;  // this step and the next ran as one kernel
        const bool timed = d.tev_used < (int64_t)d.tev_step.size();
        if (timed && cudaEventRecord(d.tev[(size_t)(2 * d.tev_used)], stream) != cudaSuccess)
            return Status::Err(ROSENNA_ERR_CUDA, "cudaEventRecord (step timing) failed");
        switch (s.kind) {
            case Step::MLP: {
                if (s.tc) {
                    TcArgs a = d.tc_args[si];
                    for (int t = 0; t < s.rsub && e == cudaSuccess; t++) {
                        a.in = ptr[(size_t)s.in] + (int64_t)t * ld[(size_t)s.in];
                        a.ld_in = (int64_t)s.rsub * ld[(size_t)s.in];
                        a.out = ptr[(size_t)s.out] + (int64_t)t * ld[(size_t)s.out];
                        a.ld_out = (int64_t)s.rsub * ld[(size_t)s.out];
                        a.n = cnt;
                        if (a.narrow) {
                            e = launch_mlp_narrow(a, d.num_sms, stream);
                        } else if (a.stream) {
                            e = launch_mlp_stream(a, d.num_sms, stream);
                            if (e == cudaErrorNotSupported) e = launch_mlp_tc(a, d.num_sms, stream);  // unaligned input
                        } else {
                            e = launch_mlp_tc(a, d.num_sms, stream);
                        }
                        launches++;
                    }
                    tc_ran = true;
                    break;
                }
                MlpArgs a{};
                a.arena = arena;
                a.layers = reinterpret_cast<const MlpLayerDev *>(arena + g_ctx.mlp_table_arena_off[si]);
                a.nlayers = (int)s.layers.size();
                const MlpLayerDev *host_layers = g_ctx.mlp_tables.data() + g_ctx.mlp_table_off[si];
                for (int t = 0; t < s.rsub; t++) {  // sub-row t: rows t + rsub*k
                    a.in = ptr[(size_t)s.in] + (int64_t)t * ld[(size_t)s.in];
                    a.ld_in = (int64_t)s.rsub * ld[(size_t)s.in];
                    a.out = ptr[(size_t)s.out] + (int64_t)t * ld[(size_t)s.out];
                    a.ld_out = (int64_t)s.rsub * ld[(size_t)s.out];
                    a.n = cnt;
                    e = launch_mlp(a, host_layers, d.num_sms, stream);
                    launches++;
                    if (e != cudaSuccess) break;
                }
                break;
            }
            case Step::LSTM: {
                if (s.fuse_next) {
                    const Step &s2 = P.steps[si + 1];
                    TcLstm2Args &a = d.lstm2_args[si];
                    a.x = ptr[(size_t)s.in];
                    a.ld_x = ld[(size_t)s.in];
                    const Step *ls[2] = {&s, &s2};
                    for (int k = 0; k < 2; k++) {
                        const Step &q = *ls[k];
                        a.h0[k] = q.h0 >= 0 ? ptr[(size_t)q.h0] : nullptr;
                        a.ld_h0[k] = q.h0 >= 0 ? ld[(size_t)q.h0] : 0;
                        a.c0[k] = q.c0 >= 0 ? ptr[(size_t)q.c0] : nullptr;
                        a.ld_c0[k] = q.c0 >= 0 ? ld[(size_t)q.c0] : 0;
                        a.hn[k] = q.hn >= 0 ? ptr[(size_t)q.hn] : nullptr;
                        a.ld_hn[k] = q.hn >= 0 ? ld[(size_t)q.hn] : 0;
                        a.cn[k] = q.cn >= 0 ? ptr[(size_t)q.cn] : nullptr;
                        a.ld_cn[k] = q.cn >= 0 ? ld[(size_t)q.cn] : 0;
                    }
                    a.y2 = s2.y >= 0 ? ptr[(size_t)s2.y] : nullptr;
                    a.ld_y2 = s2.y >= 0 ? ld[(size_t)s2.y] : 0;
                    a.n = cnt;
                    e = launch_lstm2_tc(a, d.num_sms, stream);
                    launches++;
                    tc_ran = true;
                    break;
                }
                if (s.tc) {
                    TcLstmArgs a = d.lstm_args[si];
                    a.x = ptr[(size_t)s.in];
                    a.ld_x = ld[(size_t)s.in];
                    a.h0 = nullptr;
                    a.c0 = nullptr;
                    a.y = a.hn = a.cn = nullptr;
                    if (s.h0 >= 0) { a.h0 = ptr[(size_t)s.h0]; a.ld_h0 = ld[(size_t)s.h0]; }
                    if (s.c0 >= 0) { a.c0 = ptr[(size_t)s.c0]; a.ld_c0 = ld[(size_t)s.c0]; }
                    if (s.y >= 0) { a.y = ptr[(size_t)s.y]; a.ld_y = ld[(size_t)s.y]; }
                    if (s.hn >= 0) { a.hn = ptr[(size_t)s.hn]; a.ld_hn = ld[(size_t)s.hn]; }
                    if (s.cn >= 0) { a.cn = ptr[(size_t)s.cn]; a.ld_cn = ld[(size_t)s.cn]; }
                    a.n = cnt;
                    e = s.lstm_dual ? launch_lstm_dual_tc(a, d.num_sms, stream) : launch_lstm_tc(a, d.num_sms, stream);
                    launches++;
                    tc_ran = true;
                    break;
                }
                LstmArgs a{};
                a.arena = arena;
                a.w_off = s.w_off;
                a.b_off = s.b_off;
                a.h0_const = s.h0_const;
                a.c0_const = s.c0_const;
                a.x = ptr[(size_t)s.in];
                a.ld_x = ld[(size_t)s.in];
                if (s.h0 >= 0) { a.h0 = ptr[(size_t)s.h0]; a.ld_h0 = ld[(size_t)s.h0]; }
                if (s.c0 >= 0) { a.c0 = ptr[(size_t)s.c0]; a.ld_c0 = ld[(size_t)s.c0]; }
                if (s.y >= 0) { a.y = ptr[(size_t)s.y]; a.ld_y = ld[(size_t)s.y]; }
                if (s.hn >= 0) { a.hn = ptr[(size_t)s.hn]; a.ld_hn = ld[(size_t)s.hn]; }
                if (s.cn >= 0) { a.cn = ptr[(size_t)s.cn]; a.ld_cn = ld[(size_t)s.cn]; }
                a.n = cnt;
                a.T = s.T;
                a.I = s.I;
                a.H = s.H;
                a.Ip = s.Ip;
                a.Hp = s.Hp;
                e = launch_lstm(a, d.num_sms, stream);
                launches++;
                break;
            }
            case Step::CONV: {
                // the tensor-core conv reads its input and writes its output
                // through TMA maps: 16-byte aligned bases and sample pitches
                // (otherwise the CUDA-core kernel below takes the call)
                const auto tc_io_ok = [&](const Step &q) {
                    return conv_tc_input_ok(ptr[(size_t)q.in], ld[(size_t)q.in]) &&
                           conv_tc_input_ok(ptr[(size_t)q.out], ld[(size_t)q.out]);
                };
                const auto tc_args = [&](const Step &q, ConvTcArgs &a) -> Status {
                    a = ConvTcArgs{};
                    a.arena = arena;
                    a.bt_off = q.ctc_off;
                    a.b_off = q.b_off;
                    a.out = ptr[(size_t)q.out];
                    a.ld_out = ld[(size_t)q.out];
                    a.so_c = q.so_c; a.so_h = q.so_h; a.so_w = q.so_w;
                    a.n = cnt;
                    a.err = d.err;
                    a.C = q.C; a.Hin = q.Hin; a.Win = q.Win; a.pad = q.pad_h; a.OC = q.OC;
                    a.Ho = q.Ho; a.Wo = q.Wo; a.Hq = q.Hq; a.Wq = q.Wq; a.pool = q.pool; a.relu = q.relu ? 1 : 0;
                    const ConvTcGeom geo = conv_tc_geometry(q.C, q.OC);
                    a.ocp = geo.ocp; a.bh = geo.bh; a.cb = geo.cb; a.ph = geo.ph; a.cw = geo.cw;
                    a.rows = geo.rows; a.slots = geo.slots;
                    a.group = g_ctx.conv_group;
                    const char *why = nullptr;
                    if (!conv_tc_encode_input(a, ptr[(size_t)q.in], ld[(size_t)q.in], &why))
                        return Status::Err(ROSENNA_ERR_CUDA, std::string("conv_tc input map: ") + (why ? why : "?"));
                    if (!conv_tc_encode_output(a, &why))
                        return Status::Err(ROSENNA_ERR_CUDA, std::string("conv_tc output map: ") + (why ? why : "?"));
                    return Status::Ok();
                };
                // this conv and the next one as conv_pair_tc_kernel, its
                // output passing through the slot's small per-CTA buffer
                if (s.fuse_next && mid && mid->mid && si + 1 < P.steps.size() && s.tc && P.steps[si + 1].tc &&
                    tc_io_ok(s) && tc_io_ok(P.steps[si + 1])) {
                    const Step &s2 = P.steps[si + 1];
                    ConvTcArgs a1, a2;
                    Status st = tc_args(s, a1);
                    if (st.ok()) st = tc_args(s2, a2);
                    if (!st.ok()) return st;
                    const char *why = nullptr;
                    e = launch_conv_pair(a1, s.ctc_packed_off, a2, mid->mid, mid->mid_cols, d.num_sms, stream, &why);
                    if (e != cudaSuccess && why)
                        return Status::Err(ROSENNA_ERR_CUDA, std::string(why) + ": " + cudaGetErrorString(e));
                    launches++;
                    tc_ran = true;
                    pair_ran = true;
                    break;
                }
                if (s.tc && tc_io_ok(s)) {
                    ConvTcArgs a;
                    Status st = tc_args(s, a);
                    if (!st.ok()) return st;
                    e = launch_conv_tc(a, d.num_sms, stream);
                    launches++;
                    tc_ran = true;
                    break;
                }
                ConvArgs a{};
                a.arena = arena;
                a.w_off = s.w_off;
                a.b_off = s.b_off;
                a.in = ptr[(size_t)s.in];
                a.ld_in = ld[(size_t)s.in];
                a.out = ptr[(size_t)s.out];
                a.ld_out = ld[(size_t)s.out];
                a.n = cnt;
                a.conv = s.conv;
                a.relu = s.relu;
                a.C = s.C; a.Hin = s.Hin; a.Win = s.Win; a.OC = s.OC; a.KS = s.KS;
                a.pad_h = s.pad_h; a.pad_w = s.pad_w; a.str_h = s.str_h; a.str_w = s.str_w;
                a.Ho = s.Ho; a.Wo = s.Wo;
                a.pool = s.pool; a.pk = s.pk; a.ppad_h = s.ppad_h; a.ppad_w = s.ppad_w;
                a.pstr_h = s.pstr_h; a.pstr_w = s.pstr_w; a.Hq = s.Hq; a.Wq = s.Wq;
                a.so_c = s.so_c; a.so_h = s.so_h; a.so_w = s.so_w;
                e = launch_conv(a, stream);
                launches++;
                break;
            }
            case Step::GATHER:
            case Step::COPY: {
                const int *map = s.kind == Step::GATHER ? reinterpret_cast<const int *>(arena + s.map_off) : nullptr;
                e = launch_gather(ptr[(size_t)s.in], ld[(size_t)s.in], ptr[(size_t)s.out], ld[(size_t)s.out], map,
                                  P.buf_rows[(size_t)s.out], cnt, stream);
                launches++;
                break;
            }
            case Step::DEINTERLEAVE:
                e = launch_deinterleave(ptr[(size_t)s.in], ld[(size_t)s.in], ptr[(size_t)s.out], ld[(size_t)s.out],
                                        (int)s.pre, P.buf_rows[(size_t)s.out], cnt, stream);
                launches++;
                break;
            case Step::ACT:
            case Step::ADD:
                e = launch_act(ptr[(size_t)s.in], ld[(size_t)s.in], ptr[(size_t)s.out], ld[(size_t)s.out],
                               P.buf_rows[(size_t)s.out], cnt, s.act, s.kind == Step::ADD ? arena + s.b_off : nullptr,
                               stream);
                launches++;
                break;
        }
        if (e != cudaSuccess)
            return Status::Err(ROSENNA_ERR_CUDA, std::string("kernel launch failed: ") + cudaGetErrorString(e));
        if (timed) {
            if (cudaEventRecord(d.tev[(size_t)(2 * d.tev_used + 1)], stream) != cudaSuccess)
                return Status::Err(ROSENNA_ERR_CUDA, "cudaEventRecord (step timing) failed");
            d.tev_step[(size_t)d.tev_used++] = (int)si;
        }
        if ((s.kind == Step::LSTM && s.fuse_next) || pair_ran) si++;  // the next step ran inside the fused kernel
    }
    if (tc_ran && cudaMemcpyAsync(d.err_host, d.err, 64 * sizeof(int), cudaMemcpyDeviceToHost, stream) != cudaSuccess)
        return Status::Err(ROSENNA_ERR_CUDA, "status word copy failed");
    g_launches += launches;
    return Status::Ok();
}

// A tensor-core kernel that timed out leaves a code in its status word; the
// engine then refuses further calls until it is initialized again.
std::string tc_error_text(const int *e) {
    char buf[768];
    int k = snprintf(buf, sizeof buf,
                     "a tensor-core kernel timed out waiting on its pipeline (wait %d, block %d, thread %d, at 0x%x, "
                     "parity %d, counters %d %d)",
                     e[0], e[1], e[2], e[3], e[4], e[5], e[6]);
    static const char *role[] = {"", "tma", "mma", "conv0", "conv1"};
    for (int r = 1; r <= 4 && k < (int)sizeof buf; r++) {
        const int *s = e + 8 * r;
        if (s[0] == 0 && s[1] == 0 && s[3] == 0) continue;
        k += snprintf(buf + k, sizeof buf - (size_t)k, "; %s: wait %d at 0x%x parity %d counters %d %d%s", role[r], s[0],
                      s[1], s[2], s[3], s[4], s[5] ? " (timed out)" : "");
    }
    return buf;
}

Status check_device_status() {
    for (auto &d : g_ctx.devs)
        if (d->err_host && *(volatile int *)d->err_host)
            return Status::Err(ROSENNA_ERR_CUDA, tc_error_text(d->err_host) + "; re-run initialize()");
    return Status::Ok();
}

Status check_batch(int64_t n) {
    if (n < 0) return Status::Err(ROSENNA_ERR_ARG, "negative batch size");
    Status st = check_device_status();
    if (!st.ok()) return st;
    // inputs whose batch index is not the first are de-interleaved on the
    // device; an output of that form (e.g. (N*T, H) from a Reshape that merges
    // the batch into another dimension) mixes samples: only n == 1 runs
    for (auto &io : g_ctx.plan.outputs)
        if (io.pre > 1 && n != 1)
            return Status::Err(ROSENNA_ERR_UNSUPPORTED,
                               "an output merges the batch into another dimension; only n == 1 runs");
    return Status::Ok();
}

Device *device_by_id(int id) {
    for (auto &d : g_ctx.devs)
        if (d->id == id) return d.get();
    return nullptr;
}

// Host path on one device: samples [a, b) of arrays with batch n.
Status host_range(Device &d, int64_t n, int64_t a, int64_t b, const float *const *in, float *const *out) {
    CUDA_TRY(cudaSetDevice(d.id));
    const Plan &P = g_ctx.plan;
    const int64_t total = b - a;
    if (total <= 0) return Status::Ok();
    // Chunks rotate over the slots' streams, so one chunk's copies overlap the
    // others' kernels.  The first chunk's H2D and the last one's D2H are not
    // hidden, and every chunk costs a few microseconds of launches: about
    // sqrt(I/O bytes / 440 KB) chunks (4..64, >= 16384 samples each, at most
    // 2^20) balances the two (440 KB ~ 8 us of PCIe at 55 GB/s).
    int64_t chunk = std::min<int64_t>(max_chunk(total), (int64_t)1 << 20);
    double io_bytes = 0;
    for (auto *v : {&P.inputs, &P.outputs})
        for (auto &io : *v) io_bytes += 4.0 * (double)io.rows * (double)total;
    const int64_t nch = std::min<int64_t>(64, std::max<int64_t>(4, std::llround(std::sqrt(io_bytes / 440e3))));
    chunk = std::min(chunk, std::max<int64_t>(16384, (total + nch - 1) / nch));
    chunk = (chunk + 31) / 32 * 32;
    for (int k = 0; k < kSlots; k++) {
        Status st = ensure_scratch(d.slots[k], std::min(chunk, total));
        if (!st.ok()) return st;
        if (!(st = ensure_mid(d.slots[k], d.num_sms)).ok()) return st;
        if (!(st = ensure_io(d.slots[k], std::min(chunk, total))).ok()) return st;
    }
    int64_t ci = 0;
    for (int64_t c0 = a; c0 < b; c0 += chunk, ci++) {
        Slot &s = d.slots[ci % kSlots];
        const int64_t cnt = std::min(chunk, b - c0);
        std::vector<float *> ptr(P.buf_rows.size(), nullptr);
        std::vector<int64_t> ld(P.buf_rows.size(), 0);
        for (size_t bi = 0; bi < ptr.size(); bi++) {
            ptr[bi] = s.io.empty() || !s.io[bi] ? s.scratch[bi] : s.io[bi];
            ld[bi] = s.io.empty() || !s.io[bi] ? s.cap : s.io_cap;
        }
        for (size_t i = 0; i < P.inputs.size(); i++) {
            // rows of `pre` interleaved samples' elements (pre = 1: rows of samples)
            const IoDesc &io = P.inputs[i];
            const size_t pre = (size_t)io.pre;
            CUDA_TRY(cudaMemcpy2DAsync(s.io[(size_t)io.buf], sizeof(float) * pre * (size_t)s.io_cap, in[i] + pre * c0,
                                       sizeof(float) * pre * (size_t)n, sizeof(float) * pre * (size_t)cnt,
                                       (size_t)io.rows / pre, cudaMemcpyHostToDevice, s.stream));
        }
        Status st = run_plan(d, ptr, ld, cnt, s.stream, &s);
        if (!st.ok()) return st;
        for (size_t i = 0; i < P.outputs.size(); i++) {
            const IoDesc &io = P.outputs[i];
            CUDA_TRY(cudaMemcpy2DAsync(out[i] + c0, sizeof(float) * (size_t)n, s.io[(size_t)io.buf],
                                       sizeof(float) * (size_t)s.io_cap, sizeof(float) * (size_t)cnt, (size_t)io.rows,
                                       cudaMemcpyDeviceToHost, s.stream));
        }
    }
    for (auto &s : d.slots) CUDA_TRY(cudaStreamSynchronize(s.stream));
    CUDA_TRY(cudaGetLastError());
    if (d.err_host && *(volatile int *)d.err_host) return Status::Err(ROSENNA_ERR_CUDA, tc_error_text(d.err_host));
    return Status::Ok();
}

// ---------------------------------------------------------------------------
// Allocation-free use_model on device arrays (rosenna_use_model_device_noalloc_f32).
//
// Some callers cannot have the library allocate device memory while they run:
// a solver that hands all free GPU memory to its own pool allocator at start-up
// (cudaMalloc would then fail), or a time-step loop that must not stall, since
// cudaMalloc/cudaFree synchronise the device.  rosenna_use_model_device_f32
// allocates its intermediate buffers on first use; that entry point instead
// carves them from one fixed array in device memory that every GPU loading
// this library holds until the process exits.  Its address is looked up in
// initialize(), once per selected device with that device current: with lazy
// module loading (the CUDA default) that lookup is what loads this file's
// device module and so creates the array, which therefore happens at
// initialize, not inside the first allocation-free call.
// ---------------------------------------------------------------------------
constexpr size_t kNoAllocScratchBytes = (size_t)64 << 20;  // 64 MiB per GPU

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

void noalloc_setup(Device &d) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
        d.noalloc_base = nullptr;
        d.noalloc_err = std::string("cudaGetSymbolAddress(scratch) at initialize: ") + cudaGetErrorString(e);
        cudaGetLastError();
        return;
    }
    d.noalloc_base = p;
    d.noalloc_err.clear();
}

Status do_initialize(const std::string &model, const std::string &weights, const std::string &vars) {
    release_all();
    g_ctx.mf = ModelFiles();
    Status st = read_model_files(model, weights, vars, &g_ctx.mf);
    if (!st.ok()) return st;
    if (!(st = build_plan(g_ctx.mf, &g_ctx.plan)).ok()) return st;
    Plan &P = g_ctx.plan;
    // layer tables of the MLP steps go into the arena too
    g_ctx.mlp_tables.clear();
    g_ctx.mlp_table_off.assign(P.steps.size(), -1);
    g_ctx.mlp_table_arena_off.assign(P.steps.size(), -1);
    for (size_t i = 0; i < P.steps.size(); i++) {
        const Step &s = P.steps[i];
        if (s.kind != Step::MLP) continue;
        if ((int)s.layers.size() > kMaxMlpLayers) return Status::Err(ROSENNA_ERR_UNSUPPORTED, "MLP chain longer than 24 layers");
        g_ctx.mlp_table_off[i] = (int64_t)g_ctx.mlp_tables.size();
        std::vector<MlpLayerDev> t;
        for (auto &l : s.layers) t.push_back(MlpLayerDev{l.K, l.M, l.Kp, l.Mp, l.act, 0, l.w_off, l.b_off});
        int S = 0;
        if (!mlp_smem_bytes(t.data(), (int)t.size(), &S))
            return Status::Err(ROSENNA_ERR_UNSUPPORTED, "an MLP layer is too wide for the fused kernel");
        g_ctx.mlp_tables.insert(g_ctx.mlp_tables.end(), t.begin(), t.end());
        size_t off = (P.arena.size() + 3) / 4 * 4;
        size_t words = t.size() * sizeof(MlpLayerDev) / sizeof(float);
        P.arena.resize(off + words, 0.f);
        std::memcpy(P.arena.data() + off, t.data(), t.size() * sizeof(MlpLayerDev));
        P.arena.resize((P.arena.size() + 3) / 4 * 4, 0.f);
        g_ctx.mlp_table_arena_off[i] = (int64_t)off;
    }
    for (auto &s : P.steps) {
        int S = 0;
        if (s.kind == Step::LSTM && !lstm_smem_bytes(s.Ip, s.Hp, &S))
            return Status::Err(ROSENNA_ERR_UNSUPPORTED, "LSTM hidden size too large for the on-chip kernel");
    }
    // tensor-core path for MLP chains with a layer >= 64 wide and all <= 256
    // (measured: the 10-64-64-64-5 chain runs 42 % faster there than on the FFMA
    // kernel; chains a few units wide stay on FFMA); ROSENNA_MLP_PATH=ffma forces
    // the FFMA kernel, =tc any eligible chain
    const bool tc_ok = tc_register_split_ok();
    const char *path = getenv("ROSENNA_MLP_PATH");
    const std::string mlp_path = path ? path : "";
    for (auto &s : P.steps) {
        if (s.kind != Step::MLP) continue;
        bool eligible = (int)s.layers.size() <= kTcMaxLayers;
        int widest = 0;
        for (auto &l : s.layers) {
            eligible = eligible && l.tc_w_off >= 0;
            widest = std::max(widest, l.M);
        }
        s.tc = tc_ok && eligible && mlp_path != "ffma" && (mlp_path == "tc" || widest >= 64);
    }
    // tensor-core LSTM: for 128 < 4H <= 256 the kernel whose two column groups
    // split one tile's gates; for I <= 32 and H <= 32 the dual-tile kernel (each
    // group a tile of its own, all 4H gates in one N = 4H MMA), else the FFMA
    // kernel.  ROSENNA_LSTM_PATH=ffma / =tc (the split kernel wherever it fits) /
    // =dual force a kernel
    const char *lpath = getenv("ROSENNA_LSTM_PATH");
    const std::string lstm_path = lpath ? lpath : "";
    const bool dual_ok = tc_ok && lstm_dual_tc_regs_ok();
    for (auto &s : P.steps)
        if (s.kind == Step::LSTM) {
            const bool dual_fits = s.lstm_tc_w_off >= 0 && s.I <= 32 && s.H <= 32 && s.lstm_tc_nx == 1 &&
                                   s.lstm_tc_nh == 1 && s.lstm_tc_Np <= 128;
            s.lstm_dual = dual_ok && dual_fits && lstm_path != "ffma" && lstm_path != "tc";
            s.tc = tc_ok && lstm_path != "ffma" && s.lstm_tc_w_off >= 0 &&
                   (lstm_path == "tc" || 4 * s.H > 128 || s.lstm_dual);
        }
    // two stacked LSTM layers with H = 64 (and a layer-1 input of at most 32)
    // run as one fused kernel when the second layer is the only reader of the
    // first layer's output sequence; ROSENNA_LSTM2_FUSE=0 keeps them apart
    const char *fenv = getenv("ROSENNA_LSTM2_FUSE");
    const bool fuse_ok = tc_ok && !(fenv && std::string(fenv) == "0") && lstm2_tc_regs_ok();
    for (size_t si = 0; si + 1 < P.steps.size(); si++) {
        Step &a = P.steps[si];
        const Step &b = P.steps[si + 1];
        a.fuse_next = false;
        if (!fuse_ok || a.kind != Step::LSTM || b.kind != Step::LSTM || !a.tc || !b.tc || b.in != a.y || a.H != 64 ||
            b.H != 64 || b.I != 64 || a.I > 32 || a.lstm_tc_Np != 256 || b.lstm_tc_Np != 256 || a.lstm_tc_Kp != 96 ||
            b.lstm_tc_Kp != 128)
            continue;
        bool other_reader = false;
        for (size_t k = 0; k < P.steps.size(); k++) {
            const Step &q = P.steps[k];
            if (k != si + 1 && (q.in == a.y || q.h0 == a.y || q.c0 == a.y)) other_reader = true;
        }
        for (auto *v : {&P.inputs, &P.outputs})
            for (auto &io : *v)
                if (io.buf == a.y) other_reader = true;
        if (!other_reader) a.fuse_next = true;
    }
    // tensor-core conv (implicit GEMM) for the 3x3 stride-1 conv + 2x2 pool shapes
    // it covers, with one input channel (K-steps of 8 patch positions) or at
    // least 4 (K-steps of a position's 8 channels: with 2 or 3 the zero padding
    // outweighs the tensor cores and the CUDA-core kernel is faster);
    // ROSENNA_CONV_PATH=tiled|direct keeps the CUDA-core kernels, =tc takes the
    // tensor cores for every shape they cover
    const char *cpath = getenv("ROSENNA_CONV_PATH");
    const std::string conv_path = cpath ? cpath : "";
    const char *genv = getenv("ROSENNA_CONV_GROUP");
    g_ctx.conv_group = 4;
    if (genv && atoi(genv) >= 1 && atoi(genv) <= 64) g_ctx.conv_group = atoi(genv);
    for (auto &s : P.steps)
        if (s.kind == Step::CONV)
            s.tc = tc_ok && s.conv && s.ctc_off >= 0 && conv_path != "tiled" && conv_path != "direct" &&
                   (conv_path == "tc" || s.C == 1 || s.C >= 4) &&
                   conv_tc_shape_ok(s.KS, s.str_h, s.str_w, s.pad_h, s.pad_w, s.C, s.OC, s.pool, s.pk, s.pstr_h,
                                    s.pstr_w, s.ppad_h, s.ppad_w, s.Ho, s.Wo);
    // ROSENNA_CONV_FUSE=1: a tensor-core conv whose only reader is the next
    // tensor-core conv runs with it as conv_pair_tc_kernel (shapes it
    // instantiates).  Off by default: both convs are bound by their chunk
    // pipeline (split into TMEM, MMA issue), not by the intermediate's DRAM
    // traffic, and the pair kernel, with fewer chunk slots beside both weight
    // images, measured slower than the two kernels (0.80 ms against 0.60 ms
    // for the 28x28 CNN's convs at 65,536 samples)
    const char *cfenv = getenv("ROSENNA_CONV_FUSE");
    const bool cfuse_ok = cfenv && std::string(cfenv) == "1";
    g_ctx.mid_rows = 0;
    for (size_t si = 0; si + 1 < P.steps.size(); si++) {
        Step &a = P.steps[si];
        const Step &b = P.steps[si + 1];
        if (a.kind != Step::CONV) continue;
        a.fuse_next = false;
        if (!cfuse_ok || b.kind != Step::CONV || !a.tc || !b.tc || b.in != a.out || a.ctc_packed_off < 0 ||
            a.Hq != b.Hin || a.Wq != b.Win || !conv_pair_shape_ok(a.C, a.OC, a.pool, b.C, b.OC, b.pool))
            continue;
        bool other_reader = false;
        for (size_t k = 0; k < P.steps.size(); k++) {
            const Step &q = P.steps[k];
            if (k != si + 1 && (q.in == a.out || q.h0 == a.out || q.c0 == a.out)) other_reader = true;
        }
        for (auto *v : {&P.inputs, &P.outputs})
            for (auto &io : *v)
                if (io.buf == a.out) other_reader = true;
        if (other_reader) continue;
        a.fuse_next = true;
        g_ctx.mid_rows = std::max<int64_t>(g_ctx.mid_rows, (int64_t)b.C * b.Hin * b.Win);
        si++;  // the second conv is not the first of another pair
    }
    g_ctx.is_io_in.assign(P.buf_rows.size(), false);
    g_ctx.is_io_out.assign(P.buf_rows.size(), false);
    for (auto &io : P.inputs) g_ctx.is_io_in[(size_t)io.buf] = true;
    for (auto &io : P.outputs) g_ctx.is_io_out[(size_t)io.buf] = true;
    g_ctx.desc = P.describe();

    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count <= 0)
        return Status::Err(ROSENNA_ERR_NO_DEVICE, "no CUDA device is visible");
    std::vector<int> ids = g_ctx.device_ids;
    if (ids.empty())
        for (int i = 0; i < count; i++) ids.push_back(i);
    int cur = 0;
    cudaGetDevice(&cur);
    for (int id : ids) {
        if (id < 0 || id >= count) return Status::Err(ROSENNA_ERR_NO_DEVICE, "device id out of range");
        auto d = std::make_unique<Device>();
        d->id = id;
        CUDA_TRY(cudaSetDevice(id));
        int major = 0;
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, id);
        if (major < 10) return Status::Err(ROSENNA_ERR_NO_DEVICE, "device is not sm_100 (B200)");
        cudaDeviceGetAttribute(&d->num_sms, cudaDevAttrMultiProcessorCount, id);
        CUDA_TRY(configure_kernels());
        CUDA_TRY(mlp_tc_configure());
        CUDA_TRY(mlp_narrow_configure());
        CUDA_TRY(mlp_stream_configure());
        CUDA_TRY(conv_tc_configure());
        CUDA_TRY(conv_pair_configure());
        CUDA_TRY(lstm2_tc_configure());
        CUDA_TRY(lstm_dual_tc_configure());
        CUDA_TRY(cudaMalloc(&d->arena, sizeof(float) * std::max<size_t>(P.arena.size(), 4)));
        CUDA_TRY(cudaMemcpy(d->arena, P.arena.data(), sizeof(float) * P.arena.size(), cudaMemcpyHostToDevice));
        CUDA_TRY(cudaMalloc(&d->err, 64 * sizeof(int)));
        CUDA_TRY(cudaMemset(d->err, 0, 64 * sizeof(int)));
        CUDA_TRY(cudaMallocHost(&d->err_host, 64 * sizeof(int)));
        std::memset(d->err_host, 0, 64 * sizeof(int));
        d->tc_args.assign(P.steps.size(), TcArgs{});
        d->lstm_args.assign(P.steps.size(), TcLstmArgs{});
        d->lstm2_args.assign(P.steps.size(), TcLstm2Args{});
        for (size_t si = 0; si + 1 < P.steps.size(); si++) {
            const Step &s = P.steps[si];
            if (s.kind != Step::LSTM || !s.fuse_next) continue;
            const Step &s2 = P.steps[si + 1];
            TcLstm2Args &a = d->lstm2_args[si];
            a.arena = d->arena;
            a.err = d->err;
            a.T = s.T;
            a.I = s.I;
            const Step *ls[2] = {&s, &s2};
            for (int k = 0; k < 2; k++) {
                a.h0_const[k] = ls[k]->h0_const;
                a.c0_const[k] = ls[k]->c0_const;
                float *bias = k == 0 ? a.bias1 : a.bias2;
                for (int c = 0; c < 256; c++) bias[c] = P.arena[(size_t)ls[k]->lstm_tc_b_off + (size_t)c];
                const char *why = "";
                if (!mlp_tc_encode_map(k == 0 ? &a.map1 : &a.map2, d->arena + ls[k]->lstm_tc_w_off, ls[k]->lstm_tc_Kp,
                                       256, &why, 128))
                    return Status::Err(ROSENNA_ERR_CUDA, why);
            }
        }
        for (size_t si = 0; si < P.steps.size(); si++) {
            const Step &s = P.steps[si];
            if (s.kind != Step::LSTM || !s.tc) continue;
            TcLstmArgs &a = d->lstm_args[si];
            a.arena = d->arena;
            a.err = d->err;
            a.b_off = s.lstm_tc_b_off;
            a.h0_const = s.h0_const;
            a.c0_const = s.c0_const;
            a.T = s.T;
            a.I = s.I;
            a.H = s.H;
            a.Np = s.lstm_tc_Np;
            a.nx = s.lstm_tc_nx;
            a.nh = s.lstm_tc_nh;
            const char *why = "";
            if (!mlp_tc_encode_map(&a.map, d->arena + s.lstm_tc_w_off, s.lstm_tc_Kp, s.lstm_tc_Np, &why))
                return Status::Err(ROSENNA_ERR_CUDA, why);
        }
        for (size_t si = 0; si < P.steps.size(); si++) {
            const Step &s = P.steps[si];
            if (!s.tc) continue;
            TcArgs &a = d->tc_args[si];
            a.arena = d->arena;
            a.err = d->err;
            a.nlayers = (int)s.layers.size();
            // a narrow last layer runs on the CUDA cores at the end of the kernel
            // (ROSENNA_TC_TAIL=0 keeps it on the tensor cores)
            const MlpLayer &lastl = s.layers.back();
            const char *tail_env = getenv("ROSENNA_TC_TAIL");
            if (a.nlayers >= 2 && lastl.M <= kTcTailMaxN && !(tail_env && std::string(tail_env) == "0")) {
                a.nlayers--;
                a.tail_n = lastl.M;
                a.tail_np = lastl.Mp;
                a.tail_k = lastl.K;
                a.tail_kp = lastl.Kp;
                a.tail_act = lastl.act;
                a.tail_w_off = lastl.w_off;
                a.tail_b_off = lastl.b_off;
            }
            for (int l = 0; l < a.nlayers; l++) {
                const MlpLayer &ly = s.layers[(size_t)l];
                a.L[l] = TcLayer{ly.K, ly.M, ly.tc_Kp, ly.tc_Np, ly.tc_Kp / 32, ly.act, ly.tc_w_off, ly.tc_b_off};
                const char *why = "";
                if (!mlp_tc_encode_map(&a.maps[l], d->arena + ly.tc_w_off, ly.tc_Kp, ly.tc_Np, &why))
                    return Status::Err(ROSENNA_ERR_CUDA, why);
            }
            // no layer wider than 128: each column group takes a tile of its own
            // (ROSENNA_TC_DUAL=0 splits one tile's columns between the groups instead)
            bool narrow = true;
            for (int l = 0; l < a.nlayers; l++) narrow = narrow && a.L[l].Np <= 128;
            const char *dual_env = getenv("ROSENNA_TC_DUAL");
            a.dual = narrow && !(dual_env && std::string(dual_env) == "0") ? 1 : 0;
            // no layer wider than 64 and the weights fit in shared memory: the
            // resident-weight kernel (ROSENNA_TC_NARROW=0 keeps the others)
            const char *narrow_env = getenv("ROSENNA_TC_NARROW");
            a.narrow = mlp_narrow_fits(a) && !(narrow_env && std::string(narrow_env) == "0") ? 1 : 0;
            // the same with a long first layer streamed by TMA (ROSENNA_TC_STREAM=0 keeps the others)
            const char *stream_env = getenv("ROSENNA_TC_STREAM");
            a.stream = !a.narrow && mlp_stream_fits(a) && !(stream_env && std::string(stream_env) == "0") ? 1 : 0;
        }
        for (auto &s : d->slots) {
            CUDA_TRY(cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking));
            CUDA_TRY(cudaEventCreateWithFlags(&s.done, cudaEventDisableTiming));
        }
        noalloc_setup(*d);
        // the first device's budget stands for all (the same GPU model)
        if (g_ctx.devs.empty()) g_ctx.scratch_budget = measure_scratch_budget();
        g_ctx.devs.push_back(std::move(d));
    }
    cudaSetDevice(cur);
    g_ctx.ready = true;
    return Status::Ok();
}

int report(const Status &st) { return st.ok() ? ok() : fail(st.code, st.msg); }

// Host-array use_model; the caller holds g_mu.
int use_model_f32_locked(int64_t n, const float *const *inputs, float *const *outputs) {
    if (!g_ctx.ready) return fail(ROSENNA_ERR_STATE, "initialize() has not succeeded");
    Status st = check_batch(n);
    if (!st.ok()) return report(st);
    if (!inputs || !outputs) return fail(ROSENNA_ERR_ARG, "null input/output array list");
    for (size_t i = 0; i < g_ctx.plan.inputs.size(); i++)
        if (!inputs[i]) return fail(ROSENNA_ERR_ARG, "null input pointer");
    for (size_t i = 0; i < g_ctx.plan.outputs.size(); i++)
        if (!outputs[i]) return fail(ROSENNA_ERR_ARG, "null output pointer");
    g_launches = 0;
    if (n == 0) return ok();
    int cur = 0;
    cudaGetDevice(&cur);
    const int G = (int)g_ctx.devs.size();
    std::vector<Status> res((size_t)G);
    std::vector<std::thread> th;
    for (int g = 0; g < G; g++) {
        // contiguous split; the first n % G ranks take one extra sample
        const int64_t base = n / G, rem = n % G;
        const int64_t a = g * base + std::min<int64_t>(g, rem), b = a + base + (g < rem ? 1 : 0);
        th.emplace_back([&, g, a, b] { res[(size_t)g] = host_range(*g_ctx.devs[(size_t)g], n, a, b, inputs, outputs); });
    }
    for (auto &t : th) t.join();
    cudaSetDevice(cur);
    for (auto &r : res)
        if (!r.ok()) return report(r);
    return ok();
}

// fp64 host arrays converted to fp32 around use_model_f32_locked; the caller
// holds g_mu, so the plan cannot change (finalize/initialize) during the call.
int use_model_f64_locked(int64_t n, const double *const *inputs, double *const *outputs) {
    if (!g_ctx.ready) return fail(ROSENNA_ERR_STATE, "initialize() has not succeeded");
    if (n < 0 || !inputs || !outputs) return fail(ROSENNA_ERR_ARG, "bad arguments");
    const Plan &P = g_ctx.plan;
    std::vector<std::vector<float>> fi(P.inputs.size()), fo(P.outputs.size());
    std::vector<const float *> pi;
    std::vector<float *> po;
    for (size_t i = 0; i < P.inputs.size(); i++) {
        if (!inputs[i]) return fail(ROSENNA_ERR_ARG, "null input pointer");
        size_t cnt = (size_t)(P.inputs[i].rows * n);
        fi[i].resize(cnt);
        for (size_t k = 0; k < cnt; k++) fi[i][k] = (float)inputs[i][k];
        pi.push_back(fi[i].data());
    }
    for (size_t i = 0; i < P.outputs.size(); i++) {
        if (!outputs[i]) return fail(ROSENNA_ERR_ARG, "null output pointer");
        fo[i].resize((size_t)(P.outputs[i].rows * n));
        po.push_back(fo[i].data());
    }
    int rc = use_model_f32_locked(n, pi.data(), po.data());
    if (rc) return rc;
    for (size_t i = 0; i < P.outputs.size(); i++)
        for (size_t k = 0; k < fo[i].size(); k++) outputs[i][k] = fo[i][k];
    return ok();
}

}  // namespace
}  // namespace rosenna

using namespace rosenna;

extern "C" {

int rosenna_initialize_from(const char *model_txt, const char *weights_txt, const char *variables_fpp) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!model_txt || !weights_txt) return fail(ROSENNA_ERR_ARG, "null path");
    std::string vars;
    if (variables_fpp) {
        vars = variables_fpp;
    } else {
        std::string m(model_txt);
        size_t p = m.find_last_of('/');
        vars = (p == std::string::npos ? std::string() : m.substr(0, p + 1)) + "variables.fpp";
    }
    Status st = do_initialize(model_txt, weights_txt, vars);
    if (!st.ok()) release_all();
    return report(st);
}

int rosenna_check_model(const char *model_txt, const char *weights_txt, const char *variables_fpp) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!model_txt || !weights_txt) return fail(ROSENNA_ERR_ARG, "null path");
    std::string vars;
    if (variables_fpp) {
        vars = variables_fpp;
    } else {
        std::string m(model_txt);
        size_t p = m.find_last_of('/');
        vars = (p == std::string::npos ? std::string() : m.substr(0, p + 1)) + "variables.fpp";
    }
    ModelFiles mf;
    Plan plan;
    Status st = read_model_files(model_txt, weights_txt, vars, &mf);
    if (st.ok()) st = build_plan(mf, &plan);
    if (st.ok()) g_ctx.desc = plan.describe();
    return report(st);
}

int rosenna_initialize(void) { return rosenna_initialize_from("onnxModel.txt", "onnxWeights.txt", "variables.fpp"); }

void initialize(void) { (void)rosenna_initialize(); }

// roseNNa's fixed-shape entry point, SUBROUTINE use_model(i0,..,o0,..)
// bind(c,name="use_model") (fLibrary/modelCreator.fpp:42), which C code calls as
// void use_model(double *i0, .., double *o0) (examples/cAPI.c:3): fp64 arrays of
// the export shapes, the model's inputs then its outputs, evaluated at the
// export batch.  It takes the largest argument count the engine accepts and
// reads only the model's own count, so a caller that declares it with that
// count passes exactly the arguments read.  The status is kept for
// rosenna_last_status() / rosenna_last_error(); the reference aborts instead.
void use_model(double *a0, double *a1, double *a2, double *a3, double *a4, double *a5, double *a6, double *a7, double *a8, double *a9, double *a10, double *a11, double *a12, double *a13, double *a14, double *a15) {
    double *const a[kLegacyArgs] = {a0, a1, a2, a3, a4, a5, a6, a7, a8, a9, a10, a11, a12, a13, a14, a15};
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_ctx.ready) {
        fail(ROSENNA_ERR_STATE, "initialize() has not succeeded");
        return;
    }
    const Plan &P = g_ctx.plan;
    if (P.inputs.empty() || P.inputs.size() + P.outputs.size() > (size_t)kLegacyArgs) {
        fail(ROSENNA_ERR_UNSUPPORTED, "use_model takes at most " + std::to_string(kLegacyArgs) +
                                          " arrays; call rosenna_use_model_f64 with array lists instead");
        return;
    }
    const IoDesc &d0 = P.inputs[0];
    (void)use_model_f64_locked(d0.shape[(size_t)d0.bdim], a, a + P.inputs.size());
}

int rosenna_finalize(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    release_all();
    g_ctx.plan = Plan();
    g_ctx.mf = ModelFiles();
    return ok();
}

int rosenna_set_devices(const int *ids, int count) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (count < 0 || (count > 0 && !ids)) return fail(ROSENNA_ERR_ARG, "bad device list");
    g_ctx.device_ids.assign(ids, ids + count);
    return ok();
}

int rosenna_last_status(void) { return g_status; }
const char *rosenna_last_error(void) { return g_error.c_str(); }

int rosenna_num_inputs(void) { return g_ctx.ready ? (int)g_ctx.plan.inputs.size() : -ROSENNA_ERR_STATE; }
int rosenna_num_outputs(void) { return g_ctx.ready ? (int)g_ctx.plan.outputs.size() : -ROSENNA_ERR_STATE; }

static int io_shape(const std::vector<IoDesc> &v, int i, int64_t *dims, int max_dims, int *bdim) {
    if (!g_ctx.ready) return -ROSENNA_ERR_STATE;
    if (i < 0 || i >= (int)v.size()) return -ROSENNA_ERR_ARG;
    const IoDesc &d = v[(size_t)i];
    for (int k = 0; k < (int)d.shape.size() && k < max_dims; k++) dims[k] = d.shape[(size_t)k];
    if (bdim) *bdim = d.bdim;
    return (int)d.shape.size();
}

int rosenna_input_shape(int i, int64_t *dims, int max_dims, int *bdim) { return io_shape(g_ctx.plan.inputs, i, dims, max_dims, bdim); }
int rosenna_output_shape(int i, int64_t *dims, int max_dims, int *bdim) { return io_shape(g_ctx.plan.outputs, i, dims, max_dims, bdim); }

int rosenna_use_model_f32(int64_t n, const float *const *inputs, float *const *outputs) {
    std::lock_guard<std::mutex> lk(g_mu);
    return use_model_f32_locked(n, inputs, outputs);
}

int rosenna_use_model_f64(int64_t n, const double *const *inputs, double *const *outputs) {
    std::lock_guard<std::mutex> lk(g_mu);
    return use_model_f64_locked(n, inputs, outputs);
}

int rosenna_use_model_device_f32(int64_t n, const float *const *inputs, float *const *outputs, void *stream) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_ctx.ready) return fail(ROSENNA_ERR_STATE, "initialize() has not succeeded");
    Status st = check_batch(n);
    if (!st.ok()) return report(st);
    if (!inputs || !outputs) return fail(ROSENNA_ERR_ARG, "null input/output array list");
    g_launches = 0;
    int cur = 0;
    if (cudaGetDevice(&cur) != cudaSuccess) return fail(ROSENNA_ERR_CUDA, "cudaGetDevice failed");
    // with one selected GPU that GPU is used; otherwise the current device
    Device *d = g_ctx.devs.size() == 1 ? g_ctx.devs[0].get() : device_by_id(cur);
    if (!d) return fail(ROSENNA_ERR_NO_DEVICE, "the current device was not initialized");
    if (n == 0) return ok();
    struct Restore {
        int dev;
        ~Restore() { cudaSetDevice(dev); }
    } restore{cur};
    if (cudaSetDevice(d->id) != cudaSuccess) return fail(ROSENNA_ERR_CUDA, "cudaSetDevice failed");
    const Plan &P = g_ctx.plan;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int64_t chunk = max_chunk(n);
    st = ensure_scratch(d->slots[0], chunk);
    if (st.ok()) st = ensure_mid(d->slots[0], d->num_sms);
    if (!st.ok()) return report(st);
    // the scratch buffers are shared by every device-path call on this device
    if (cudaStreamWaitEvent(s, d->slots[0].done, 0) != cudaSuccess) return fail(ROSENNA_ERR_CUDA, "cudaStreamWaitEvent failed");
    for (int64_t c0 = 0; c0 < n; c0 += chunk) {
        const int64_t cnt = std::min(chunk, n - c0);
        std::vector<float *> ptr(P.buf_rows.size(), nullptr);
        std::vector<int64_t> ld(P.buf_rows.size(), d->slots[0].cap);
        for (size_t b = 0; b < ptr.size(); b++) ptr[b] = d->slots[0].scratch.empty() ? nullptr : d->slots[0].scratch[b];
        for (size_t i = 0; i < P.inputs.size(); i++) {
            if (!inputs[i]) return fail(ROSENNA_ERR_ARG, "null input pointer");
            ptr[(size_t)P.inputs[i].buf] = const_cast<float *>(inputs[i]) + P.inputs[i].pre * c0;
            ld[(size_t)P.inputs[i].buf] = n;
        }
        for (size_t i = 0; i < P.outputs.size(); i++) {
            if (!outputs[i]) return fail(ROSENNA_ERR_ARG, "null output pointer");
            ptr[(size_t)P.outputs[i].buf] = outputs[i] + c0;
            ld[(size_t)P.outputs[i].buf] = n;
        }
        st = run_plan(*d, ptr, ld, cnt, s, &d->slots[0]);
        if (!st.ok()) return report(st);
    }
    if (cudaEventRecord(d->slots[0].done, s) != cudaSuccess) return fail(ROSENNA_ERR_CUDA, "cudaEventRecord failed");
    return ok();
}

int rosenna_step_timing_begin(int64_t max_records) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_ctx.ready) return fail(ROSENNA_ERR_STATE, "initialize() has not succeeded");
    if (max_records < 0 || max_records > ((int64_t)1 << 20)) return fail(ROSENNA_ERR_ARG, "max_records out of range");
    int cur = 0;
    cudaGetDevice(&cur);
    for (auto &dp : g_ctx.devs) {
        Device &d = *dp;
        if (cudaSetDevice(d.id) != cudaSuccess) return fail(ROSENNA_ERR_CUDA, "cudaSetDevice failed");
        for (auto e : d.tev) cudaEventDestroy(e);
        d.tev.assign((size_t)(2 * max_records), nullptr);
        for (auto &e : d.tev)
            if (cudaEventCreate(&e) != cudaSuccess) {
                cudaSetDevice(cur);
                return fail(ROSENNA_ERR_CUDA, "cudaEventCreate (step timing) failed");
            }
        d.tev_step.assign((size_t)max_records, -1);
        d.tev_used = 0;
    }
    cudaSetDevice(cur);
    return ok();
}

int rosenna_step_timing_end(double *ms, int64_t *runs, int max_steps) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_ctx.ready) return fail(ROSENNA_ERR_STATE, "initialize() has not succeeded");
    if (max_steps < 0 || (max_steps > 0 && (!ms || !runs))) return fail(ROSENNA_ERR_ARG, "bad step arrays");
    for (int i = 0; i < max_steps; i++) {
        ms[i] = 0.0;
        runs[i] = 0;
    }
    int cur = 0;
    cudaGetDevice(&cur);
    int rc = 0;
    for (auto &dp : g_ctx.devs) {
        Device &d = *dp;
        cudaSetDevice(d.id);
        for (int64_t k = 0; k < d.tev_used && !rc; k++) {
            float t = 0.f;
            if (cudaEventSynchronize(d.tev[(size_t)(2 * k + 1)]) != cudaSuccess ||
                cudaEventElapsedTime(&t, d.tev[(size_t)(2 * k)], d.tev[(size_t)(2 * k + 1)]) != cudaSuccess) {
                rc = fail(ROSENNA_ERR_CUDA, "step timing events could not be read");
                break;
            }
            const int si = d.tev_step[(size_t)k];
            if (si >= 0 && si < max_steps) {
                ms[si] += t;
                runs[si]++;
            }
        }
        for (auto e : d.tev) cudaEventDestroy(e);
        d.tev.clear();
        d.tev_step.clear();
        d.tev_used = 0;
    }
    cudaSetDevice(cur);
    return rc ? rc : ok();
}

int rosenna_step_count(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    return g_ctx.ready ? (int)g_ctx.plan.steps.size() : -ROSENNA_ERR_STATE;
}

int rosenna_step_info(int i, char *kernel, int kernel_len, double *flops_per_sample) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_ctx.ready) return fail(ROSENNA_ERR_STATE, "initialize() has not succeeded");
    if (i < 0 || i >= (int)g_ctx.plan.steps.size()) return fail(ROSENNA_ERR_ARG, "step index out of range");
    const Step &s = g_ctx.plan.steps[(size_t)i];
    std::string name;
    double f = 0.0;
    switch (s.kind) {
        case Step::MLP: {
            const bool dual = s.tc && !g_ctx.devs.empty() && g_ctx.devs[0]->tc_args[(size_t)i].dual;
            const bool narrow = s.tc && !g_ctx.devs.empty() && g_ctx.devs[0]->tc_args[(size_t)i].narrow;
            const bool stream = s.tc && !g_ctx.devs.empty() && g_ctx.devs[0]->tc_args[(size_t)i].stream;
            name = s.tc ? (narrow   ? "mlp_narrow_tc_kernel"
                           : stream ? "mlp_stream_tc_kernel"
                           : dual   ? "mlp_tc_dual_kernel"
                                    : "mlp_tc_kernel")
                        : "mlp_ffma_kernel";
            for (auto &l : s.layers) f += 2.0 * l.K * l.M;
            f *= s.rsub;
            break;
        }
        case Step::LSTM:
            if (s.fuse_next) {  // both layers
                const Step &s2 = g_ctx.plan.steps[(size_t)i + 1];
                name = "lstm2_tc_kernel";
                f = 2.0 * s.T * 4.0 * s.H * (double)(s.I + s.H) + 2.0 * s2.T * 4.0 * s2.H * (double)(s2.I + s2.H);
            } else if (i > 0 && g_ctx.plan.steps[(size_t)i - 1].fuse_next) {
                name = "(in lstm2_tc_kernel)";
            } else {
                name = s.tc ? (s.lstm_dual ? "lstm_dual_tc_kernel" : "lstm_tc_kernel") : "lstm_ffma_kernel";
                f = 2.0 * s.T * 4.0 * s.H * (double)(s.I + s.H);
            }
            break;
        case Step::CONV: {
            ConvArgs a{};
            a.conv = s.conv; a.relu = s.relu; a.C = s.C; a.Hin = s.Hin; a.Win = s.Win; a.OC = s.OC; a.KS = s.KS;
            a.str_h = s.str_h; a.str_w = s.str_w; a.pool = s.pool; a.pk = s.pk;
            name = s.tc ? "conv_tc_kernel" : conv_kernel_name(a);
            if (s.conv) f = 2.0 * s.Ho * s.Wo * s.OC * (double)s.C * s.KS * s.KS;
            if (s.fuse_next) {  // both convs
                const Step &s2 = g_ctx.plan.steps[(size_t)i + 1];
                name = "conv_pair_tc_kernel";
                f += 2.0 * s2.Ho * s2.Wo * s2.OC * (double)s2.C * s2.KS * s2.KS;
            } else if (i > 0 && g_ctx.plan.steps[(size_t)i - 1].kind == Step::CONV &&
                       g_ctx.plan.steps[(size_t)i - 1].fuse_next) {
                name = "(in conv_pair_tc_kernel)";
                f = 0;
            }
            break;
        }
        case Step::GATHER:
        case Step::COPY: name = "gather_kernel"; break;
        case Step::DEINTERLEAVE: name = "deinterleave_kernel"; break;
        case Step::ACT:
        case Step::ADD: name = "act_kernel"; break;
    }
    if (kernel && kernel_len > 0) snprintf(kernel, (size_t)kernel_len, "%s", name.c_str());
    if (flops_per_sample) *flops_per_sample = f;
    return ok();
}

int64_t rosenna_last_launch_count(void) { return g_launches.load(); }

const char *rosenna_plan_description(void) { return g_ctx.desc.c_str(); }

}  // extern "C"

extern "C" int rosenna_use_model_device_noalloc_f32(int64_t n, const float *const *inputs, float *const *outputs,
                                                    void *stream) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_ctx.ready) return fail(ROSENNA_ERR_STATE, "initialize() has not succeeded");
    Status st = check_batch(n);
    if (!st.ok()) return report(st);
    if (!inputs || !outputs) return fail(ROSENNA_ERR_ARG, "null input/output array list");
    const Plan &P = g_ctx.plan;
    for (size_t i = 0; i < P.inputs.size(); i++)
        if (!inputs[i]) return fail(ROSENNA_ERR_ARG, "null input pointer");
    for (size_t i = 0; i < P.outputs.size(); i++)
        if (!outputs[i]) return fail(ROSENNA_ERR_ARG, "null output pointer");
    g_launches = 0;
    int cur = 0;
    if (cudaGetDevice(&cur) != cudaSuccess) return fail(ROSENNA_ERR_CUDA, "cudaGetDevice failed");
    Device *d = g_ctx.devs.size() == 1 ? g_ctx.devs[0].get() : device_by_id(cur);
    if (!d) return fail(ROSENNA_ERR_NO_DEVICE, "the current device was not initialized");
    if (n == 0) return ok();

    // intermediates of the plan, each rows x n floats, 256-byte aligned
    const std::vector<bool> used = used_buffers();
    std::vector<size_t> off(P.buf_rows.size(), 0);
    size_t need = 0;
    for (size_t b = 0; b < used.size(); b++) {
        if (!used[b] || !is_scratch((int)b)) continue;
        off[b] = need;
        need += ((size_t)P.buf_rows[b] * (size_t)n * sizeof(float) + 255) / 256 * 256;
    }
    if (need > kNoAllocScratchBytes) {
        size_t per_sample = 0;
        for (size_t b = 0; b < used.size(); b++)
            if (used[b] && is_scratch((int)b)) per_sample += (size_t)P.buf_rows[b] * sizeof(float);
        char msg[256];
        snprintf(msg, sizeof msg,
                 "n=%lld needs %zu bytes of intermediates; the allocation-free entry point has %zu bytes "
                 "(at most about %zu samples for this model)",
                 (long long)n, need, kNoAllocScratchBytes, per_sample ? kNoAllocScratchBytes / per_sample : 0);
        return fail(ROSENNA_ERR_SHAPE, msg);
    }

    struct Restore {
        int dev;
        ~Restore() { cudaSetDevice(dev); }
    } restore{cur};
    if (cudaSetDevice(d->id) != cudaSuccess) return fail(ROSENNA_ERR_CUDA, "cudaSetDevice failed");
    // the array's device address was looked up at initialize, with this device current
    if (!d->noalloc_base) return fail(ROSENNA_ERR_CUDA, d->noalloc_err);
    unsigned char *base = static_cast<unsigned char *>(d->noalloc_base);

    std::vector<float *> ptr(P.buf_rows.size(), nullptr);
    std::vector<int64_t> ld(P.buf_rows.size(), n);
    for (size_t b = 0; b < used.size(); b++)
        if (used[b] && is_scratch((int)b)) ptr[b] = reinterpret_cast<float *>(base + off[b]);
    for (size_t i = 0; i < P.inputs.size(); i++) ptr[(size_t)P.inputs[i].buf] = const_cast<float *>(inputs[i]);
    for (size_t i = 0; i < P.outputs.size(); i++) ptr[(size_t)P.outputs[i].buf] = outputs[i];
    st = run_plan(*d, ptr, ld, n, reinterpret_cast<cudaStream_t>(stream), nullptr);  // no mid: two conv kernels
    return report(st);
}
