// Builds the launch plan by interpreting variables.fpp's `architecture` list
// the way fLibrary/modelCreator.fpp:79-171 expands it into Fortran calls:
// one entry per ONNX node, operating on named allocatable arrays.  Instead of
// emitting layer calls, each entry extends the plan:
//   Gemm (+ Relu/Tanh/Sigmoid) chains      -> one fused MLP step
//   LSTM                                   -> one persistent LSTM step
//   Conv (+ Relu) (+ MaxPool/AveragePool)  -> one fused conv/pool step
//   Transpose / Squeeze / Reshape          -> nothing when the per-sample element
//                                             order is unchanged, else a gather
//   Reshape of a stored constant           -> a constant, read by MatMul
//   MatMul by a constant                   -> a bias-free layer of the MLP step
//   Add of a constant                      -> folded into the bias of the step
//                                             that produced its operand, else
//                                             an ADD step (+ activation)
// Data movement ops are evaluated with the reference's own index formulas
// (Fortran RESHAPE with ORDER) at a probe batch of 3, which both checks that the
// op keeps samples independent and yields the per-sample row map.
#include "plan.hpp"

#include <algorithm>
#include <cstring>
#include <map>
#include <set>
#include <sstream>

#include "../../include/rosenna.h"
#include "conv_tc.cuh"

namespace rosenna {
namespace {

using Shape = std::vector<int64_t>;
constexpr int64_t kProbe = 3;

int64_t numel(const Shape &s) {
    int64_t n = 1;
    for (auto d : s) n *= d;
    return n;
}

int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

std::string shape_str(const Shape &s) {
    std::ostringstream o;
    o << "(";
    for (size_t i = 0; i < s.size(); i++) o << (i ? "," : "") << s[i];
    o << ")";
    return o.str();
}

void unravel(int64_t L, const Shape &s, int64_t *sub) {
    for (size_t i = 0; i < s.size(); i++) {
        sub[i] = L % s[i];
        L /= s[i];
    }
}

int64_t ravel(const int64_t *sub, const Shape &s) {
    int64_t L = 0, st = 1;
    for (size_t i = 0; i < s.size(); i++) {
        L += sub[i] * st;
        st *= s[i];
    }
    return L;
}

// Fortran RESHAPE(SOURCE, SHAPE=R, ORDER=order1): source elements in array
// element order fill R with subscript order1(1) varying fastest.
// Returns, for each element of R (column-major linear index), its source index.
std::vector<int64_t> fortran_reshape_order_map(const Shape &src, const Shape &R, const std::vector<int64_t> &order1) {
    std::vector<int64_t> m((size_t)numel(R), -1);
    int64_t n = std::min(numel(src), numel(R));
    std::vector<int64_t> stride(R.size()), sub(R.size(), 0);
    int64_t st = 1;
    for (size_t i = 0; i < R.size(); i++) {
        stride[i] = st;
        st *= R[i];
    }
    for (int64_t L = 0; L < n; L++) {
        int64_t off = 0;
        for (size_t k = 0; k < R.size(); k++) off += sub[order1[k] - 1] * stride[order1[k] - 1];
        m[(size_t)off] = L;
        for (size_t k = 0; k < R.size(); k++) {
            int64_t d = order1[k] - 1;
            if (++sub[d] < R[d]) break;
            sub[d] = 0;
        }
    }
    return m;
}

// C-order reshape (the two RESHAPEs of modelCreator.fpp:125-126 compose to it).
std::vector<int64_t> c_order_reshape_map(const Shape &src, const Shape &R) {
    std::vector<int64_t> m((size_t)numel(R), -1);
    std::vector<int64_t> sr(R.size()), ss(src.size());
    for (int64_t L = 0; L < numel(R); L++) {
        unravel(L, R, sr.data());
        int64_t c = 0;
        for (size_t i = 0; i < R.size(); i++) c = c * R[i] + sr[i];
        for (size_t i = src.size(); i-- > 0;) {
            ss[i] = c % src[i];
            c /= src[i];
        }
        m[(size_t)L] = ravel(ss.data(), src);
    }
    return m;
}

// From a full index map at the probe batch, derive the per-sample row map.
bool per_sample_map(const Shape &S, int b, const Shape &R, int b2, const std::vector<int64_t> &r2s,
                    std::vector<int32_t> *map) {
    int64_t rows_r = numel(R) / R[b2];
    map->assign((size_t)rows_r, -1);
    std::vector<int64_t> sr(R.size()), ss(S.size());
    for (int64_t L = 0; L < numel(R); L++) {
        int64_t Ls = r2s[(size_t)L];
        if (Ls < 0) return false;
        unravel(L, R, sr.data());
        unravel(Ls, S, ss.data());
        if (sr[b2] != ss[b]) return false;
        int64_t pr = 0, st = 1;
        for (size_t i = 0; i < R.size(); i++)
            if ((int)i != b2) { pr += sr[i] * st; st *= R[i]; }
        int64_t ps = 0;
        st = 1;
        for (size_t i = 0; i < S.size(); i++)
            if ((int)i != b) { ps += ss[i] * st; st *= S[i]; }
        int32_t &slot = (*map)[(size_t)pr];
        if (slot == -1) slot = (int32_t)ps;
        else if (slot != ps) return false;
    }
    for (auto v : *map)
        if (v < 0) return false;
    return true;
}

// fp32 -> tf32 (10 mantissa bits), round to nearest with ties away from zero,
// as the device's cvt.rna.tf32.f32 does.
float tf32_round(float x) {
    uint32_t b;
    std::memcpy(&b, &x, 4);
    if ((b & 0x7f800000u) != 0x7f800000u) b = (b + 0x1000u) & 0xffffe000u;
    float y;
    std::memcpy(&y, &b, 4);
    return y;
}

bool is_identity(const std::vector<int32_t> &m, int64_t src_rows) {
    if ((int64_t)m.size() != src_rows) return false;
    for (size_t i = 0; i < m.size(); i++)
        if (m[i] != (int32_t)i) return false;
    return true;
}

struct TVal {
    Shape shape;
    int bdim = 0;
    int buf = -1;  // -2: value not representable per sample (an error if read); -3: a stored constant;
                   // -4: a Concat, read only through a Slice/Gather selecting one of its parts
    int64_t rows() const { return numel(shape) / shape[(size_t)bdim]; }
};

class Builder {
  public:
    Builder(const ModelFiles &mf, Plan *plan) : mf_(mf), plan_(plan) {}
    Status run();

  private:
    const ModelFiles &mf_;
    Plan *plan_;
    std::map<std::string, TVal> vars_;
    std::vector<int> refc_;
    int64_t B0_ = 1;
    int n_gemm_ = 0, n_lstm_ = 0, n_conv_ = 0, n_max_ = 0, n_avg_ = 0, n_add_ = 0, n_resh_ = 0;
    std::map<std::string, HostArray> consts_;  // variables bound to a stored constant (-3)

    int new_buf(int64_t rows) {
        plan_->buf_rows.push_back(rows);
        refc_.push_back(0);
        return (int)plan_->buf_rows.size() - 1;
    }
    void bind(const std::string &name, const TVal &v) {
        if (v.buf != -4) concats_.erase(name);
        auto it = vars_.find(name);
        if (it != vars_.end() && it->second.buf >= 0) refc_[(size_t)it->second.buf]--;
        if (v.buf >= 0) refc_[(size_t)v.buf]++;
        vars_[name] = v;
    }
    Status get(const std::string &name, TVal *v) {
        auto it = vars_.find(name);
        if (it == vars_.end()) return Status::Err(ROSENNA_ERR_FORMAT, "architecture reads undefined variable '" + name + "'");
        if (it->second.buf == -3)
            return Status::Err(ROSENNA_ERR_UNSUPPORTED, "variable '" + name + "' is a stored constant; only MatMul's second operand may be one");
        if (it->second.buf == -4)
            return Status::Err(ROSENNA_ERR_UNSUPPORTED,
                               "variable '" + name + "' is a Concat; it is read only through a Slice or Gather of one part");
        if (it->second.buf < 0)
            return Status::Err(ROSENNA_ERR_UNSUPPORTED, "variable '" + name + "' mixes samples after a Reshape; not batched");
        *v = it->second;
        return Status::Ok();
    }
    int64_t put(const float *p, size_t n) {
        auto &a = plan_->arena;
        size_t off = (size_t)round_up((int64_t)a.size(), 4);
        a.resize(off + n, 0.f);
        if (n) std::memcpy(a.data() + off, p, n * sizeof(float));
        a.resize((size_t)round_up((int64_t)a.size(), 4), 0.f);
        return (int64_t)off;
    }
    int64_t put_map(const std::vector<int32_t> &m) {
        static_assert(sizeof(int32_t) == sizeof(float), "map words");
        return put(reinterpret_cast<const float *>(m.data()), m.size());
    }
    Step *last_producing(int buf) {
        if (plan_->steps.empty()) return nullptr;
        Step &s = plan_->steps.back();
        if (s.out != buf || refc_[(size_t)buf] != 1) return nullptr;
        return &s;
    }
    // data movement: bind `name` to `x` rearranged through a full-index map at the
    // probe batch; `Rx` is the result shape at the export batch.
    Status move(const std::string &name, const TVal &x, const Shape &Rx, const Shape &R, int b2,
                const std::vector<int64_t> &r2s, const Shape &S, bool poison_on_fail) {
        std::vector<int32_t> m;
        TVal out{Rx, b2, -1};
        if (!per_sample_map(S, x.bdim, R, b2, r2s, &m)) {
            if (!poison_on_fail)
                return Status::Err(ROSENNA_ERR_UNSUPPORTED, "a data-movement op on " + shape_str(x.shape) + " mixes samples");
            out.buf = -2;
            bind(name, out);
            return Status::Ok();
        }
        if (is_identity(m, x.rows())) {
            out.buf = x.buf;
        } else {
            Step s;
            s.kind = Step::GATHER;
            s.in = x.buf;
            s.out = new_buf((int64_t)m.size());
            s.map_off = put_map(m);
            plan_->steps.push_back(s);
            out.buf = s.out;
        }
        bind(name, out);
        return Status::Ok();
    }
    Shape probe(const TVal &x) {
        Shape S = x.shape;
        S[(size_t)x.bdim] = kProbe;
        return S;
    }

    Status push_layer(const std::string &name, const TVal &x, int M, int K, const std::vector<double> &w_mk,
                      const std::vector<double> &bias);
    Status op_gemm(const PyVal &e);
    Status op_matmul(const PyVal &e);
    Status op_add(const PyVal &e);
    Status op_act(const PyVal &e, int act);
    Status op_lstm(const PyVal &e);
    Status op_conv(const PyVal &e);
    Status op_pool(const PyVal &e, bool avg);
    Status op_transpose(const PyVal &e);
    Status op_reshape(const PyVal &e);
    Status op_squeeze(const PyVal &e);
    Status op_slice(const PyVal &e, bool gather);
    Status op_concat(const PyVal &e);
    Status finish();
    void hoist_state_moves();
    std::map<std::string, std::pair<int, std::vector<TVal>>> concats_;  // name -> (axis, parts)
    void fold_gathers_into_convs();
};

// Appends Y = X . W^T + bias (W[m][k] = w_mk[m + M*k], the Fortran (M,K)
// array) as a layer of the MLP step producing x, or starts an MLP step.
Status Builder::push_layer(const std::string &name, const TVal &x, int M, int K, const std::vector<double> &w_mk,
                           const std::vector<double> &bias) {
    int rsub = 1;
    if (x.shape.size() == 3 && x.bdim == 1) rsub = (int)x.shape[0];  // (r, batch, K): r sub-rows per sample
    else if (x.shape.size() != 2 || x.bdim != 0)
        return Status::Err(ROSENNA_ERR_UNSUPPORTED, "Gemm/MatMul input must be (batch, K), got " + shape_str(x.shape));
    if (x.shape.back() != K)
        return Status::Err(ROSENNA_ERR_SHAPE, "Gemm/MatMul: input " + shape_str(x.shape) + " vs weights (" + std::to_string(M) + "," +
                                                  std::to_string(K) + ")");
    MlpLayer ly;
    ly.K = K;
    ly.M = M;
    ly.Kp = (int)round_up(K, 8);
    ly.Mp = (int)round_up(M, 8);
    std::vector<float> wt((size_t)ly.Kp * ly.Mp, 0.f), b((size_t)ly.Mp, 0.f);
    for (int k = 0; k < K; k++)
        for (int m = 0; m < M; m++) wt[(size_t)k * ly.Mp + m] = (float)w_mk[(size_t)m + (size_t)M * k];
    for (int m = 0; m < M; m++) b[(size_t)m] = (float)bias[(size_t)m];
    ly.w_off = put(wt.data(), wt.size());
    ly.b_off = put(b.data(), b.size());
    if (M <= 256) {  // tensor-core block: rows n < Np hold tf32(W[n][k]), rows Np + n the rounded remainder
        ly.tc_Kp = (int)round_up(K, 32);
        ly.tc_Np = (int)round_up(M, 16);
        std::vector<float> blk((size_t)2 * ly.tc_Np * ly.tc_Kp, 0.f), tb((size_t)ly.tc_Np, 0.f);
        for (int n = 0; n < M; n++)
            for (int k = 0; k < K; k++) {
                const float w = (float)w_mk[(size_t)n + (size_t)M * k];
                const float hi = tf32_round(w);
                blk[(size_t)n * ly.tc_Kp + k] = hi;
                blk[(size_t)(ly.tc_Np + n) * ly.tc_Kp + k] = tf32_round(w - hi);
            }
        for (int n = 0; n < M; n++) tb[(size_t)n] = (float)bias[(size_t)n];
        ly.tc_w_off = put(blk.data(), blk.size());
        ly.tc_b_off = put(tb.data(), tb.size());
    }
    Step *prev = last_producing(x.buf);
    int out;
    if (prev && prev->kind == Step::MLP && prev->rsub == rsub) {
        prev->layers.push_back(ly);
        out = prev->out;
    } else {
        Step s;
        s.kind = Step::MLP;
        s.in = x.buf;
        s.out = out = new_buf((int64_t)rsub * M);
        s.rsub = rsub;
        s.layers.push_back(ly);
        plan_->steps.push_back(s);
    }
    plan_->buf_rows[(size_t)out] = (int64_t)rsub * M;
    Shape os = x.shape;
    os.back() = M;
    bind(name, TVal{os, x.bdim, out});
    return Status::Ok();
}

Status Builder::op_gemm(const PyVal &e) {  // modelCreator.fpp:87-89, layers.f90:11-23
    TVal x;
    Status st = get(e.at(1).at(0).s, &x);
    if (!st.ok()) return st;
    int transB = (int)e.at(1).at(1).as_int();
    if (n_gemm_ >= (int)mf_.lin.size()) return Status::Err(ROSENNA_ERR_FORMAT, "more Gemm nodes than Gemm weights");
    const LinearWeights &L = mf_.lin[(size_t)n_gemm_++];
    if (transB != 1) return Status::Err(ROSENNA_ERR_UNSUPPORTED, "Gemm with transB=0 (W.inp form) is not supported");
    int M = (int)L.w.dims[0], K = (int)L.w.dims[1];
    if ((int64_t)L.b.v.size() != M) return Status::Err(ROSENNA_ERR_FORMAT, "Gemm: bias size");
    return push_layer(e.at(1).at(0).s, x, M, K, L.w.v, L.b.v);
}

// matmul2D (layers.f90:25-31): inp1 = MATMUL(inp1, inp2) with inp2 a stored
// constant (K, M) -- a bias-free layer with W = inp2^T.  Products of two
// per-sample values, and the rank-3/4 forms, are not batched.
Status Builder::op_matmul(const PyVal &e) {  // modelCreator.fpp:146-149
    const std::string &an = e.at(1).at(0).s, &bn = e.at(1).at(1).s;
    const int rank = (int)e.at(2).at(0).as_int();
    auto it = consts_.find(bn);
    auto vb = vars_.find(bn);
    if (it == consts_.end() || vb == vars_.end() || vb->second.buf != -3)
        return Status::Err(ROSENNA_ERR_UNSUPPORTED, "MatMul whose second operand is not a stored constant");
    if (rank != 2) return Status::Err(ROSENNA_ERR_UNSUPPORTED, "MatMul of rank " + std::to_string(rank) + " (only matmul2D is batched)");
    TVal x;
    Status st = get(an, &x);
    if (!st.ok()) return st;
    const HostArray &W = it->second;
    if (W.dims.size() != 2) return Status::Err(ROSENNA_ERR_SHAPE, "MatMul: constant operand is not 2-D");
    const int K = (int)W.dims[0], M = (int)W.dims[1];
    std::vector<double> w_mk((size_t)M * K), zero((size_t)M, 0.0);
    for (int m = 0; m < M; m++)
        for (int k = 0; k < K; k++) w_mk[(size_t)m + (size_t)M * k] = W.v[(size_t)k + (size_t)K * m];
    return push_layer(an, x, M, K, w_mk, zero);
}

// Add of a stored constant (modelCreator.fpp:137-144): the adder is broadcast
// to trueShape by broadc (layers.f90:351-375), RESHAPEd to the operand's shape
// and added.  Per sample that is one constant per row; it must not depend on
// the sample.  It folds into the bias of the step that produced the operand
// when that step is an MLP (no activation yet) or a conv (no ReLU or pooling
// yet) and the constant is per output unit / channel.
Status Builder::op_add(const PyVal &e) {
    const std::string &name = e.at(1).at(0).s;
    TVal x;
    Status st = get(name, &x);
    if (!st.ok()) return st;
    if (n_add_ >= (int)mf_.add.size()) return Status::Err(ROSENNA_ERR_FORMAT, "more Add nodes than Add layers");
    const HostArray &A = mf_.add[(size_t)n_add_++];
    Shape ts = e.at(2).at(0).ints(), sp = e.at(2).at(1).ints();
    const int rank = (int)e.at(2).at(2).as_int();
    if (ts.size() != 4 || A.dims.size() != 4 || (sp.size() & 1) || rank < 1 || rank > 4 || rank != (int)x.shape.size())
        return Status::Err(ROSENNA_ERR_FORMAT, "Add: malformed entry");
    // broadc: SPREAD along each (dim, copies) pair, RESHAPEd (first elements,
    // column-major) to trueShape(:dim) + the adder's original trailing dims
    std::vector<double> cur = A.v;
    Shape cd = A.dims;
    for (size_t i = 0; i + 1 < sp.size(); i += 2) {
        const int d = (int)sp[i];
        const int64_t n = sp[i + 1];
        if (d < 1 || d > 4 || n < 1) return Status::Err(ROSENNA_ERR_FORMAT, "Add: spread entry");
        int64_t P = 1, rest = 1;
        for (int k = 0; k < d - 1; k++) P *= cd[(size_t)k];
        for (int k = d - 1; k < 4; k++) rest *= cd[(size_t)k];
        std::vector<double> spd((size_t)(P * n * rest));
        for (int64_t b = 0; b < rest; b++)
            for (int64_t k = 0; k < n; k++)
                for (int64_t a = 0; a < P; a++) spd[(size_t)(a + P * (k + n * b))] = cur[(size_t)(a + P * b)];
        Shape nd(4);
        for (int k = 0; k < 4; k++) nd[(size_t)k] = (i + 2 < sp.size()) ? (k < d ? ts[(size_t)k] : A.dims[(size_t)k]) : ts[(size_t)k];
        if (numel(nd) > (int64_t)spd.size()) return Status::Err(ROSENNA_ERR_SHAPE, "Add: broadcast shapes do not fit");
        spd.resize((size_t)numel(nd));
        cur.swap(spd);
        cd = nd;
    }
    int64_t tn = 1;
    for (int k = 4 - rank; k < 4; k++) tn *= ts[(size_t)k];
    if (tn != numel(x.shape) || (int64_t)cur.size() < tn) return Status::Err(ROSENNA_ERR_SHAPE, "Add: adder does not fit its operand");
    // per-sample rows: element (row r, sample b) of x sits at pre_i + pre*(b + B*post_i)
    int64_t pre = 1;
    for (int k = 0; k < x.bdim; k++) pre *= x.shape[(size_t)k];
    const int64_t B = x.shape[(size_t)x.bdim], rows = x.rows();
    std::vector<double> c((size_t)rows);
    for (int64_t r = 0; r < rows; r++) {
        const int64_t pi = r % pre, qi = r / pre;
        c[(size_t)r] = cur[(size_t)(pi + pre * (B * qi))];
        for (int64_t b = 1; b < B; b++)
            if (cur[(size_t)(pi + pre * (b + B * qi))] != c[(size_t)r])
                return Status::Err(ROSENNA_ERR_UNSUPPORTED, "Add: the constant differs between the samples of the export batch");
    }
    Step *prev = last_producing(x.buf);
    if (prev && prev->kind == Step::MLP && prev->layers.back().act == ACT_NONE) {
        MlpLayer &ly = prev->layers.back();
        const int rs = prev->rsub;  // row t + rs*m
        bool per_unit = true;
        for (int64_t r = 0; r < rows && per_unit; r++) per_unit = c[(size_t)r] == c[(size_t)(rs * (r / rs))];
        if (per_unit) {
            for (int m = 0; m < ly.M; m++) {
                plan_->arena[(size_t)(ly.b_off + m)] += (float)c[(size_t)(rs * m)];
                if (ly.tc_b_off >= 0) plan_->arena[(size_t)(ly.tc_b_off + m)] += (float)c[(size_t)(rs * m)];
            }
            return Status::Ok();
        }
    }
    if (prev && prev->kind == Step::CONV && prev->conv && !prev->relu && prev->pool == 0) {
        bool per_channel = true;  // row oc + OC*(h + Ho*w)
        for (int64_t r = 0; r < rows && per_channel; r++) per_channel = c[(size_t)r] == c[(size_t)(r % prev->OC)];
        if (per_channel) {
            for (int oc = 0; oc < prev->OC; oc++) plan_->arena[(size_t)(prev->b_off + oc)] += (float)c[(size_t)oc];
            return Status::Ok();
        }
    }
    std::vector<float> cf((size_t)rows);
    for (int64_t r = 0; r < rows; r++) cf[(size_t)r] = (float)c[(size_t)r];
    Step s;
    s.kind = Step::ADD;
    s.in = x.buf;
    s.out = new_buf(rows);
    s.b_off = put(cf.data(), cf.size());
    plan_->steps.push_back(s);
    x.buf = s.out;
    bind(name, x);
    return Status::Ok();
}

Status Builder::op_act(const PyVal &e, int act) {  // modelCreator.fpp:151-161
    const std::string &name = e.at(1).at(0).s;
    TVal x;
    Status st = get(name, &x);
    if (!st.ok()) return st;
    Step *prev = last_producing(x.buf);
    if (prev && prev->kind == Step::MLP && prev->layers.back().act == ACT_NONE) {
        prev->layers.back().act = act;
        return Status::Ok();
    }
    if (prev && prev->kind == Step::ADD && prev->act == ACT_NONE) {
        prev->act = act;
        return Status::Ok();
    }
    if (prev && prev->kind == Step::CONV && prev->conv && !prev->relu && prev->pool == 0 && act == ACT_RELU) {
        prev->relu = true;
        return Status::Ok();
    }
    Step s;
    s.kind = Step::ACT;
    s.act = act;
    s.in = x.buf;
    s.out = new_buf(x.rows());
    plan_->steps.push_back(s);
    x.buf = s.out;
    bind(name, x);
    return Status::Ok();
}

Status Builder::op_lstm(const PyVal &e) {  // modelCreator.fpp:92-100, layers.f90:62-132
    const std::string &xn = e.at(1).at(0).s, &hn = e.at(1).at(1).s, &cn = e.at(1).at(2).s;
    const std::string &yn = e.at(2).at(0).s;
    int flag = (int)e.at(e.size() - 1).at(0).as_int();
    if (n_lstm_ >= (int)mf_.lstm.size()) return Status::Err(ROSENNA_ERR_FORMAT, "more LSTM nodes than LSTM weights");
    const LstmWeights &L = mf_.lstm[(size_t)n_lstm_++];
    TVal x;
    Status st = get(xn, &x);
    if (!st.ok()) return st;
    if (x.shape.size() != 3 || x.bdim != 1)
        return Status::Err(ROSENNA_ERR_UNSUPPORTED, "LSTM input must be (T, batch, I), got " + shape_str(x.shape));
    int T = (int)x.shape[0], I = (int)x.shape[2];
    if (L.wih.dims.size() != 3 || L.wih.dims[1] % 4) return Status::Err(ROSENNA_ERR_FORMAT, "LSTM weights");
    int H = (int)(L.wih.dims[1] / 4);
    if (L.wih.dims[2] != I || L.whh.dims[1] != 4 * H || L.whh.dims[2] != H || (int64_t)L.bih.v.size() != 4 * H ||
        (int64_t)L.bhh.v.size() != 4 * H)
        return Status::Err(ROSENNA_ERR_SHAPE, "LSTM weight shapes do not match input " + shape_str(x.shape));
    Step s;
    s.kind = Step::LSTM;
    s.in = x.buf;
    s.T = T;
    s.I = I;
    s.H = H;
    s.Ip = (int)round_up(I, 4);
    s.Hp = (int)round_up(H, 2);
    if (flag == 0) {
        TVal h, c;
        if (!(st = get(hn, &h)).ok() || !(st = get(cn, &c)).ok()) return st;
        if (h.rows() != H || c.rows() != H || h.bdim != 1 || c.bdim != 1)
            return Status::Err(ROSENNA_ERR_SHAPE, "LSTM state must be (1, batch, H)");
        s.h0 = h.buf;
        s.c0 = c.buf;
    } else {  // constant initial state from the weights file (modelParserONNX.py:210-226 writes zeros)
        auto constant = [&](const HostArray &a, int64_t *off) -> Status {
            bool zero = true;
            for (double v : a.v) zero = zero && v == 0.0;
            if (zero) return Status::Ok();
            if (a.dims.size() != 3 || a.dims[1] != 1 || a.dims[2] != H)
                return Status::Err(ROSENNA_ERR_UNSUPPORTED, "non-zero constant LSTM state exported at batch > 1");
            std::vector<float> v((size_t)s.Hp, 0.f);
            for (int j = 0; j < H; j++) v[(size_t)j] = (float)a.v[(size_t)j];
            *off = put(v.data(), v.size());
            return Status::Ok();
        };
        if (!(st = constant(L.hid, &s.h0_const)).ok() || !(st = constant(L.cell, &s.c0_const)).ok()) return st;
    }
    // W = [Wih | Whh]^T with gate columns interleaved per unit: column 4j+q is
    // gate q (i, f, g, o; layers.f90:88-93) of unit j, i.e. PyTorch row q*H+j.
    int G = 4 * s.Hp, Kr = s.Ip + s.Hp;
    std::vector<float> wt((size_t)Kr * G, 0.f), bias((size_t)G, 0.f);
    for (int j = 0; j < H; j++)
        for (int q = 0; q < 4; q++) {
            int col = 4 * j + q, r = q * H + j;
            for (int k = 0; k < I; k++) wt[(size_t)k * G + col] = (float)L.wih.v[(size_t)r + (size_t)4 * H * k];
            for (int k = 0; k < H; k++) wt[(size_t)(s.Ip + k) * G + col] = (float)L.whh.v[(size_t)r + (size_t)4 * H * k];
            bias[(size_t)col] = (float)(L.bih.v[(size_t)r] + L.bhh.v[(size_t)r]);
        }
    s.w_off = put(wt.data(), wt.size());
    s.b_off = put(bias.data(), bias.size());
    if (4 * H <= 256) {  // tensor-core block: tf32 hi rows, then the rounded remainders
        const int Np = (int)round_up(4 * H, 16), Ix = (int)round_up(I, 32), Hh = (int)round_up(H, 32);
        const int Kp = Ix + Hh;
        std::vector<float> blk((size_t)2 * Np * Kp, 0.f), tb((size_t)Np, 0.f);
        for (int j = 0; j < H; j++)
            for (int q = 0; q < 4; q++) {
                const int n = 4 * j + q, r = q * H + j;
                for (int k = 0; k < I + H; k++) {
                    const double wv = k < I ? L.wih.v[(size_t)r + (size_t)4 * H * k]
                                            : L.whh.v[(size_t)r + (size_t)4 * H * (k - I)];
                    const int col = k < I ? k : Ix + (k - I);
                    const float w = (float)wv, hi = tf32_round(w);
                    blk[(size_t)n * Kp + col] = hi;
                    blk[(size_t)(Np + n) * Kp + col] = tf32_round(w - hi);
                }
                tb[(size_t)n] = (float)(L.bih.v[(size_t)r] + L.bhh.v[(size_t)r]);
            }
        s.lstm_tc_w_off = put(blk.data(), blk.size());
        s.lstm_tc_b_off = put(tb.data(), tb.size());
        s.lstm_tc_Np = Np;
        s.lstm_tc_Kp = Kp;
        s.lstm_tc_nx = Ix / 32;
        s.lstm_tc_nh = Hh / 32;
    }
    s.y = new_buf((int64_t)T * H);
    s.hn = new_buf(H);
    s.cn = new_buf(H);
    plan_->steps.push_back(s);
    int64_t N = x.shape[1];
    bind(yn, TVal{{T, 1, N, H}, 2, s.y});
    bind(hn, TVal{{1, N, H}, 1, s.hn});
    bind(cn, TVal{{1, N, H}, 1, s.cn});
    return Status::Ok();
}

Status Builder::op_conv(const PyVal &e) {  // modelCreator.fpp:103-105, layers.f90:183-233
    const std::string &name = e.at(1).at(0).s;
    TVal x;
    Status st = get(name, &x);
    if (!st.ok()) return st;
    if (n_conv_ >= (int)mf_.conv.size()) return Status::Err(ROSENNA_ERR_FORMAT, "more Conv nodes than Conv weights");
    const ConvWeights &W = mf_.conv[(size_t)n_conv_++];
    if (x.shape.size() != 4 || x.bdim != 0) return Status::Err(ROSENNA_ERR_UNSUPPORTED, "Conv input must be (batch, C, H, W)");
    auto pads = e.at(2).at(2).ints(), strides = e.at(2).at(3).ints();
    if (pads.size() < 2 || strides.size() < 2) return Status::Err(ROSENNA_ERR_FORMAT, "Conv pads/strides");
    Step s;
    s.kind = Step::CONV;
    s.conv = true;
    s.C = (int)x.shape[1];
    s.Hin = (int)x.shape[2];
    s.Win = (int)x.shape[3];
    s.OC = (int)W.w.dims[0];
    s.KS = (int)W.w.dims[2];
    if (W.w.dims[1] != s.C) return Status::Err(ROSENNA_ERR_SHAPE, "Conv channels");
    if (W.w.dims[3] != s.KS) return Status::Err(ROSENNA_ERR_UNSUPPORTED, "non-square Conv kernel (the reference assumes square)");
    s.pad_h = (int)pads[0];
    s.pad_w = (int)pads[1];
    s.str_h = (int)strides[0];
    s.str_w = (int)strides[1];
    s.Ho = (s.Hin + 2 * s.pad_h - s.KS) / s.str_h + 1;
    s.Wo = (s.Win + 2 * s.pad_w - s.KS) / s.str_w + 1;
    if (s.Ho < 1 || s.Wo < 1 || s.str_h < 1 || s.str_w < 1) return Status::Err(ROSENNA_ERR_SHAPE, "Conv output is empty");
    s.Hq = s.Ho;
    s.Wq = s.Wo;
    std::vector<float> w((size_t)s.OC * s.C * s.KS * s.KS), b((size_t)s.OC);
    for (int oc = 0; oc < s.OC; oc++)
        for (int ic = 0; ic < s.C; ic++)
            for (int kh = 0; kh < s.KS; kh++)
                for (int kw = 0; kw < s.KS; kw++)
                    w[(((size_t)oc * s.C + ic) * s.KS + kh) * s.KS + kw] =
                        (float)W.w.v[(size_t)oc + (size_t)s.OC * (ic + (size_t)s.C * (kh + (size_t)s.KS * kw))];
    for (int oc = 0; oc < s.OC; oc++) b[(size_t)oc] = (float)W.b.v[(size_t)oc];
    s.w_off = put(w.data(), w.size());
    s.b_off = put(b.data(), b.size());
    if (s.KS == 3 && s.str_h == 1 && s.str_w == 1 && s.C <= 8 && s.OC <= 16) {
        std::vector<float> img((size_t)kConvTcBFloats);
        conv_tc_pack(w.data(), s.OC, s.C, img.data());
        s.ctc_off = put(img.data(), img.size());
        if (s.C == 1 && s.OC <= 8) {
            std::vector<float> packed((size_t)kConvTcBFloats / 2);
            conv_pair_pack1(w.data(), s.OC, s.C, packed.data());
            s.ctc_packed_off = put(packed.data(), packed.size());
        }
    }
    s.in = x.buf;
    s.out = new_buf((int64_t)s.OC * s.Ho * s.Wo);
    s.so_c = 1;
    s.so_h = s.OC;
    s.so_w = (int64_t)s.OC * s.Ho;
    plan_->steps.push_back(s);
    bind(name, TVal{{x.shape[0], s.OC, s.Ho, s.Wo}, 0, s.out});
    return Status::Ok();
}

Status Builder::op_pool(const PyVal &e, bool avg) {  // modelCreator.fpp:107-114, layers.f90:236-310
    const std::string &name = e.at(1).at(0).s;
    TVal x;
    Status st = get(name, &x);
    if (!st.ok()) return st;
    int &ctr = avg ? n_avg_ : n_max_;
    const std::vector<int> &ks = avg ? mf_.avgpool : mf_.maxpool;
    if (ctr >= (int)ks.size()) return Status::Err(ROSENNA_ERR_FORMAT, "more pool nodes than pool layers");
    int k = ks[(size_t)ctr++];
    if (x.shape.size() != 4 || x.bdim != 0) return Status::Err(ROSENNA_ERR_UNSUPPORTED, "pool input must be (batch, C, H, W)");
    auto pads = e.at(2).at(1).ints(), strides = e.at(2).at(2).ints();
    if (pads.size() < 2 || strides.size() < 2) return Status::Err(ROSENNA_ERR_FORMAT, "pool pads/strides");
    int C = (int)x.shape[1], H = (int)x.shape[2], W = (int)x.shape[3];
    int Hq = (H + 2 * (int)pads[0] - k) / (int)strides[0] + 1, Wq = (W + 2 * (int)pads[1] - k) / (int)strides[1] + 1;
    if (Hq < 1 || Wq < 1) return Status::Err(ROSENNA_ERR_SHAPE, "pool output is empty");
    if (Hq != Wq)
        return Status::Err(ROSENNA_ERR_UNSUPPORTED,
                           "pooling with a non-square output (the reference writes its columns with MODULO(.,rows))");
    Step *prev = last_producing(x.buf);
    Step *s;
    if (prev && prev->kind == Step::CONV && prev->conv && prev->pool == 0) {
        s = prev;
    } else {
        Step n;
        n.kind = Step::CONV;
        n.conv = false;
        n.C = n.OC = C;
        n.Hin = n.Ho = H;
        n.Win = n.Wo = W;
        n.in = x.buf;
        n.out = new_buf(1);
        plan_->steps.push_back(n);
        s = &plan_->steps.back();
    }
    s->pool = avg ? 2 : 1;
    s->pk = k;
    s->ppad_h = (int)pads[0];
    s->ppad_w = (int)pads[1];
    s->pstr_h = (int)strides[0];
    s->pstr_w = (int)strides[1];
    s->Hq = Hq;
    s->Wq = Wq;
    s->so_c = 1;
    s->so_h = C;
    s->so_w = (int64_t)C * Hq;
    plan_->buf_rows[(size_t)s->out] = (int64_t)C * Hq * Wq;
    bind(name, TVal{{x.shape[0], C, Hq, Wq}, 0, s->out});
    return Status::Ok();
}

Status Builder::op_transpose(const PyVal &e) {  // modelCreator.fpp:117-119
    const std::string &name = e.at(1).at(0).s;
    TVal x;
    Status st = get(name, &x);
    if (!st.ok()) return st;
    auto order = e.at(2).at(0).ints();
    if (order.size() != x.shape.size()) return Status::Err(ROSENNA_ERR_FORMAT, "Transpose order rank");
    Shape S = probe(x), R(order.size()), Rx(order.size());
    int b2 = -1;
    for (size_t i = 0; i < order.size(); i++) {
        if (order[i] < 1 || order[i] > (int64_t)order.size()) return Status::Err(ROSENNA_ERR_FORMAT, "Transpose order");
        R[i] = S[(size_t)order[i] - 1];
        Rx[i] = x.shape[(size_t)order[i] - 1];
        if (order[i] - 1 == x.bdim) b2 = (int)i;
    }
    return move(name, x, Rx, R, b2, fortran_reshape_order_map(S, R, order), S, false);
}

Status Builder::op_reshape(const PyVal &e) {  // modelCreator.fpp:122-130
    const std::string &xn = e.at(1).at(0).s;
    const std::string &on = e.at(2).at(0).s;
    int flag = (int)e.at(e.size() - 1).at(0).as_int();
    if (flag != 0) {
        // reshapeLayers(i) = its own axis reversal, then the RESHAPE with the
        // reversed ORDER: a C-order reshape of the stored constant.  (The
        // reference keeps the reversed array, so its later calls reshape the
        // reversed data; this is the first call's result.)
        if (n_resh_ >= (int)mf_.reshape.size()) return Status::Err(ROSENNA_ERR_FORMAT, "more constant Reshapes than stored constants");
        const HostArray &A = mf_.reshape[(size_t)n_resh_++];
        Shape tgt = e.at(3).at(0).ints();
        if (tgt.empty() || numel(tgt) != A.numel()) return Status::Err(ROSENNA_ERR_SHAPE, "Reshape size mismatch");
        HostArray out;
        out.dims = tgt;
        out.v.resize((size_t)A.numel());
        const Shape &ad = A.dims;
        std::vector<int64_t> ia(ad.size(), 0), it(tgt.size(), 0);
        for (int64_t q = 0; q < A.numel(); q++) {  // q: C-order position in both
            int64_t la = 0, lt = 0, sa = 1, stt = 1;
            for (size_t k = 0; k < ad.size(); k++) { la += ia[k] * sa; sa *= ad[k]; }
            for (size_t k = 0; k < tgt.size(); k++) { lt += it[k] * stt; stt *= tgt[k]; }
            out.v[(size_t)lt] = A.v[(size_t)la];
            for (size_t k = ad.size(); k-- > 0;) { if (++ia[k] < ad[k]) break; ia[k] = 0; }
            for (size_t k = tgt.size(); k-- > 0;) { if (++it[k] < tgt[k]) break; it[k] = 0; }
        }
        consts_[on] = std::move(out);
        bind(on, TVal{tgt, 0, -3});
        return Status::Ok();
    }
    TVal x;
    Status st = get(xn, &x);
    if (!st.ok()) return st;
    Shape tgt = e.at(3).at(0).ints();
    if (tgt.empty() || numel(tgt) != numel(x.shape)) return Status::Err(ROSENNA_ERR_SHAPE, "Reshape size mismatch");
    if (tgt[0] % B0_) return Status::Err(ROSENNA_ERR_UNSUPPORTED, "Reshape target does not lead with the batch");
    Shape S = probe(x);
    // out = C-order reshape of x.  A target whose first dim is r*batch (r > 1)
    // keeps r sub-rows per sample: it is held as (r, batch, ...) with the batch
    // second, which has the same column-major element order.
    int64_t r = tgt[0] / B0_;
    Shape Tfull = tgt, Tx, Tp;
    Tfull[0] = r * kProbe;
    int b2;
    if (r == 1) {
        Tx = tgt;
        Tp = Tfull;
        b2 = 0;
    } else {
        Tx = {r, B0_};
        Tp = {r, kProbe};
        Tx.insert(Tx.end(), tgt.begin() + 1, tgt.end());
        Tp.insert(Tp.end(), tgt.begin() + 1, tgt.end());
        b2 = 1;
    }
    TVal ox = x;
    if (!(st = move(on, x, Tx, Tp, b2, c_order_reshape_map(S, Tfull), S, false)).ok()) return st;
    // side effect of modelCreator.fpp:125: x itself is left with its axes reversed
    int rk = (int)x.shape.size();
    Shape Rv(x.shape.rbegin(), x.shape.rend()), Rp(S.rbegin(), S.rend());
    std::vector<int64_t> ord((size_t)rk);
    for (int i = 0; i < rk; i++) ord[(size_t)i] = rk - i;
    return move(xn, ox, Rv, Rp, rk - 1 - x.bdim, fortran_reshape_order_map(S, Rp, ord), S, true);
}

Status Builder::op_squeeze(const PyVal &e) {  // modelCreator.fpp:133-135
    const std::string &xn = e.at(1).at(0).s;
    const std::string &on = e.at(2).at(0).s;
    TVal x;
    Status st = get(xn, &x);
    if (!st.ok()) return st;
    auto axes = e.at(3).at(0).ints();
    Shape R;
    int b2 = x.bdim;
    for (int i = 0; i < (int)x.shape.size(); i++) {
        bool sq = std::find(axes.begin(), axes.end(), (int64_t)i) != axes.end();
        if (!sq) { R.push_back(x.shape[(size_t)i]); continue; }
        if (i == x.bdim) return Status::Err(ROSENNA_ERR_UNSUPPORTED, "Squeeze of the batch dimension");
        if (x.shape[(size_t)i] != 1) return Status::Err(ROSENNA_ERR_SHAPE, "Squeeze of a non-unit dimension");
        if (i < x.bdim) b2--;
    }
    bind(on, TVal{R, b2, x.buf});  // same element order: no data movement
    return Status::Ok();
}

// ONNX Slice (axes/starts/ends, step 1) and Gather (one index, axis dropped),
// written as architecture entries by this build's front end (the reference
// parser passes them through, modelParserONNX.py:519-523): data movement
// through a per-sample row map, or a whole part of a Concat.
Status Builder::op_slice(const PyVal &e, bool gather) {
    const std::string &xn = e.at(1).at(0).s, &on = e.at(2).at(0).s;
    const PyVal &prm = e.at(3);
    auto cit = concats_.find(xn);
    std::vector<int64_t> axes, starts, ends;
    if (gather) {
        axes = {prm.at(0).as_int()};
        starts = {prm.at(1).as_int()};
        ends = {starts[0] + 1};
    } else {
        axes = prm.at(0).ints();
        starts = prm.at(1).ints();
        ends = prm.at(2).ints();
        if (axes.size() != starts.size() || axes.size() != ends.size())
            return Status::Err(ROSENNA_ERR_FORMAT, "Slice parameters");
    }
    TVal x;
    if (cit != concats_.end()) {
        // a selection of exactly one part of a Concat reads that part
        const int cax = cit->second.first;
        const auto &parts = cit->second.second;
        const int rank = (int)parts[0].shape.size();
        if (axes.size() != 1 || (axes[0] < 0 ? axes[0] + rank : axes[0]) != cax)
            return Status::Err(ROSENNA_ERR_UNSUPPORTED, "a Slice/Gather of a Concat must select along its axis");
        int64_t total = 0;
        for (auto &p : parts) total += p.shape[(size_t)cax];
        int64_t a = starts[0] < 0 ? starts[0] + total : starts[0];
        int64_t b = ends[0] < 0 ? ends[0] + total : std::min(ends[0], total);
        if (gather) b = a + 1;
        int64_t off = 0;
        const TVal *hit = nullptr;
        for (auto &p : parts) {
            if (a == off && b == off + p.shape[(size_t)cax]) hit = &p;
            off += p.shape[(size_t)cax];
        }
        if (!hit) return Status::Err(ROSENNA_ERR_UNSUPPORTED, "a Slice/Gather of a Concat must select one whole part");
        TVal v = *hit;
        if (gather) {  // drop the (unit) axis
            if (v.shape[(size_t)cax] != 1 || cax == v.bdim) return Status::Err(ROSENNA_ERR_UNSUPPORTED, "Gather of a Concat part");
            v.shape.erase(v.shape.begin() + cax);
            if (cax < v.bdim) v.bdim--;
        }
        concats_.erase(on);
        bind(on, v);
        return Status::Ok();
    }
    Status st = get(xn, &x);
    if (!st.ok()) return st;
    const int rank = (int)x.shape.size();
    Shape lo(rank, 0), hi = x.shape;
    for (size_t j = 0; j < axes.size(); j++) {
        int ax = (int)(axes[j] < 0 ? axes[j] + rank : axes[j]);
        if (ax < 0 || ax >= rank) return Status::Err(ROSENNA_ERR_FORMAT, "Slice axis");
        if (ax == x.bdim) return Status::Err(ROSENNA_ERR_UNSUPPORTED, "Slice of the batch dimension");
        int64_t d = x.shape[(size_t)ax];
        int64_t a = starts[j] < 0 ? starts[j] + d : starts[j], b = ends[j] < 0 ? ends[j] + d : ends[j];
        a = std::max<int64_t>(0, std::min(a, d));
        b = std::max(a, std::min(b, d));
        if (gather) b = a + 1;
        if (b <= a) return Status::Err(ROSENNA_ERR_SHAPE, "empty Slice");
        lo[(size_t)ax] = a;
        hi[(size_t)ax] = b;
    }
    const int drop = gather ? (int)(axes[0] < 0 ? axes[0] + rank : axes[0]) : -1;
    Shape S = probe(x), box(rank), R, Rx;
    int b2 = x.bdim;
    for (int i = 0; i < rank; i++) {
        box[(size_t)i] = i == x.bdim ? S[(size_t)i] : hi[(size_t)i] - lo[(size_t)i];
        if (i == drop) {
            if (i < x.bdim) b2--;
            continue;
        }
        R.push_back(box[(size_t)i]);
        Rx.push_back(i == x.bdim ? x.shape[(size_t)i] : box[(size_t)i]);
    }
    // result element L (column-major over the box) <- source element at box index + lo
    std::vector<int64_t> r2s((size_t)numel(box));
    std::vector<int64_t> sub((size_t)rank);
    for (int64_t L = 0; L < numel(box); L++) {
        unravel(L, box, sub.data());
        for (int i = 0; i < rank; i++) sub[(size_t)i] += i == x.bdim ? 0 : lo[(size_t)i];
        r2s[(size_t)L] = ravel(sub.data(), S);
    }
    concats_.erase(on);
    return move(on, x, Rx, R, b2, r2s, S, false);
}

// ONNX Concat (see op_slice): kept as its parts; only a Slice/Gather that
// selects one whole part may read it (a stacked LSTM's h_n, read as h_n[-1]).
Status Builder::op_concat(const PyVal &e) {
    const std::string &on = e.at(2).at(0).s;
    const int64_t axis = e.at(3).at(0).as_int();
    std::vector<TVal> parts;
    for (auto &n : e.at(1).items) {
        TVal v;
        Status st = get(n.s, &v);
        if (!st.ok()) return st;
        parts.push_back(v);
    }
    if (parts.empty()) return Status::Err(ROSENNA_ERR_FORMAT, "Concat without inputs");
    const int rank = (int)parts[0].shape.size();
    const int ax = (int)(axis < 0 ? axis + rank : axis);
    Shape shape = parts[0].shape;
    shape[(size_t)ax] = 0;
    for (auto &p : parts) {
        if ((int)p.shape.size() != rank || p.bdim != parts[0].bdim || ax == p.bdim)
            return Status::Err(ROSENNA_ERR_UNSUPPORTED, "Concat operands");
        shape[(size_t)ax] += p.shape[(size_t)ax];
    }
    bind(on, TVal{shape, parts[0].bdim, -4});
    concats_[on] = {ax, parts};
    return Status::Ok();
}

Status Builder::finish() {
    const ModelFiles &m = mf_;
    // outputs: o<index> = outputs[<index>-th key]  (modelCreator.fpp:169-171)
    std::set<int> used;
    for (auto &io : plan_->inputs) used.insert(io.buf);
    for (size_t i = 0; i < m.out_shape.size(); i++) {
        if (i >= m.outputs.items.size()) return Status::Err(ROSENNA_ERR_FORMAT, "outputs dict shorter than outShape");
        TVal v;
        Status st = get(m.outputs.items[i].s, &v);
        if (!st.ok()) return st;
        IoDesc d;
        d.shape = m.out_shape.at(i).at(1).ints();
        if (numel(d.shape) != numel(v.shape))
            return Status::Err(ROSENNA_ERR_SHAPE, "output " + std::to_string(i) + " size differs from outShape");
        d.pre = 1;
        for (int k = 0; k < v.bdim; k++) d.pre *= v.shape[(size_t)k];
        d.bdim = v.bdim;
        d.rows = v.rows();
        d.buf = v.buf;
        if (used.count(d.buf)) {  // an input (or another output) would be aliased: copy
            Step s;
            s.kind = Step::COPY;
            s.in = d.buf;
            s.out = d.buf = new_buf(d.rows);
            plan_->steps.push_back(s);
        }
        used.insert(d.buf);
        plan_->outputs.push_back(d);
    }
    // drop steps whose results nobody reads
    std::set<int> live;
    for (auto &o : plan_->outputs) live.insert(o.buf);
    std::vector<Step> kept;
    for (size_t i = plan_->steps.size(); i-- > 0;) {
        Step s = plan_->steps[i];
        bool alive;
        if (s.kind == Step::LSTM) {
            if (!live.count(s.y)) s.y = -1;
            if (!live.count(s.hn)) s.hn = -1;
            if (!live.count(s.cn)) s.cn = -1;
            alive = s.y >= 0 || s.hn >= 0 || s.cn >= 0;
        } else {
            alive = live.count(s.out) > 0;
        }
        if (!alive) continue;
        live.insert(s.in);
        if (s.h0 >= 0) live.insert(s.h0);
        if (s.c0 >= 0) live.insert(s.c0);
        kept.push_back(s);
    }
    std::reverse(kept.begin(), kept.end());
    plan_->steps = kept;
    fold_gathers_into_convs();
    hoist_state_moves();
    return Status::Ok();
}

// A stacked LSTM's later layers take their initial state through data movement
// (a Slice of the (L, N, H) state: a gather) issued between the layers.  Such
// steps read nothing the earlier layer writes, so they move in front of it and
// the two layers become adjacent (the runtime can then fuse them).
void Builder::hoist_state_moves() {
    auto &steps = plan_->steps;
    for (size_t j = 0; j < steps.size(); j++) {
        if (steps[j].kind != Step::LSTM) continue;
        size_t k = j + 1;
        while (k < steps.size() && (steps[k].kind == Step::GATHER || steps[k].kind == Step::COPY ||
                                    steps[k].kind == Step::DEINTERLEAVE))
            k++;
        if (k == j + 1 || k >= steps.size() || steps[k].kind != Step::LSTM || steps[k].in != steps[j].y) continue;
        bool independent = true;
        for (size_t m = j + 1; m < k; m++)
            for (int b : {steps[j].y, steps[j].hn, steps[j].cn})
                if (b >= 0 && steps[m].in == b) independent = false;
        if (!independent) continue;
        std::rotate(steps.begin() + (std::ptrdiff_t)j, steps.begin() + (std::ptrdiff_t)j + 1,
                    steps.begin() + (std::ptrdiff_t)k);
        // steps j..k-2 are now the moves, k-1 the first LSTM, k the second
    }
}

// A gather that only permutes the rows a conv/pool step just wrote (the C-order
// flatten of a (C, H, W) result, modelCreator.fpp:122-130) folds into that
// step: the kernels write output row c*so_c + h*so_h + w*so_w, so when the
// permutation maps (c, h, w) affinely the step writes the gathered order
// directly and the gather pass goes away.
void Builder::fold_gathers_into_convs() {
    auto &steps = plan_->steps;
    for (size_t i = 1; i < steps.size(); i++) {
        Step &g = steps[i], &c = steps[i - 1];
        if (g.kind != Step::GATHER || c.kind != Step::CONV || c.out != g.in) continue;
        bool other_reader = false;
        for (size_t k = 0; k < steps.size(); k++)
            if (k != i && (steps[k].in == c.out || steps[k].h0 == c.out || steps[k].c0 == c.out)) other_reader = true;
        for (auto *v : {&plan_->inputs, &plan_->outputs})
            for (auto &io : *v)
                if (io.buf == c.out) other_reader = true;
        const int64_t rows = plan_->buf_rows[(size_t)g.out];
        if (other_reader || rows != plan_->buf_rows[(size_t)c.out] || rows != (int64_t)c.OC * c.Hq * c.Wq) continue;
        const int32_t *map = reinterpret_cast<const int32_t *>(plan_->arena.data() + g.map_off);
        std::vector<int64_t> inv((size_t)rows, -1);
        bool perm = true;
        for (int64_t r = 0; r < rows && perm; r++) {
            const int64_t src = map[r];
            if (src < 0 || src >= rows || inv[(size_t)src] >= 0) perm = false;
            else inv[(size_t)src] = r;
        }
        if (!perm) continue;
        auto old_row = [&](int64_t ch, int64_t h, int64_t w) { return ch * c.so_c + h * c.so_h + w * c.so_w; };
        const int64_t r0 = inv[(size_t)old_row(0, 0, 0)];
        const int64_t sc = c.OC > 1 ? inv[(size_t)old_row(1, 0, 0)] - r0 : 1;
        const int64_t sh = c.Hq > 1 ? inv[(size_t)old_row(0, 1, 0)] - r0 : 1;
        const int64_t sw = c.Wq > 1 ? inv[(size_t)old_row(0, 0, 1)] - r0 : 1;
        bool affine = r0 == 0;
        for (int64_t ch = 0; ch < c.OC && affine; ch++)
            for (int64_t h = 0; h < c.Hq && affine; h++)
                for (int64_t w = 0; w < c.Wq && affine; w++)
                    affine = inv[(size_t)old_row(ch, h, w)] == ch * sc + h * sh + w * sw;
        if (!affine) continue;
        c.so_c = sc;
        c.so_h = sh;
        c.so_w = sw;
        c.out = g.out;
        steps.erase(steps.begin() + (std::ptrdiff_t)i);
        i--;
    }
}

Status Builder::run() {
    const PyVal &arch = mf_.architecture;
    // batch dimension of each model input: 1 when the first entry that reads it
    // is an LSTM (X is (T,N,I), h/c are (1,N,H)) or a Slice (a stacked LSTM's
    // (L,N,H) initial state), else 0
    std::set<std::string> lstm_operands, seen;
    for (auto &e : arch.items) {
        std::vector<std::string> names;
        const PyVal &a1 = e.at(1);
        if (a1.is_list()) {
            for (auto &n : a1.items)
                if (n.kind == PyVal::STR) names.push_back(n.s);
        }
        for (auto &n : names) {
            if (seen.count(n)) continue;
            seen.insert(n);
            if (e.at(0).s == "LSTM" || e.at(0).s == "Slice") lstm_operands.insert(n);
        }
    }
    for (size_t i = 0; i < mf_.true_inputs.size(); i++) {
        const PyVal &ti = mf_.true_inputs.at(i);
        IoDesc d;
        d.shape = ti.at(1).ints();
        if (d.shape.empty()) return Status::Err(ROSENNA_ERR_FORMAT, "input without shape");
        d.bdim = lstm_operands.count(ti.at(0).s) && d.shape.size() >= 2 ? 1 : 0;
        int64_t b = d.shape[(size_t)d.bdim];
        if (i == 0) B0_ = b;
        else if (b != B0_) return Status::Err(ROSENNA_ERR_SHAPE, "inputs disagree on the export batch size");
        d.pre = 1;
        for (int k = 0; k < d.bdim; k++) d.pre *= d.shape[(size_t)k];
        d.rows = numel(d.shape) / b;
        d.buf = new_buf(d.rows);
        plan_->inputs.push_back(d);
        int vbuf = d.buf;
        if (d.pre > 1) {  // samples are strided in the reference layout: rows of samples first
            Step s;
            s.kind = Step::DEINTERLEAVE;
            s.in = d.buf;
            s.out = vbuf = new_buf(d.rows);
            s.pre = d.pre;
            plan_->steps.push_back(s);
        }
        bind(ti.at(0).s, TVal{d.shape, d.bdim, vbuf});
    }
    plan_->export_batch = B0_;
    for (auto &e : arch.items) {
        const std::string &op = e.at(0).s;
        Status st;
        if (op == "Gemm") st = op_gemm(e);
        else if (op == "MatMul") st = op_matmul(e);
        else if (op == "Add") st = op_add(e);
        else if (op == "Relu") st = op_act(e, ACT_RELU);
        else if (op == "Tanh") st = op_act(e, ACT_TANH);
        else if (op == "Sigmoid") st = op_act(e, ACT_SIGMOID);
        else if (op == "LSTM") st = op_lstm(e);
        else if (op == "Conv") st = op_conv(e);
        else if (op == "MaxPool") st = op_pool(e, false);
        else if (op == "AveragePool") st = op_pool(e, true);
        else if (op == "Transpose") st = op_transpose(e);
        else if (op == "Reshape") st = op_reshape(e);
        else if (op == "Squeeze") st = op_squeeze(e);
        else if (op == "Slice") st = op_slice(e, false);
        else if (op == "Gather") st = op_slice(e, true);
        else if (op == "Concat") st = op_concat(e);
        else st = Status::Err(ROSENNA_ERR_UNSUPPORTED, "op " + op + " is not supported by the engine");
        if (!st.ok()) return st;
    }
    return finish();
}

}  // namespace

Status build_plan(const ModelFiles &mf, Plan *plan) {
    *plan = Plan();
    Builder b(mf, plan);
    return b.run();
}

std::string Plan::describe() const {
    std::ostringstream o;
    static const char *acts[] = {"", "relu", "tanh", "sigmoid"};
    for (size_t si = 0; si < steps.size(); si++) {
        const Step &s = steps[si];
        if (s.kind == Step::LSTM && s.fuse_next) o << "lstm2_tc (fused with the next step) ";
        if (s.kind == Step::CONV && s.fuse_next) o << "conv_pair_tc (fused with the next step) ";
        if (si > 0 && steps[si - 1].fuse_next) o << (steps[si - 1].kind == Step::CONV ? "(in conv_pair_tc) " : "(in lstm2_tc) ");
        switch (s.kind) {
            case Step::MLP:
                o << (s.tc ? "mlp_tc b" : "mlp b") << s.in << "->b" << s.out << " [";
                for (size_t i = 0; i < s.layers.size(); i++)
                    o << (i ? " " : "") << s.layers[i].K << "x" << s.layers[i].M << (s.layers[i].act ? ":" : "")
                      << acts[s.layers[i].act];
                o << "]\n";
                break;
            case Step::LSTM:
                o << (s.tc ? (s.lstm_dual ? "lstm_tc_dual b" : "lstm_tc b") : "lstm b") << s.in << " T=" << s.T << " I=" << s.I << " H=" << s.H << " h0=b" << s.h0 << " c0=b"
                  << s.c0 << " -> y=b" << s.y << " hn=b" << s.hn << " cn=b" << s.cn << "\n";
                break;
            case Step::CONV:
                o << (s.conv ? (s.tc ? "conv_tc" : "conv") : "pool") << " b" << s.in << "->b" << s.out << " C=" << s.C << " " << s.Hin << "x"
                  << s.Win;
                if (s.conv) o << " OC=" << s.OC << " k=" << s.KS << " pad=" << s.pad_h << "," << s.pad_w << " s=" << s.str_h << "," << s.str_w;
                if (s.relu) o << " relu";
                if (s.pool) o << (s.pool == 1 ? " maxpool" : " avgpool") << " k=" << s.pk << " s=" << s.pstr_h;
                o << " -> " << s.Hq << "x" << s.Wq << "\n";
                break;
            case Step::GATHER: o << "gather b" << s.in << "->b" << s.out << "\n"; break;
            case Step::ACT: o << "act:" << acts[s.act] << " b" << s.in << "->b" << s.out << "\n"; break;
            case Step::ADD: o << "add" << (s.act ? "+" : "") << acts[s.act] << " b" << s.in << "->b" << s.out << "\n"; break;
            case Step::COPY: o << "copy b" << s.in << "->b" << s.out << "\n"; break;
            case Step::DEINTERLEAVE: o << "deinterleave b" << s.in << "->b" << s.out << " pre=" << s.pre << "\n"; break;
        }
    }
    return o.str();
}

}  // namespace rosenna
