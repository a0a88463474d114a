// Readers for roseNNa's model files.
//
// onnxModel.txt / onnxWeights.txt follow fLibrary/reader.f90:38-290: the model
// file starts with a node count, then each node's op name and, for ops that
// carry tensors, one dims line per tensor; the weights file holds one tensor per
// line in Fortran order.  Each tensor is one Fortran list-directed READ: it
// starts on a fresh line, may continue over lines, and skips the rest of its
// last line.  A node-name READ that hits end of file ends the loop
// (reader.f90:55-58), so the node count is an upper bound.
#include "model_files.hpp"

#include <cctype>
#include <charconv>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <sstream>

#include "../../include/rosenna.h"

namespace rosenna {

static const PyVal kNone;

const PyVal &PyVal::at(size_t j) const { return j < items.size() ? items[j] : kNone; }

std::vector<int64_t> PyVal::ints() const {
    std::vector<int64_t> r;
    if (kind == LIST)
        for (auto &x : items) r.push_back(x.as_int());
    return r;
}

namespace {

struct LitParser {
    const std::string &s;
    size_t p = 0;
    std::string err;

    void ws() {
        while (p < s.size() && std::isspace((unsigned char)s[p])) p++;
    }
    bool fail(const char *why) {
        if (err.empty()) err = std::string(why) + " at offset " + std::to_string(p);
        return false;
    }
    bool value(PyVal *v) {
        ws();
        if (p >= s.size()) return fail("unexpected end");
        char c = s[p];
        if (c == '[' || c == '(') return seq(v, c == '[' ? ']' : ')', false);
        if (c == '{') return seq(v, '}', true);
        if (c == '\'' || c == '"') {
            size_t e = s.find(c, p + 1);
            if (e == std::string::npos) return fail("unterminated string");
            v->kind = PyVal::STR;
            v->s = s.substr(p + 1, e - p - 1);
            p = e + 1;
            return true;
        }
        if (s.compare(p, 4, "None") == 0) { v->kind = PyVal::NONE; p += 4; return true; }
        if (s.compare(p, 4, "True") == 0) { v->kind = PyVal::INT; v->i = 1; p += 4; return true; }
        if (s.compare(p, 5, "False") == 0) { v->kind = PyVal::INT; v->i = 0; p += 5; return true; }
        if (s.compare(p, 3, "np.") == 0) {  // numpy scalar repr, e.g. np.int64(3)
            size_t o = s.find('(', p);
            if (o == std::string::npos) return fail("bad numpy scalar");
            p = o + 1;
            if (!value(v)) return false;
            ws();
            if (p >= s.size() || s[p] != ')') return fail("bad numpy scalar");
            p++;
            return true;
        }
        if (c == '-' || c == '+' || c == '.' || std::isdigit((unsigned char)c)) {
            size_t e = p + 1;
            bool flt = false;
            while (e < s.size() && (std::isalnum((unsigned char)s[e]) || s[e] == '.' ||
                                    ((s[e] == '-' || s[e] == '+') && (s[e - 1] == 'e' || s[e - 1] == 'E')))) {
                if (s[e] == '.' || s[e] == 'e' || s[e] == 'E') flt = true;
                e++;
            }
            std::string tok = s.substr(p, e - p);
            char *end = nullptr;
            if (flt) {
                v->kind = PyVal::FLOAT;
                v->f = std::strtod(tok.c_str(), &end);
            } else {
                v->kind = PyVal::INT;
                v->i = std::strtoll(tok.c_str(), &end, 10);
                v->f = (double)v->i;
            }
            if (!end || *end) return fail("bad number");
            p = e;
            return true;
        }
        return fail("unexpected character");
    }
    bool seq(PyVal *v, char close, bool dict) {
        v->kind = dict ? PyVal::DICT : PyVal::LIST;
        p++;
        for (;;) {
            ws();
            if (p < s.size() && s[p] == close) { p++; return true; }
            PyVal key, item;
            if (dict) {
                if (!value(&key)) return false;
                ws();
                if (p >= s.size() || s[p] != ':') return fail("expected ':'");
                p++;
            }
            if (!value(&item)) return false;
            v->items.push_back(std::move(item));
            if (dict) v->keys.push_back(std::move(key));
            ws();
            if (p < s.size() && s[p] == ',') { p++; continue; }
            if (p < s.size() && s[p] == close) { p++; return true; }
            return fail("expected ',' or closing bracket");
        }
    }
};

// Line-oriented reader with Fortran list-directed semantics (see file header),
// over the whole file read at once.
struct RecordReader {
    std::string buf;
    size_t pos = 0;
    bool eof = false;
    bool open(const std::string &path) {
        FILE *f = std::fopen(path.c_str(), "rb");
        if (!f) return false;
        char chunk[1 << 16];
        size_t got;
        while ((got = std::fread(chunk, 1, sizeof(chunk), f)) > 0) buf.append(chunk, got);
        const bool ok = !std::ferror(f);
        std::fclose(f);
        return ok;
    }
    // [*b, *e) = the next line without its terminator
    bool next_span(const char **b, const char **e) {
        if (pos >= buf.size()) { eof = true; return false; }
        const char *p = buf.data() + pos, *end = buf.data() + buf.size();
        const char *nl = static_cast<const char *>(std::memchr(p, '\n', (size_t)(end - p)));
        const char *le = nl ? nl : end;
        *b = p;
        *e = (le > p && le[-1] == '\r') ? le - 1 : le;
        pos = (size_t)(le - buf.data()) + (nl ? 1 : 0);
        return true;
    }
    bool next_line(std::string *line) {
        const char *b, *e;
        if (!next_span(&b, &e)) return false;
        line->assign(b, e);
        return true;
    }
    bool numbers(int64_t count, std::vector<double> *out) {
        out->clear();
        out->reserve((size_t)count);
        while ((int64_t)out->size() < count) {
            const char *c, *le;
            if (!next_span(&c, &le)) return false;
            while ((int64_t)out->size() < count) {
                while (c < le && (std::isspace((unsigned char)*c) || *c == ',')) c++;
                if (c >= le) break;
                // from_chars is correctly rounded like strtod and several times
                // faster; strtod takes what it does not accept ('+1.5', hex forms)
                double x;
                auto r = std::from_chars(c, le, x);
                if (r.ec == std::errc() && (r.ptr == le || std::isspace((unsigned char)*r.ptr) || *r.ptr == ',')) {
                    c = r.ptr;
                } else {
                    std::string tok(c, le);
                    char *end = nullptr;
                    x = std::strtod(tok.c_str(), &end);
                    if (end == tok.c_str()) return false;
                    c += end - tok.c_str();
                }
                out->push_back(x);
            }
        }
        return true;
    }
};

bool read_dims(RecordReader &mf, int rank, std::vector<int64_t> *dims) {
    std::vector<double> d;
    if (!mf.numbers(rank, &d)) return false;
    dims->clear();
    for (double x : d) {
        if (x < 0 || x != (double)(int64_t)x) return false;
        dims->push_back((int64_t)x);
    }
    return true;
}

bool read_tensor(RecordReader &mf, RecordReader &wf, int rank, HostArray *a) {
    if (!read_dims(mf, rank, &a->dims)) return false;
    return wf.numbers(a->numel(), &a->v);
}

}  // namespace

bool parse_pyval(const std::string &text, PyVal *out, std::string *err) {
    LitParser lp{text};
    if (!lp.value(out)) {
        if (err) *err = lp.err;
        return false;
    }
    return true;
}

Status read_model_files(const std::string &model_txt, const std::string &weights_txt,
                        const std::string &variables_fpp, ModelFiles *out) {
    RecordReader mf, wf;
    if (!mf.open(model_txt)) return Status::Err(ROSENNA_ERR_IO, "cannot open " + model_txt);
    if (!wf.open(weights_txt)) return Status::Err(ROSENNA_ERR_IO, "cannot open " + weights_txt);

    std::vector<int64_t> cnt;
    if (!read_dims(mf, 1, &cnt)) return Status::Err(ROSENNA_ERR_FORMAT, model_txt + ": missing node count");
    for (int64_t i = 0; i < cnt[0]; i++) {
        std::string line;
        if (!mf.next_line(&line)) break;  // reader.f90:55-58
        std::istringstream ls(line);
        std::string name;
        if (!(ls >> name)) break;
        bool ok = true;
        if (name == "LSTM") {  // read_lstm, reader.f90:203-252
            std::vector<int64_t> flag;
            LstmWeights L;
            ok = read_dims(mf, 1, &flag) && read_tensor(mf, wf, 3, &L.wih) && read_tensor(mf, wf, 3, &L.whh) &&
                 read_tensor(mf, wf, 1, &L.bih) && read_tensor(mf, wf, 1, &L.bhh);
            if (ok && flag[0] == 1) {
                ok = read_tensor(mf, wf, 3, &L.hid) && read_tensor(mf, wf, 3, &L.cell);
                L.has_consts = true;
            }
            out->lstm.push_back(std::move(L));
        } else if (name == "Gemm") {  // read_linear, reader.f90:254-287
            LinearWeights L;
            ok = read_tensor(mf, wf, 2, &L.w) && read_tensor(mf, wf, 1, &L.b);
            out->lin.push_back(std::move(L));
        } else if (name == "Conv") {  // read_conv, reader.f90:178-201
            ConvWeights C;
            ok = read_tensor(mf, wf, 4, &C.w) && read_tensor(mf, wf, 1, &C.b);
            out->conv.push_back(std::move(C));
        } else if (name == "MaxPool" || name == "AveragePool") {  // reader.f90:157-177
            std::vector<int64_t> k;
            ok = read_dims(mf, 1, &k);
            if (ok) (name == "MaxPool" ? out->maxpool : out->avgpool).push_back((int)k[0]);
        } else if (name == "Add") {  // read_add, reader.f90:143-155
            HostArray a;
            ok = read_tensor(mf, wf, 4, &a);
            out->add.push_back(std::move(a));
        } else if (name == "Reshape") {  // reader.f90:74-82, 101-141
            std::vector<int64_t> flag;
            ok = read_dims(mf, 1, &flag);
            if (ok && flag[0] >= 2 && flag[0] <= 4) {
                HostArray a;
                ok = read_tensor(mf, wf, (int)flag[0], &a);
                out->reshape.push_back(std::move(a));
            }
        }
        if (!ok) return Status::Err(ROSENNA_ERR_FORMAT, "malformed model files at node " + std::to_string(i + 1) + " (" + name + ")");
    }

    std::ifstream vf(variables_fpp);
    if (!vf) return Status::Err(ROSENNA_ERR_IO, "cannot open " + variables_fpp);
    std::string line;
    int found = 0;
    while (std::getline(vf, line)) {
        size_t p = line.find("#:set");
        if (p == std::string::npos) continue;
        p += 5;
        while (p < line.size() && std::isspace((unsigned char)line[p])) p++;
        size_t q = p;
        while (q < line.size() && (std::isalnum((unsigned char)line[q]) || line[q] == '_')) q++;
        std::string key = line.substr(p, q - p);
        size_t eq = line.find('=', q);
        if (eq == std::string::npos) return Status::Err(ROSENNA_ERR_FORMAT, variables_fpp + ": bad #:set line");
        PyVal v;
        std::string err;
        if (!parse_pyval(line.substr(eq + 1), &v, &err))
            return Status::Err(ROSENNA_ERR_FORMAT, variables_fpp + ": " + key + ": " + err);
        PyVal *slot = key == "architecture" ? &out->architecture
                      : key == "inputs"     ? &out->inputs
                      : key == "trueInputs" ? &out->true_inputs
                      : key == "outShape"   ? &out->out_shape
                      : key == "outputs"    ? &out->outputs
                                            : nullptr;
        if (slot) {
            *slot = std::move(v);
            found++;
        }
    }
    if (!out->architecture.is_list() || !out->true_inputs.is_list() || !out->out_shape.is_list() ||
        out->outputs.kind != PyVal::DICT)
        return Status::Err(ROSENNA_ERR_FORMAT, variables_fpp + " lacks architecture/trueInputs/outShape/outputs");
    return Status::Ok();
}

}  // namespace rosenna
