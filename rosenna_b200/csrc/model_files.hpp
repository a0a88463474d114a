// Model files of roseNNa: onnxModel.txt + onnxWeights.txt (read as
// fLibrary/reader.f90:38-290 reads them) and variables.fpp (the Python-literal
// `#:set` lines fLibrary/modelParserONNX.py:531-541 writes).
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace rosenna {

struct Status {
    int code = 0;
    std::string msg;
    bool ok() const { return code == 0; }
    static Status Ok() { return Status(); }
    static Status Err(int c, std::string m) {
        Status s;
        s.code = c;
        s.msg = std::move(m);
        return s;
    }
};

// Fortran array: logical dims, values in column-major order.
struct HostArray {
    std::vector<int64_t> dims;
    std::vector<double> v;
    int64_t numel() const {
        int64_t n = 1;
        for (auto d : dims) n *= d;
        return n;
    }
};

struct LinearWeights { HostArray w, b; };                              // linLayer
struct LstmWeights { HostArray wih, whh, bih, bhh, hid, cell; bool has_consts = false; };  // lstmLayer
struct ConvWeights { HostArray w, b; };                                // convLayer

// A Python literal (lists, tuples, dicts, strings, ints, floats, None).
struct PyVal {
    enum Kind { NONE, INT, FLOAT, STR, LIST, DICT } kind = NONE;
    int64_t i = 0;
    double f = 0;
    std::string s;
    std::vector<PyVal> items;
    std::vector<PyVal> keys;  // DICT only

    const PyVal &at(size_t j) const;
    size_t size() const { return items.size(); }
    bool is_list() const { return kind == LIST; }
    int64_t as_int() const { return kind == FLOAT ? (int64_t)f : i; }
    std::vector<int64_t> ints() const;
};

bool parse_pyval(const std::string &text, PyVal *out, std::string *err);

struct ModelFiles {
    std::vector<LinearWeights> lin;
    std::vector<LstmWeights> lstm;
    std::vector<ConvWeights> conv;
    std::vector<int> maxpool, avgpool;
    std::vector<HostArray> add, reshape;
    PyVal architecture, inputs, true_inputs, out_shape, outputs;
};

Status read_model_files(const std::string &model_txt, const std::string &weights_txt,
                        const std::string &variables_fpp, ModelFiles *out);

}  // namespace rosenna
