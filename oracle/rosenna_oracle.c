/*
 * rosenna_oracle.c -- CPU oracle for roseNNa's use_model hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker used by tests/, by
 * __graft_entry__.smoke() and by bench.py's cpu_baseline leg.  The product
 * (rosenna_b200/) never links, loads or calls it.
 *
 * It is an fp64 restatement of roseNNa's Fortran library, written in C because
 * no Fortran compiler exists in this image (the reference cannot be built):
 *   - the weight reader             fLibrary/reader.f90:38-290
 *   - the layers                    fLibrary/layers.f90:11-375
 *   - the activations               fLibrary/activation_funcs.f90:7-64
 *   - the generated use_model body  fLibrary/modelCreator.fpp:42-171
 * The generated use_model is a straight-line Fortran program that fypp expands
 * from the `architecture` list in variables.fpp.  Here that list is parsed and
 * interpreted op by op with the same semantics, including the reference's
 * quirks (column index of pooled outputs, in-place axis reversal on Reshape,
 * zero padding for max pooling, avg-pool divisor k*k).
 *
 * Arrays are Fortran arrays: column-major, logical shape = the ONNX shape.
 */
#include <ctype.h>
#include <math.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define MAXR 6

typedef struct {
    int rank;
    int d[MAXR];
    double *v;
} Arr;

static int64_t arr_numel(const Arr *a) {
    int64_t n = 1;
    for (int i = 0; i < a->rank; i++) n *= a->d[i];
    return n;
}

static Arr arr_new(int rank, const int *d) {
    Arr a;
    a.rank = rank;
    for (int i = 0; i < MAXR; i++) a.d[i] = i < rank ? d[i] : 1;
    int64_t n = arr_numel(&a);
    a.v = (double *)calloc((size_t)(n > 0 ? n : 1), sizeof(double));
    return a;
}

static Arr arr_copy(const Arr *s) {
    Arr a = arr_new(s->rank, s->d);
    memcpy(a.v, s->v, (size_t)arr_numel(s) * sizeof(double));
    return a;
}

static void arr_free(Arr *a) {
    free(a->v);
    a->v = NULL;
    a->rank = 0;
}

/* ------------------------------------------------------------------ errors */

static void set_err(char *err, int errlen, const char *fmt, ...) {
    if (!err || errlen <= 0) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err, (size_t)errlen, fmt, ap);
    va_end(ap);
}

/* ------------------------------------------- Python-literal values (variables.fpp) */

typedef enum { PV_NONE, PV_INT, PV_FLOAT, PV_STR, PV_LIST, PV_DICT } PVKind;

typedef struct PV {
    PVKind k;
    long long i;
    double f;
    char *s;
    int n;
    struct PV **items;
    struct PV **keys; /* for dicts */
} PV;

static void pv_free(PV *p) {
    if (!p) return;
    free(p->s);
    for (int j = 0; j < p->n; j++) {
        pv_free(p->items[j]);
        if (p->keys) pv_free(p->keys[j]);
    }
    free(p->items);
    free(p->keys);
    free(p);
}

typedef struct {
    const char *s;
    int pos;
    int bad;
} PVP;

static void pvp_ws(PVP *p) {
    while (p->s[p->pos] && isspace((unsigned char)p->s[p->pos])) p->pos++;
}

static PV *pv_alloc(PVKind k) {
    PV *v = (PV *)calloc(1, sizeof(PV));
    v->k = k;
    return v;
}

static void pv_push(PV *v, PV *item, PV *key) {
    v->items = (PV **)realloc(v->items, sizeof(PV *) * (size_t)(v->n + 1));
    if (key || v->keys) v->keys = (PV **)realloc(v->keys, sizeof(PV *) * (size_t)(v->n + 1));
    v->items[v->n] = item;
    if (v->keys) v->keys[v->n] = key;
    v->n++;
}

static PV *pv_parse(PVP *p);

static PV *pv_parse_seq(PVP *p, char close, int is_dict) {
    PV *v = pv_alloc(is_dict ? PV_DICT : PV_LIST);
    if (is_dict) v->keys = NULL;
    p->pos++; /* opening bracket */
    for (;;) {
        pvp_ws(p);
        if (p->s[p->pos] == close) {
            p->pos++;
            return v;
        }
        PV *key = NULL;
        if (is_dict) {
            key = pv_parse(p);
            if (p->bad) { pv_free(key); return v; }
            pvp_ws(p);
            if (p->s[p->pos] != ':') { p->bad = 1; pv_free(key); return v; }
            p->pos++;
        }
        PV *item = pv_parse(p);
        if (p->bad) { pv_free(item); pv_free(key); return v; }
        if (is_dict && !v->keys) v->keys = (PV **)calloc(1, sizeof(PV *));
        pv_push(v, item, key);
        pvp_ws(p);
        if (p->s[p->pos] == ',') { p->pos++; continue; }
        if (p->s[p->pos] == close) { p->pos++; return v; }
        p->bad = 1;
        return v;
    }
}

static PV *pv_parse(PVP *p) {
    pvp_ws(p);
    char c = p->s[p->pos];
    if (c == '[') return pv_parse_seq(p, ']', 0);
    if (c == '(') return pv_parse_seq(p, ')', 0);
    if (c == '{') return pv_parse_seq(p, '}', 1);
    if (c == '\'' || c == '"') {
        char q = c;
        int st = ++p->pos;
        while (p->s[p->pos] && p->s[p->pos] != q) p->pos++;
        if (!p->s[p->pos]) { p->bad = 1; return pv_alloc(PV_NONE); }
        PV *v = pv_alloc(PV_STR);
        int len = p->pos - st;
        v->s = (char *)malloc((size_t)len + 1);
        memcpy(v->s, p->s + st, (size_t)len);
        v->s[len] = 0;
        p->pos++;
        return v;
    }
    if (strncmp(p->s + p->pos, "None", 4) == 0) { p->pos += 4; return pv_alloc(PV_NONE); }
    if (strncmp(p->s + p->pos, "True", 4) == 0) { p->pos += 4; PV *v = pv_alloc(PV_INT); v->i = 1; return v; }
    if (strncmp(p->s + p->pos, "False", 5) == 0) { p->pos += 5; PV *v = pv_alloc(PV_INT); v->i = 0; return v; }
    /* numpy scalar reprs such as np.int64(3) */
    if (strncmp(p->s + p->pos, "np.", 3) == 0) {
        while (p->s[p->pos] && p->s[p->pos] != '(') p->pos++;
        if (!p->s[p->pos]) { p->bad = 1; return pv_alloc(PV_NONE); }
        p->pos++;
        PV *v = pv_parse(p);
        pvp_ws(p);
        if (p->s[p->pos] == ')') p->pos++; else p->bad = 1;
        return v;
    }
    if (c == '-' || c == '+' || isdigit((unsigned char)c) || c == '.') {
        char *end = NULL;
        const char *st = p->s + p->pos;
        int is_float = 0;
        for (const char *q = st + 1; *q && (isalnum((unsigned char)*q) || *q == '.' || *q == '-' || *q == '+'); q++)
            if (*q == '.' || *q == 'e' || *q == 'E') is_float = 1;
        PV *v;
        if (is_float) {
            v = pv_alloc(PV_FLOAT);
            v->f = strtod(st, &end);
        } else {
            v = pv_alloc(PV_INT);
            v->i = strtoll(st, &end, 10);
            v->f = (double)v->i;
        }
        if (end == st) p->bad = 1;
        p->pos += (int)(end - st);
        return v;
    }
    p->bad = 1;
    return pv_alloc(PV_NONE);
}

static long long pv_int(const PV *v) {
    if (!v) return 0;
    return v->k == PV_FLOAT ? (long long)v->f : v->i;
}

static const PV *pv_at(const PV *v, int j) {
    if (!v || (v->k != PV_LIST && v->k != PV_DICT) || j < 0 || j >= v->n) return NULL;
    return v->items[j];
}

/* ------------------------------------------------------------- the model */

typedef struct { Arr w, b; } LinLayer;                        /* derived_types.f90:14-17 */
typedef struct { Arr whh, wih, bhh, bih, hid, cell; } LstmLayer; /* derived_types.f90:19-26 */
typedef struct { Arr w, b; } ConvLayer;                        /* derived_types.f90:28-32 */
typedef struct { Arr adder; } AddLayer;                        /* derived_types.f90:42-44 */
typedef struct { Arr r; } ReshapeLayer;                        /* derived_types.f90:46-50 */

typedef struct ro_model {
    LinLayer *lin; int nlin;
    LstmLayer *lstm; int nlstm;
    ConvLayer *conv; int nconv;
    int *maxpool; int nmaxpool;
    int *avgpool; int navgpool;
    AddLayer *add; int nadd;
    ReshapeLayer *resh; int nresh;
    PV *architecture, *inputs, *trueInputs, *outShape, *outputs;
} ro_model;

/* Fortran list-directed READ of `count` numbers: starts at the next record and
 * continues over records until enough values are read; the rest of the last
 * record is skipped (reader.f90 reads every tensor with one READ statement). */
typedef struct {
    FILE *f;
    char *line;
    size_t cap;
    int eof;
} Rec;

static int rec_next(Rec *r) {
    ssize_t n = getline(&r->line, &r->cap, r->f);
    if (n < 0) { r->eof = 1; return 0; }
    return 1;
}

static int read_numbers(Rec *r, int64_t count, double *out) {
    int64_t got = 0;
    while (got < count) {
        if (!rec_next(r)) return -1;
        char *s = r->line;
        while (got < count) {
            while (*s && (isspace((unsigned char)*s) || *s == ',')) s++;
            if (!*s) break;
            char *end = NULL;
            double x = strtod(s, &end);
            if (end == s) return -2;
            out[got++] = x;
            s = end;
        }
    }
    return 0;
}

static int read_ints(Rec *r, int count, int *out) {
    double tmp[MAXR];
    if (count > MAXR) return -2;
    int rc = read_numbers(r, count, tmp);
    if (rc) return rc;
    for (int i = 0; i < count; i++) out[i] = (int)tmp[i];
    return 0;
}

/* read dims (count ints) from the model file and the tensor values from the weights file */
static int read_tensor(Rec *mf, Rec *wf, int rank, Arr *out) {
    int d[MAXR];
    if (read_ints(mf, rank, d)) return -1;
    *out = arr_new(rank, d);
    if (read_numbers(wf, arr_numel(out), out->v)) return -2;
    return 0;
}

#define APPEND(arr, n, item) do { (arr) = realloc((arr), sizeof(*(arr)) * (size_t)((n) + 1)); (arr)[(n)++] = (item); } while (0)

static void free_model(ro_model *m);

static PV *parse_variables(const char *path, ro_model *m, char *err, int errlen) {
    FILE *f = fopen(path, "r");
    if (!f) { set_err(err, errlen, "cannot open %s", path); return NULL; }
    char *line = NULL;
    size_t cap = 0;
    int ok = 1;
    while (getline(&line, &cap, f) >= 0) {
        char *s = line;
        while (*s && isspace((unsigned char)*s)) s++;
        if (strncmp(s, "#:set", 5) != 0) continue;
        s += 5;
        while (*s && isspace((unsigned char)*s)) s++;
        char name[64];
        int k = 0;
        while (*s && (isalnum((unsigned char)*s) || *s == '_') && k < 63) name[k++] = *s++;
        name[k] = 0;
        while (*s && isspace((unsigned char)*s)) s++;
        if (*s != '=') { ok = 0; break; }
        s++;
        PVP p = {s, 0, 0};
        PV *v = pv_parse(&p);
        if (p.bad) { pv_free(v); ok = 0; set_err(err, errlen, "cannot parse %s in %s", name, path); break; }
        PV **slot = NULL;
        if (!strcmp(name, "architecture")) slot = &m->architecture;
        else if (!strcmp(name, "inputs")) slot = &m->inputs;
        else if (!strcmp(name, "trueInputs")) slot = &m->trueInputs;
        else if (!strcmp(name, "outShape")) slot = &m->outShape;
        else if (!strcmp(name, "outputs")) slot = &m->outputs;
        if (slot) { pv_free(*slot); *slot = v; } else pv_free(v);
    }
    free(line);
    fclose(f);
    if (!ok) return NULL;
    if (!m->architecture || !m->trueInputs || !m->outShape || !m->outputs) {
        set_err(err, errlen, "%s lacks architecture/trueInputs/outShape/outputs", path);
        return NULL;
    }
    return m->architecture;
}

/* initialize(): fLibrary/reader.f90:38-99, with the read_* helpers at :101-290 */
ro_model *ro_load(const char *model_txt, const char *weights_txt, const char *variables_fpp, char *err, int errlen) {
    ro_model *m = (ro_model *)calloc(1, sizeof(ro_model));
    Rec mf = {0}, wf = {0};
    mf.f = fopen(model_txt, "r");
    wf.f = fopen(weights_txt, "r");
    if (!mf.f || !wf.f) {
        set_err(err, errlen, "cannot open %s or %s", model_txt, weights_txt);
        goto fail;
    }
    int numLayers = 0;
    if (read_ints(&mf, 1, &numLayers)) { set_err(err, errlen, "bad node count"); goto fail; }
    for (int i = 0; i < numLayers; i++) {
        if (!rec_next(&mf)) break; /* IOSTAT < 0: exit readloop (reader.f90:55-58) */
        char name[101] = {0};
        if (sscanf(mf.line, "%100s", name) != 1) break;
        int rc = 0;
        if (!strcmp(name, "LSTM")) { /* read_lstm, reader.f90:203-252 */
            int flag = 0;
            if (read_ints(&mf, 1, &flag)) { rc = -1; goto bad; }
            LstmLayer L;
            memset(&L, 0, sizeof(L));
            rc |= read_tensor(&mf, &wf, 3, &L.wih);
            rc |= read_tensor(&mf, &wf, 3, &L.whh);
            rc |= read_tensor(&mf, &wf, 1, &L.bih);
            rc |= read_tensor(&mf, &wf, 1, &L.bhh);
            if (flag == 1) {
                rc |= read_tensor(&mf, &wf, 3, &L.hid);
                rc |= read_tensor(&mf, &wf, 3, &L.cell);
            }
            APPEND(m->lstm, m->nlstm, L);
        } else if (!strcmp(name, "Gemm")) { /* read_linear, reader.f90:254-287 */
            LinLayer L;
            rc |= read_tensor(&mf, &wf, 2, &L.w);
            rc |= read_tensor(&mf, &wf, 1, &L.b);
            APPEND(m->lin, m->nlin, L);
        } else if (!strcmp(name, "Conv")) { /* read_conv, reader.f90:178-201 */
            ConvLayer C;
            rc |= read_tensor(&mf, &wf, 4, &C.w);
            rc |= read_tensor(&mf, &wf, 1, &C.b);
            APPEND(m->conv, m->nconv, C);
        } else if (!strcmp(name, "MaxPool")) { /* reader.f90:168-177 */
            int k = 0;
            rc |= read_ints(&mf, 1, &k);
            APPEND(m->maxpool, m->nmaxpool, k);
        } else if (!strcmp(name, "AveragePool")) { /* reader.f90:157-166 */
            int k = 0;
            rc |= read_ints(&mf, 1, &k);
            APPEND(m->avgpool, m->navgpool, k);
        } else if (!strcmp(name, "Add")) { /* reader.f90:143-155 */
            AddLayer A;
            rc |= read_tensor(&mf, &wf, 4, &A.adder);
            APPEND(m->add, m->nadd, A);
        } else if (!strcmp(name, "Reshape")) { /* reader.f90:74-82, 101-141 */
            int flag = 0;
            if (read_ints(&mf, 1, &flag)) { rc = -1; goto bad; }
            if (flag >= 2 && flag <= 4) {
                ReshapeLayer R;
                rc |= read_tensor(&mf, &wf, flag, &R.r);
                APPEND(m->resh, m->nresh, R);
            }
        }
        /* MatMul, Transpose, Squeeze, Pad, Relu and anything else: cycle */
    bad:
        if (rc) { set_err(err, errlen, "malformed weight files at node %d (%s)", i + 1, name); goto fail; }
    }
    fclose(mf.f);
    fclose(wf.f);
    free(mf.line);
    free(wf.line);
    mf.f = wf.f = NULL;
    if (!parse_variables(variables_fpp, m, err, errlen)) goto fail;
    return m;
fail:
    if (mf.f) fclose(mf.f);
    if (wf.f) fclose(wf.f);
    free(mf.line);
    free(wf.line);
    free_model(m);
    return NULL;
}

static void free_model(ro_model *m) {
    if (!m) return;
    for (int i = 0; i < m->nlin; i++) { arr_free(&m->lin[i].w); arr_free(&m->lin[i].b); }
    for (int i = 0; i < m->nlstm; i++) {
        arr_free(&m->lstm[i].wih); arr_free(&m->lstm[i].whh); arr_free(&m->lstm[i].bih);
        arr_free(&m->lstm[i].bhh); arr_free(&m->lstm[i].hid); arr_free(&m->lstm[i].cell);
    }
    for (int i = 0; i < m->nconv; i++) { arr_free(&m->conv[i].w); arr_free(&m->conv[i].b); }
    for (int i = 0; i < m->nadd; i++) arr_free(&m->add[i].adder);
    for (int i = 0; i < m->nresh; i++) arr_free(&m->resh[i].r);
    free(m->lin); free(m->lstm); free(m->conv); free(m->maxpool); free(m->avgpool); free(m->add); free(m->resh);
    pv_free(m->architecture); pv_free(m->inputs); pv_free(m->trueInputs); pv_free(m->outShape); pv_free(m->outputs);
    free(m);
}

void ro_free(ro_model *m) { free_model(m); }

/* ------------------------------------------------------------ activations
 * fLibrary/activation_funcs.f90:7-64 */

static double sigmoid_d(double x) { return 1.0 / (1.0 + exp(-1.0 * x)); }
static double relu_d(double x) { return x < 0 ? 0.0 : x; }
static double tanhh_d(double x) { return (exp(x) - exp(-1.0 * x)) / (exp(x) + exp(-1.0 * x)); }

/* ------------------------------------------------------------- RESHAPE
 * Fortran RESHAPE(SOURCE, SHAPE, ORDER): the elements of SOURCE, in array
 * element order, fill the result with subscript ORDER(1) varying fastest. */
static Arr fortran_reshape_order(const Arr *src, int rank, const int *shape, const int *order1) {
    Arr r = arr_new(rank, shape);
    int64_t n = arr_numel(src), rn = arr_numel(&r);
    if (rn < n) n = rn;
    int64_t stride[MAXR];
    stride[0] = 1;
    for (int i = 1; i < rank; i++) stride[i] = stride[i - 1] * shape[i - 1];
    int sub[MAXR] = {0};
    for (int64_t L = 0; L < n; L++) {
        int64_t off = 0;
        for (int k = 0; k < rank; k++) off += (int64_t)sub[order1[k] - 1] * stride[order1[k] - 1];
        r.v[off] = src->v[L];
        /* advance the permuted subscript counter */
        for (int k = 0; k < rank; k++) {
            int dim = order1[k] - 1;
            if (++sub[dim] < shape[dim]) break;
            sub[dim] = 0;
        }
    }
    return r;
}

/* ---------------------------------------------------------------- layers */

/* linear_layer, fLibrary/layers.f90:11-23 */
static int linear_layer(Arr *inp, const LinLayer *lin, int transInp) {
    const Arr *W = &lin->w;
    int M = W->d[0], K = W->d[1];
    if (inp->rank != 2) return -1;
    if (transInp == 0) { /* inp(N,K) . W(M,K)^T + b; each sum runs over k in order */
        int N = inp->d[0];
        if (inp->d[1] != K) return -2;
        int d[2] = {N, M};
        Arr o = arr_new(2, d);
        double *acc = (double *)malloc(sizeof(double) * (size_t)M);
        for (int i = 0; i < N; i++) {
            for (int m = 0; m < M; m++) acc[m] = 0;
            for (int k = 0; k < K; k++) {
                const double x = inp->v[i + (int64_t)N * k];
                const double *w = W->v + (int64_t)M * k;
                for (int m = 0; m < M; m++) acc[m] += x * w[m];
            }
            for (int m = 0; m < M; m++) o.v[i + (int64_t)N * m] = acc[m] + lin->b.v[m];
        }
        free(acc);
        arr_free(inp);
        *inp = o;
    } else { /* W(M,K) . inp(K,N) + b */
        int N = inp->d[1];
        if (inp->d[0] != K) return -2;
        int d[2] = {M, N};
        Arr o = arr_new(2, d);
        for (int j = 0; j < N; j++)
            for (int m = 0; m < M; m++) {
                double s = 0;
                for (int k = 0; k < K; k++) s += W->v[m + (int64_t)M * k] * inp->v[k + (int64_t)K * j];
                o.v[m + (int64_t)M * j] = s + lin->b.v[m];
            }
        arr_free(inp);
        *inp = o;
    }
    return 0;
}

/* lstm_cell, fLibrary/layers.f90:62-99.  x (I,N), h and c (H,N), Wih (4H,I), Whh (4H,H) */
static void lstm_cell(const double *x, int I, int N, double *h, double *c, int H,
                      const double *Wih, const double *Whh, const double *bih, const double *bhh, double *gates) {
    int G = 4 * H;
    double *a = gates + (int64_t)G * N; /* scratch: 2*G doubles after the gates */
    double *b = a + G;
    for (int j = 0; j < N; j++) {
        for (int r = 0; r < G; r++) a[r] = b[r] = 0;
        for (int k = 0; k < I; k++) {
            const double xv = x[k + (int64_t)I * j];
            const double *w = Wih + (int64_t)G * k;
            for (int r = 0; r < G; r++) a[r] += w[r] * xv;
        }
        for (int k = 0; k < H; k++) {
            const double hv = h[k + (int64_t)H * j];
            const double *w = Whh + (int64_t)G * k;
            for (int r = 0; r < G; r++) b[r] += w[r] * hv;
        }
        for (int r = 0; r < G; r++) gates[r + (int64_t)G * j] = ((a[r] + bih[r]) + b[r]) + bhh[r];
    }
    /* chunks = RESHAPE(gates, (H,4,N)): chunk q holds gate rows q*H..q*H+H-1 (i, f, g, o) */
    for (int j = 0; j < N; j++)
        for (int u = 0; u < H; u++) {
            const double *g = gates + (int64_t)G * j;
            double ig = sigmoid_d(g[u]);
            double fg = sigmoid_d(g[H + u]);
            double gg = tanhh_d(g[2 * H + u]);
            double og = sigmoid_d(g[3 * H + u]);
            double cn = (fg * c[u + (int64_t)H * j]) + (ig * gg);
            c[u + (int64_t)H * j] = cn;
            h[u + (int64_t)H * j] = og * tanhh_d(cn);
        }
}

/* lstm, fLibrary/layers.f90:101-132.  input (T,N,I), hid/cell (1,N,H) updated in place,
 * output (T,1,N,H). */
static int lstm_layer(const Arr *input, Arr *hid, Arr *cell, const LstmLayer *L, Arr *output) {
    if (input->rank != 3 || hid->rank != 3 || cell->rank != 3) return -1;
    int T = input->d[0], N = input->d[1], I = input->d[2];
    int H = hid->d[2];
    if (L->wih.d[1] != 4 * H || L->wih.d[2] != I || L->whh.d[2] != H || hid->d[1] != N) return -2;
    /* input reshaped to (T,I,N), hid/cell to (1,H,N) (order [1,3,2]) */
    double *x = (double *)malloc(sizeof(double) * (size_t)I * (size_t)N);
    double *h = (double *)malloc(sizeof(double) * (size_t)H * (size_t)N);
    double *c = (double *)malloc(sizeof(double) * (size_t)H * (size_t)N);
    double *gates = (double *)malloc(sizeof(double) * (size_t)(4 * H) * (size_t)(N + 2));
    for (int j = 0; j < N; j++)
        for (int u = 0; u < H; u++) {
            h[u + (int64_t)H * j] = hid->v[0 + (int64_t)j + (int64_t)N * u];
            c[u + (int64_t)H * j] = cell->v[0 + (int64_t)j + (int64_t)N * u];
        }
    int od[4] = {T, 1, N, H};
    *output = arr_new(4, od);
    for (int t = 0; t < T; t++) {
        for (int j = 0; j < N; j++)
            for (int k = 0; k < I; k++) x[k + (int64_t)I * j] = input->v[t + (int64_t)T * j + (int64_t)T * N * k];
        lstm_cell(x, I, N, h, c, H, L->wih.v, L->whh.v, L->bih.v, L->bhh.v, gates);
        for (int j = 0; j < N; j++)
            for (int u = 0; u < H; u++)
                output->v[t + (int64_t)T * 0 + (int64_t)T * 1 * j + (int64_t)T * N * u] = h[u + (int64_t)H * j];
    }
    for (int j = 0; j < N; j++)
        for (int u = 0; u < H; u++) {
            hid->v[j + (int64_t)N * u] = h[u + (int64_t)H * j];
            cell->v[j + (int64_t)N * u] = c[u + (int64_t)H * j];
        }
    free(x); free(h); free(c); free(gates);
    return 0;
}

/* padding, fLibrary/layers.f90:134-181: zero rows/cols, arr(1) rows and arr(2) cols on each side */
static Arr pad4(const Arr *in, int p1, int p2) {
    int B = in->d[0], C = in->d[1], H = in->d[2], W = in->d[3];
    int d[4] = {B, C, H + 2 * p1, W + 2 * p2};
    Arr o = arr_new(4, d);
    for (int w = 0; w < W; w++)
        for (int h = 0; h < H; h++)
            for (int c = 0; c < C; c++)
                for (int b = 0; b < B; b++)
                    o.v[b + (int64_t)B * (c + (int64_t)C * ((h + p1) + (int64_t)d[2] * (w + p2)))] =
                        in->v[b + (int64_t)B * (c + (int64_t)C * (h + (int64_t)H * w))];
    return o;
}

#define A4(a, i0, i1, i2, i3) ((a)->v[(i0) + (int64_t)(a)->d[0] * ((i1) + (int64_t)(a)->d[1] * ((i2) + (int64_t)(a)->d[2] * (i3)))])

/* conv, fLibrary/layers.f90:183-233 (dilations ignored, square kernel of size(W,3)) */
static int conv_layer(Arr *inp, const ConvLayer *cv, const int *pads, const int *strides) {
    if (inp->rank != 4) return -1;
    Arr padded = pad4(inp, pads[0], pads[1]);
    int B = inp->d[0], C = inp->d[1];
    int OC = cv->w.d[0], ks = cv->w.d[2];
    if (cv->w.d[1] != C) { arr_free(&padded); return -2; }
    int Ho = (padded.d[2] - ks) / strides[0] + 1, Wo = (padded.d[3] - ks) / strides[1] + 1;
    int od[4] = {B, OC, Ho, Wo};
    Arr out = arr_new(4, od);
    int outRowDim = Wo;
    for (int b = 0; b < B; b++)
        for (int oc = 0; oc < OC; oc++)
            for (int ov = 0; ov < Ho * Wo; ov++) {
                int r = ov / outRowDim, q = ov % outRowDim;
                double sumini = 0;
                for (int ic = 0; ic < C; ic++) {
                    double s = 0;
                    for (int kw = 0; kw < ks; kw++)
                        for (int kh = 0; kh < ks; kh++)
                            s += A4(&padded, b, ic, r * strides[0] + kh, q * strides[1] + kw) * A4(&cv->w, oc, ic, kh, kw);
                    sumini += s;
                }
                A4(&out, b, oc, r, q) = sumini + cv->b.v[oc];
            }
    arr_free(&padded);
    arr_free(inp);
    *inp = out;
    return 0;
}

/* max_pool and avgpool, fLibrary/layers.f90:236-310.  Batch index 1 only; the
 * output column subscript is MODULO(overImage, outColDim) as in the reference. */
static int pool_layer(Arr *inp, int ks, const int *pads, const int *strides, int is_avg) {
    if (inp->rank != 4) return -1;
    Arr padded = pad4(inp, pads[0], pads[1]);
    int C = padded.d[1];
    int Ho = (padded.d[2] - ks) / strides[0] + 1, Wo = (padded.d[3] - ks) / strides[1] + 1;
    int od[4] = {1, C, Ho, Wo};
    Arr out = arr_new(4, od);
    int outRowDim = Wo, outColDim = Ho;
    double total = (double)(ks * ks);
    for (int ov = 0; ov < Ho * Wo; ov++)
        for (int c = 0; c < C; c++) {
            int r = ov / outRowDim, q = ov % outRowDim;
            double acc = is_avg ? 0.0 : -INFINITY;
            for (int kw = 0; kw < ks; kw++)
                for (int kh = 0; kh < ks; kh++) {
                    double v = A4(&padded, 0, c, r * strides[0] + kh, q * strides[1] + kw);
                    if (is_avg) acc += v; else if (v > acc) acc = v;
                }
            A4(&out, 0, c, r, ov % outColDim) = is_avg ? acc / total : acc;
        }
    arr_free(&padded);
    arr_free(inp);
    *inp = out;
    return 0;
}

/* broadc, fLibrary/layers.f90:351-375: SPREAD the 4-D adder along each
 * (dim, copies) pair of spreadInfo in turn, each time RESHAPEd (column-major,
 * the first elements taken, as Fortran's RESHAPE does) to trueShape(:dim)
 * followed by the adder's ORIGINAL trailing dims (`inter` is never updated);
 * the last pair RESHAPEs to trueShape. */
static int broadc(const Arr *inp, const int *trueShape, const int *spread, int npairs, Arr *out) {
    Arr cur = arr_copy(inp);
    for (int i = 0; i < npairs; i++) {
        const int d = spread[2 * i], n = spread[2 * i + 1];
        if (d < 1 || d > 4 || n < 1) { arr_free(&cur); return -1; }
        int64_t P = 1, rest = 1;
        for (int k = 0; k < d - 1; k++) P *= cur.d[k];
        for (int k = d - 1; k < 4; k++) rest *= cur.d[k];
        /* SPREAD(cur, d, n): sp(a, k, b) = cur(a, b), a over dims < d, b over dims >= d */
        double *sp = (double *)malloc(sizeof(double) * (size_t)(P * n * rest > 0 ? P * n * rest : 1));
        for (int64_t b = 0; b < rest; b++)
            for (int k = 0; k < n; k++)
                for (int64_t a = 0; a < P; a++) sp[a + P * (k + (int64_t)n * b)] = cur.v[a + P * b];
        int shape[4];
        if (i != npairs - 1) {
            for (int k = 0; k < 4; k++) shape[k] = k < d ? trueShape[k] : inp->d[k];
        } else {
            for (int k = 0; k < 4; k++) shape[k] = trueShape[k];
        }
        Arr nx = arr_new(4, shape);
        int64_t need = arr_numel(&nx);
        if (need > P * n * rest) { free(sp); arr_free(&nx); arr_free(&cur); return -1; }
        memcpy(nx.v, sp, sizeof(double) * (size_t)need);
        free(sp);
        arr_free(&cur);
        cur = nx;
    }
    *out = cur;
    return 0;
}

/* matmul2D / matmul3D / matmul4D, fLibrary/layers.f90:25-60: inp1 = inp1 . inp2
 * over the last two dims, per index of the leading dims of inp1 (inp2 indexed
 * by the same leading indices). */
static int matmul_nd(Arr *inp1, const Arr *inp2, int rank) {
    if (rank < 2 || rank > 4 || inp1->rank != rank || inp2->rank != rank) return -1;
    const int P = inp1->d[rank - 2], K = inp1->d[rank - 1], M = inp2->d[rank - 1];
    if (inp2->d[rank - 2] != K) return -2;
    int lead1[2] = {1, 1}, lead2[2] = {1, 1};
    for (int k = 0; k < rank - 2; k++) {
        lead1[k] = inp1->d[k];
        lead2[k] = inp2->d[k];
        if (lead2[k] < lead1[k]) return -2;
    }
    int d[MAXR];
    for (int k = 0; k < rank; k++) d[k] = inp1->d[k];
    d[rank - 1] = M;
    Arr o = arr_new(rank, d);
    /* element (i, j, p, q) of a rank-4 array with dims (D1, D2, D3, D4) sits at
     * i + D1*(j + D2*(p + D3*q)); leading dims first */
    const int64_t L1 = (int64_t)lead1[0] * lead1[1], L2 = (int64_t)lead2[0] * lead2[1];
    for (int j = 0; j < lead1[1]; j++)
        for (int i = 0; i < lead1[0]; i++) {
            const int64_t o1 = i + (int64_t)lead1[0] * j, o2 = i + (int64_t)lead2[0] * j;
            for (int p = 0; p < P; p++)
                for (int q = 0; q < M; q++) {
                    double acc = 0;
                    for (int k = 0; k < K; k++)
                        acc += inp1->v[o1 + L1 * (p + (int64_t)P * k)] * inp2->v[o2 + L2 * (k + (int64_t)K * q)];
                    o.v[o1 + L1 * (p + (int64_t)P * q)] = acc;
                }
        }
    arr_free(inp1);
    *inp1 = o;
    return 0;
}

/* --------------------------------------------------------- interpreter */

typedef struct {
    char name[96];
    Arr a;
} Var;

typedef struct {
    Var *v;
    int n;
} Vars;

static Arr *var_get(Vars *vs, const char *name) {
    for (int i = 0; i < vs->n; i++)
        if (!strcmp(vs->v[i].name, name)) return &vs->v[i].a;
    return NULL;
}

static Arr *var_set(Vars *vs, const char *name, Arr a) {
    Arr *cur = var_get(vs, name);
    if (cur) {
        arr_free(cur);
        *cur = a;
        return cur;
    }
    vs->v = (Var *)realloc(vs->v, sizeof(Var) * (size_t)(vs->n + 1));
    snprintf(vs->v[vs->n].name, sizeof(vs->v[vs->n].name), "%s", name);
    vs->v[vs->n].a = a;
    return &vs->v[vs->n++].a;
}

static void vars_free(Vars *vs) {
    for (int i = 0; i < vs->n; i++) arr_free(&vs->v[i].a);
    free(vs->v);
    vs->v = NULL;
    vs->n = 0;
}

static const char *pv_str(const PV *v) { return (v && v->k == PV_STR) ? v->s : NULL; }

static int pv_ints(const PV *v, int *out, int max) {
    if (!v || v->k != PV_LIST) return -1;
    int n = v->n < max ? v->n : max;
    for (int i = 0; i < n; i++) out[i] = (int)pv_int(v->items[i]);
    return n;
}

int ro_num_inputs(const ro_model *m) { return m->trueInputs->n; }
int ro_num_outputs(const ro_model *m) { return m->outShape->n; }

/* shape of input / output i (export shape); returns rank */
int ro_input_shape(const ro_model *m, int i, int *dims) {
    const PV *shape = pv_at(pv_at(m->trueInputs, i), 1);
    return pv_ints(shape, dims, MAXR);
}

int ro_output_shape(const ro_model *m, int i, int *dims) {
    const PV *shape = pv_at(pv_at(m->outShape, i), 1);
    return pv_ints(shape, dims, MAXR);
}

static int64_t shape_numel(const int *d, int r) {
    int64_t n = 1;
    for (int i = 0; i < r; i++) n *= d[i];
    return n;
}

/* counters of layer_dict (modelCreator.fpp:79-85,164-166) */
typedef struct { int gemm, lstm, conv, maxpool, avgpool, add, reshape; } Counters;

static int run_op(const ro_model *m, Vars *vs, const PV *tup, Counters *cnt, char *err, int errlen) {
    const char *op = pv_str(pv_at(tup, 0));
    const PV *a1 = pv_at(tup, 1), *a2 = pv_at(tup, 2), *a3 = pv_at(tup, 3), *alast = pv_at(tup, tup->n - 1);
    if (!op) { set_err(err, errlen, "architecture entry without op name"); return -1; }
    if (!strcmp(op, "Gemm")) { /* modelCreator.fpp:87-89 */
        Arr *x = var_get(vs, pv_str(pv_at(a1, 0)));
        int transB = (int)pv_int(pv_at(a1, 1));
        if (!x || cnt->gemm >= m->nlin) { set_err(err, errlen, "Gemm: missing input or weights"); return -1; }
        if (linear_layer(x, &m->lin[cnt->gemm], 1 - transB)) { set_err(err, errlen, "Gemm: shape mismatch"); return -1; }
        cnt->gemm++;
    } else if (!strcmp(op, "LSTM")) { /* modelCreator.fpp:92-100 */
        if (cnt->lstm >= m->nlstm) { set_err(err, errlen, "LSTM: no weights"); return -1; }
        const LstmLayer *L = &m->lstm[cnt->lstm];
        const char *xn = pv_str(pv_at(a1, 0)), *hn = pv_str(pv_at(a1, 1)), *cn = pv_str(pv_at(a1, 2));
        const char *yn = pv_str(pv_at(a2, 0));
        int flag = (int)pv_int(pv_at(alast, 0));
        if (flag == 1) {
            var_set(vs, hn, arr_copy(&L->hid));
            var_set(vs, cn, arr_copy(&L->cell));
        }
        Arr *x = var_get(vs, xn), *h = var_get(vs, hn), *c = var_get(vs, cn);
        if (!x || !h || !c) { set_err(err, errlen, "LSTM: missing input"); return -1; }
        Arr y;
        if (lstm_layer(x, h, c, L, &y)) { set_err(err, errlen, "LSTM: shape mismatch"); return -1; }
        var_set(vs, yn, y);
        cnt->lstm++;
    } else if (!strcmp(op, "Conv")) { /* modelCreator.fpp:103-105 */
        Arr *x = var_get(vs, pv_str(pv_at(a1, 0)));
        int pads[4] = {0, 0, 0, 0}, strides[2] = {1, 1};
        pv_ints(pv_at(a2, 2), pads, 4);
        pv_ints(pv_at(a2, 3), strides, 2);
        if (!x || cnt->conv >= m->nconv || conv_layer(x, &m->conv[cnt->conv], pads, strides)) {
            set_err(err, errlen, "Conv failed");
            return -1;
        }
        cnt->conv++;
    } else if (!strcmp(op, "MaxPool") || !strcmp(op, "AveragePool")) { /* modelCreator.fpp:107-114 */
        int is_avg = op[0] == 'A';
        Arr *x = var_get(vs, pv_str(pv_at(a1, 0)));
        int pads[4] = {0, 0, 0, 0}, strides[2] = {1, 1};
        pv_ints(pv_at(a2, 1), pads, 4);
        pv_ints(pv_at(a2, 2), strides, 2);
        int *ctr = is_avg ? &cnt->avgpool : &cnt->maxpool;
        int nk = is_avg ? m->navgpool : m->nmaxpool;
        if (!x || *ctr >= nk) { set_err(err, errlen, "%s: missing input or layer", op); return -1; }
        int ks = is_avg ? m->avgpool[*ctr] : m->maxpool[*ctr];
        if (pool_layer(x, ks, pads, strides, is_avg)) { set_err(err, errlen, "%s failed", op); return -1; }
        (*ctr)++;
    } else if (!strcmp(op, "Transpose")) { /* modelCreator.fpp:117-119 */
        Arr *x = var_get(vs, pv_str(pv_at(a1, 0)));
        int order[MAXR];
        int r = pv_ints(pv_at(a2, 0), order, MAXR);
        if (!x || r != x->rank) { set_err(err, errlen, "Transpose: bad input"); return -1; }
        int shape[MAXR];
        for (int i = 0; i < r; i++) shape[i] = x->d[order[i] - 1];
        Arr t = fortran_reshape_order(x, r, shape, order);
        arr_free(x);
        *x = t;
    } else if (!strcmp(op, "Reshape")) { /* modelCreator.fpp:122-130 */
        const char *xn = pv_str(pv_at(a1, 0));
        int rank = (int)pv_int(pv_at(a1, 1));
        const char *on = pv_str(pv_at(a2, 0));
        int ns[MAXR];
        int nr = pv_ints(pv_at(a3, 0), ns, MAXR);
        int flag = (int)pv_int(pv_at(alast, 0));
        Arr *x;
        Arr konst = {0};
        if (flag == 0) {
            x = var_get(vs, xn);
        } else {
            /* The reference reverses the stored constant in place, so its result
             * alternates between calls; the oracle keeps the first-call result. */
            if (cnt->reshape >= m->nresh) { set_err(err, errlen, "Reshape: no constant"); return -1; }
            konst = arr_copy(&m->resh[cnt->reshape].r);
            x = &konst;
        }
        if (!x || nr <= 0 || x->rank != rank) { arr_free(&konst); set_err(err, errlen, "Reshape: bad input"); return -1; }
        /* x = RESHAPE(x, reversed dims, order = reversed): axis reversal, in place */
        int rs[MAXR], ro[MAXR];
        for (int i = 0; i < rank; i++) { rs[i] = x->d[rank - 1 - i]; ro[i] = rank - i; }
        Arr xr = fortran_reshape_order(x, rank, rs, ro);
        arr_free(x);
        *x = xr;
        int no[MAXR];
        for (int i = 0; i < nr; i++) no[i] = nr - i;
        Arr o = fortran_reshape_order(x, nr, ns, no);
        int64_t xn_el = arr_numel(x);
        arr_free(&konst);
        if (shape_numel(ns, nr) != xn_el) { arr_free(&o); set_err(err, errlen, "Reshape: size mismatch"); return -1; }
        var_set(vs, on, o);
        if (flag != 0) cnt->reshape++;
    } else if (!strcmp(op, "Squeeze")) { /* modelCreator.fpp:133-135 */
        const char *xn = pv_str(pv_at(a1, 0));
        int rank = (int)pv_int(pv_at(a1, 1));
        const char *on = pv_str(pv_at(a2, 0));
        int axes[MAXR];
        int na = pv_ints(pv_at(a3, 0), axes, MAXR);
        Arr *x = var_get(vs, xn);
        if (!x || x->rank != rank) { set_err(err, errlen, "Squeeze: bad input"); return -1; }
        int ns[MAXR], nr = 0;
        for (int i = 0; i < rank; i++) {
            int sq = 0;
            for (int j = 0; j < na; j++) if (axes[j] == i) sq = 1;
            if (!sq) ns[nr++] = x->d[i];
        }
        Arr o = arr_new(nr, ns);
        memcpy(o.v, x->v, sizeof(double) * (size_t)arr_numel(x));
        var_set(vs, on, o);
    } else if (!strcmp(op, "Add")) { /* modelCreator.fpp:137-144 */
        Arr *x = var_get(vs, pv_str(pv_at(a1, 0)));
        int ts[4], sp[2 * MAXR * 2];
        const int nt = pv_ints(pv_at(a2, 0), ts, 4);
        const int ns = pv_ints(pv_at(a2, 1), sp, 2 * MAXR * 2);
        const int rank = (int)pv_int(pv_at(a2, 2));
        if (!x || cnt->add >= m->nadd || nt != 4 || ns < 0 || (ns & 1) || rank < 1 || rank > 4 || x->rank != rank) {
            set_err(err, errlen, "Add: bad input or layer");
            return -1;
        }
        const Arr *A = &m->add[cnt->add].adder;
        Arr b;
        if (ns == 0) b = arr_copy(A);
        else if (broadc(A, ts, sp, ns / 2, &b)) { set_err(err, errlen, "Add: broadcast shapes do not fit"); return -1; }
        /* x = x + RESHAPE(b, trueShape(5-rank:)): the first numel(x) elements, column-major */
        const int64_t n = arr_numel(x);
        int64_t tn = 1;
        for (int k = 4 - rank; k < 4; k++) tn *= ts[k];
        if (tn != n || arr_numel(&b) < n) { arr_free(&b); set_err(err, errlen, "Add: shape mismatch"); return -1; }
        for (int64_t i = 0; i < n; i++) x->v[i] += b.v[i];
        arr_free(&b);
        cnt->add++;
    } else if (!strcmp(op, "MatMul")) { /* modelCreator.fpp:146-149 */
        Arr *x = var_get(vs, pv_str(pv_at(a1, 0)));
        const Arr *y = var_get(vs, pv_str(pv_at(a1, 1)));
        const int rank = (int)pv_int(pv_at(a2, 0));
        if (!x || !y || matmul_nd(x, y, rank)) { set_err(err, errlen, "MatMul: bad operands"); return -1; }
    } else if (!strcmp(op, "Slice") || !strcmp(op, "Gather")) {
        /* ONNX Slice (axes, starts, ends; step 1) and Gather (axis, one index,
         * the axis dropped).  modelParserONNX.py:519-523 writes nothing for
         * these ops; this build's front end writes them as architecture entries
         * (a stacked LSTM's per-layer initial states and the last layer's h_n). */
        const int is_gather = op[0] == 'G';
        Arr *x = var_get(vs, pv_str(pv_at(a1, 0)));
        const char *on = pv_str(pv_at(a2, 0));
        if (!x || !on) { set_err(err, errlen, "%s: missing input", op); return -1; }
        int lo[MAXR], hi[MAXR];
        for (int i = 0; i < x->rank; i++) { lo[i] = 0; hi[i] = x->d[i]; }
        int drop = -1;
        if (is_gather) {
            int ax = (int)pv_int(pv_at(a3, 0)), idx = (int)pv_int(pv_at(a3, 1));
            if (ax < 0) ax += x->rank;
            if (ax < 0 || ax >= x->rank) { set_err(err, errlen, "Gather: bad axis"); return -1; }
            if (idx < 0) idx += x->d[ax];
            if (idx < 0 || idx >= x->d[ax]) { set_err(err, errlen, "Gather: index out of range"); return -1; }
            lo[ax] = idx;
            hi[ax] = idx + 1;
            drop = ax;
        } else {
            int axes[MAXR], st[MAXR], en[MAXR];
            const int na = pv_ints(pv_at(a3, 0), axes, MAXR), ns = pv_ints(pv_at(a3, 1), st, MAXR),
                      ne = pv_ints(pv_at(a3, 2), en, MAXR);
            if (na < 0 || na != ns || na != ne) { set_err(err, errlen, "Slice: bad parameters"); return -1; }
            for (int j = 0; j < na; j++) {
                int ax = axes[j] < 0 ? axes[j] + x->rank : axes[j];
                if (ax < 0 || ax >= x->rank) { set_err(err, errlen, "Slice: bad axis"); return -1; }
                int a = st[j] < 0 ? st[j] + x->d[ax] : st[j], b = en[j] < 0 ? en[j] + x->d[ax] : en[j];
                a = a < 0 ? 0 : (a > x->d[ax] ? x->d[ax] : a);
                b = b < a ? a : (b > x->d[ax] ? x->d[ax] : b);
                lo[ax] = a;
                hi[ax] = b;
            }
        }
        int od[MAXR], orank = 0;
        for (int i = 0; i < x->rank; i++)
            if (i != drop) od[orank++] = hi[i] - lo[i];
        int full[MAXR];
        for (int i = 0; i < x->rank; i++) full[i] = hi[i] - lo[i];
        Arr o = arr_new(orank, od);
        const int64_t n = arr_numel(&o);
        for (int64_t L = 0; L < n; L++) {  /* column-major walk of the kept box */
            int64_t rem = L, src = 0, stride = 1;
            for (int i = 0; i < x->rank; i++) {
                const int64_t k = rem % full[i];
                rem /= full[i];
                src += (k + lo[i]) * stride;
                stride *= x->d[i];
            }
            o.v[L] = x->v[src];
        }
        var_set(vs, on, o);
    } else if (!strcmp(op, "Concat")) {
        /* ONNX Concat along `axis` (no reference counterpart: see Slice) */
        const char *on = pv_str(pv_at(a2, 0));
        int ax = (int)pv_int(pv_at(a3, 0));
        const int k = a1 ? a1->n : 0;
        Arr *parts[16];
        if (k < 1 || k > 16 || !on) { set_err(err, errlen, "Concat: bad operands"); return -1; }
        for (int j = 0; j < k; j++) {
            parts[j] = var_get(vs, pv_str(pv_at(a1, j)));
            if (!parts[j]) { set_err(err, errlen, "Concat: missing input"); return -1; }
        }
        const int r = parts[0]->rank;
        if (ax < 0) ax += r;
        if (ax < 0 || ax >= r) { set_err(err, errlen, "Concat: bad axis"); return -1; }
        int od[MAXR];
        for (int i = 0; i < r; i++) od[i] = parts[0]->d[i];
        od[ax] = 0;
        for (int j = 0; j < k; j++) {
            for (int i = 0; i < r; i++)
                if (i != ax && (parts[j]->rank != r || parts[j]->d[i] != od[i])) {
                    set_err(err, errlen, "Concat: shapes differ");
                    return -1;
                }
            od[ax] += parts[j]->d[ax];
        }
        Arr o = arr_new(r, od);
        int64_t inner = 1, outer = 1;
        for (int i = 0; i < ax; i++) inner *= od[i];
        for (int i = ax + 1; i < r; i++) outer *= od[i];
        for (int64_t q = 0; q < outer; q++) {
            int64_t base = 0;
            for (int j = 0; j < k; j++) {
                const int64_t blk = inner * parts[j]->d[ax];
                memcpy(o.v + q * inner * od[ax] + base, parts[j]->v + q * blk, sizeof(double) * (size_t)blk);
                base += blk;
            }
        }
        var_set(vs, on, o);
    } else if (!strcmp(op, "Relu") || !strcmp(op, "Tanh") || !strcmp(op, "Sigmoid")) { /* modelCreator.fpp:151-161 */
        Arr *x = var_get(vs, pv_str(pv_at(a1, 0)));
        if (!x) { set_err(err, errlen, "%s: missing input", op); return -1; }
        int64_t n = arr_numel(x);
        for (int64_t i = 0; i < n; i++)
            x->v[i] = op[0] == 'R' ? relu_d(x->v[i]) : op[0] == 'T' ? tanhh_d(x->v[i]) : sigmoid_d(x->v[i]);
    } else {
        set_err(err, errlen, "op %s is not supported by the oracle", op);
        return -1;
    }
    return 0;
}

/* One call of the generated use_model (modelCreator.fpp:42-171) at the export shapes. */
int ro_run(const ro_model *m, const double *const *inputs, double *const *outputs, char *err, int errlen) {
    Vars vs = {0};
    int rc = 0;
    for (int i = 0; i < m->trueInputs->n; i++) {
        const PV *ti = pv_at(m->trueInputs, i);
        int d[MAXR];
        int r = pv_ints(pv_at(ti, 1), d, MAXR);
        Arr a = arr_new(r, d);
        memcpy(a.v, inputs[i], sizeof(double) * (size_t)arr_numel(&a));
        var_set(&vs, pv_str(pv_at(ti, 0)), a);
    }
    Counters cnt = {0};
    for (int j = 0; j < m->architecture->n && rc == 0; j++) rc = run_op(m, &vs, m->architecture->items[j], &cnt, err, errlen);
    if (rc == 0) {
        /* o<index> = outputs[key<index>] in dict order, shape from outShape[index] */
        for (int i = 0; i < m->outShape->n; i++) {
            const PV *key = m->outputs->keys ? m->outputs->items[i] : NULL;
            const char *vn = pv_str(key);
            Arr *a = vn ? var_get(&vs, vn) : NULL;
            int d[MAXR];
            int r = ro_output_shape(m, i, d);
            int64_t n = shape_numel(d, r);
            if (!a || arr_numel(a) != n) { set_err(err, errlen, "output %d (%s) missing or wrong size", i, vn ? vn : "?"); rc = -1; break; }
            memcpy(outputs[i], a->v, sizeof(double) * (size_t)n);
        }
    }
    vars_free(&vs);
    return rc;
}

/* Batched evaluation: the model is exported at batch 1 and use_model is called
 * once per sample (the CPU baseline).  Arrays use the batched reference layout:
 * the Fortran column-major array of the export shape with its batch dimension
 * widened to n.  pre[i] is the product of the export dims in front of the batch
 * dimension of tensor i (1 when the batch dim leads). */
int ro_run_batched(const ro_model *m, int64_t n, const double *const *inputs, double *const *outputs,
                   const int *in_pre, const int *out_pre, int nthreads, char *err, int errlen) {
    int ni = m->trueInputs->n, no = m->outShape->n;
    int64_t in_numel[16], out_numel[16];
    if (ni > 16 || no > 16) { set_err(err, errlen, "too many model arguments"); return -1; }
    for (int i = 0; i < ni; i++) { int d[MAXR]; int r = ro_input_shape(m, i, d); in_numel[i] = shape_numel(d, r); }
    for (int i = 0; i < no; i++) { int d[MAXR]; int r = ro_output_shape(m, i, d); out_numel[i] = shape_numel(d, r); }
    int failed = 0;
    char first_err[256] = {0};
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel num_threads(nthreads)
#endif
    {
        double *ib[16], *ob[16];
        for (int i = 0; i < ni; i++) ib[i] = (double *)malloc(sizeof(double) * (size_t)in_numel[i]);
        for (int i = 0; i < no; i++) ob[i] = (double *)malloc(sizeof(double) * (size_t)out_numel[i]);
        char lerr[256];
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
        for (int64_t s = 0; s < n; s++) {
            if (failed) continue;
            for (int i = 0; i < ni; i++) {
                int64_t pre = in_pre ? in_pre[i] : 1, post = in_numel[i] / pre;
                for (int64_t q = 0; q < post; q++)
                    for (int64_t p = 0; p < pre; p++) ib[i][p + pre * q] = inputs[i][p + pre * (s + n * q)];
            }
            if (ro_run(m, (const double *const *)ib, ob, lerr, sizeof(lerr))) {
#ifdef _OPENMP
#pragma omp critical
#endif
                {
                    if (!failed) snprintf(first_err, sizeof(first_err), "%s", lerr);
                    failed = 1;
                }
                continue;
            }
            for (int i = 0; i < no; i++) {
                int64_t pre = out_pre ? out_pre[i] : 1, post = out_numel[i] / pre;
                for (int64_t q = 0; q < post; q++)
                    for (int64_t p = 0; p < pre; p++) outputs[i][p + pre * (s + n * q)] = ob[i][p + pre * q];
            }
        }
        for (int i = 0; i < ni; i++) free(ib[i]);
        for (int i = 0; i < no; i++) free(ob[i]);
    }
    if (failed) { set_err(err, errlen, "%s", first_err); return -1; }
    return 0;
}

int ro_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
