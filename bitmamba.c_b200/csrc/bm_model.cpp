// Reader of jserv/bitmamba.c's packed model file for the tensors the decode
// tail needs: the final RMSNorm weight (norm_f), the lm_head BitLinear's
// RMSNorm weight and its 2-bit ternary weights with their scale.
//
// Format (written by scripts/export-bin.py:110-200, read by src/model.c:
// 367-475 and 554-626): a header of five int32 (magic 0x42495432,
// vocab_size, d_model, n_layers, n_heads), then every tensor in a fixed
// order (embed; per layer in_proj.norm, in_proj, conv1d.weight, conv1d.bias,
// dt_bias, A_log, D, out_proj.norm, out_proj; norm_f, lm_head.norm,
// lm_head), each either float (int32 0, int32 ndim <= 4, the dims, fp32
// data) or packed ternary (int32 2, int32 rows, int32 cols, fp32 scale,
// rows * ((cols + 3) / 4) bytes).  Tensors are read sequentially, so the
// reader walks all of them; it applies the reference loader's checks (the
// header bounds, each tensor's bounds, and the shape and type checks of
// src/model.c:630-783) and fails with BM_ERR_INVALID_ARG naming the check.
#include <climits>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cuda_runtime.h>

#include "bm_sampler.h"

int bm_detail_fail(int code, const char *msg);

namespace {

constexpr int MAGIC = 0x42495432;   // src/bitmamba.h:15
constexpr int MAX_DIM = 1 << 20;    // src/bitmamba.h:54
constexpr int MAX_VOCAB = 256000;   // src/bitmamba.h:55
constexpr int EXPAND = 2;           // src/bitmamba.h:48
constexpr int CONV = 4;             // src/bitmamba.h:49

int mfail(int code, const std::string &msg) { return bm_detail_fail(code, msg.c_str()); }

int rd_int(const uint8_t *p) {
    int v;
    memcpy(&v, p, 4);
    return v;
}
float rd_float(const uint8_t *p) {
    float v;
    memcpy(&v, p, 4);
    return v;
}

struct Tensor {
    const uint8_t *data = nullptr;  // fp32 values or packed bytes
    int rows = 0, cols = 0;
    size_t n = 0;
    bool bitnet = false;
    float scale = 1.0f;
};

// One tensor at p (src/model.c:367-475); bytes consumed, 0 on error.
size_t read_tensor(const uint8_t *p, const uint8_t *end, Tensor *t, std::string *why) {
    *t = Tensor();
    const uint8_t *start = p;
    if (end - p < 4) return 0;
    const int type = rd_int(p);
    p += 4;
    if (type == 2) {
        if (end - p < 12) return 0;
        t->bitnet = true;
        t->rows = rd_int(p);
        t->cols = rd_int(p + 4);
        t->scale = rd_float(p + 8);
        p += 12;
        if (!std::isfinite(t->scale) || t->scale <= 0.0f) {
            *why = "invalid bitnet scale";
            return 0;
        }
        if (t->rows <= 0 || t->rows > MAX_DIM || t->cols <= 0 || t->cols > MAX_DIM) {
            *why = "invalid tensor dims";
            return 0;
        }
        const size_t bytes = (size_t)t->rows * (size_t)((t->cols + 3) / 4);
        if (bytes > (size_t)(end - p)) return 0;
        t->data = p;
        t->n = (size_t)t->rows * (size_t)t->cols;
        p += bytes;
    } else {
        if (end - p < 4) return 0;
        const int ndim = rd_int(p);
        p += 4;
        if (ndim < 0 || ndim > 4) return 0;
        if ((size_t)(end - p) < (size_t)ndim * 4) return 0;
        size_t total = 1;
        for (int i = 0; i < ndim; ++i) {
            const int d = rd_int(p);
            p += 4;
            if (d <= 0 || d > MAX_DIM) return 0;
            if (total > SIZE_MAX / (size_t)d) {
                *why = "float tensor size overflow";
                return 0;
            }
            total *= (size_t)d;
            if (i == 0) t->rows = d;
            if (i == 1) t->cols = d;
        }
        if (total > SIZE_MAX / 4) return 0;
        if (total * 4 > (size_t)(end - p)) return 0;
        t->data = p;
        t->n = total;
        p += total * 4;
    }
    return (size_t)(p - start);
}

struct Layer {
    Tensor in_norm, in_proj, conv_w, conv_b, dt_bias, a_log, d, out_norm, out_proj;
};

// The whole file walk with the reference loader's checks; the three head
// tensors out.
int parse(const uint8_t *base, size_t size, int cfg[4], Tensor *norm_f, Tensor *lmh_norm,
          Tensor *lm_head) {
    if (size < 20) return mfail(BM_ERR_INVALID_ARG, "model file too small");
    const uint8_t *p = base, *end = base + size;
    if (rd_int(p) != MAGIC) return mfail(BM_ERR_INVALID_ARG, "wrong format (need packed .bin)");
    for (int i = 0; i < 4; ++i) cfg[i] = rd_int(p + 4 + 4 * i);
    p += 20;
    const int vocab = cfg[0], dm = cfg[1], nl = cfg[2], nh = cfg[3];
    if (vocab <= 0 || vocab > MAX_VOCAB || dm <= 0 || dm > MAX_DIM || nl <= 0 || nl > 256 ||
        nh <= 0 || nh > MAX_DIM)
        return mfail(BM_ERR_INVALID_ARG, "invalid model config (vocab " + std::to_string(vocab) +
                                             ", d_model " + std::to_string(dm) + ", n_layers " +
                                             std::to_string(nl) + ", n_heads " +
                                             std::to_string(nh) + ")");
    std::string why;
    auto rd = [&](Tensor *t, const std::string &name) -> int {
        const size_t c = read_tensor(p, end, t, &why);
        if (!c)
            return mfail(BM_ERR_INVALID_ARG,
                         "failed to read tensor " + name + (why.empty() ? "" : ": " + why));
        p += c;
        return BM_OK;
    };
    Tensor embed;
    int rc = rd(&embed, "embed");
    if (rc) return rc;
    std::vector<Layer> L((size_t)nl);
    for (int i = 0; i < nl; ++i) {
        const std::string pre = "layers." + std::to_string(i) + ".";
        Layer &l = L[(size_t)i];
        if ((rc = rd(&l.in_norm, pre + "in_proj.norm")) || (rc = rd(&l.in_proj, pre + "in_proj")) ||
            (rc = rd(&l.conv_w, pre + "conv1d.weight")) || (rc = rd(&l.conv_b, pre + "conv1d.bias")) ||
            (rc = rd(&l.dt_bias, pre + "dt_bias")) || (rc = rd(&l.a_log, pre + "A_log")) ||
            (rc = rd(&l.d, pre + "D")) || (rc = rd(&l.out_norm, pre + "out_proj.norm")) ||
            (rc = rd(&l.out_proj, pre + "out_proj")))
            return rc;
    }
    if ((rc = rd(norm_f, "norm_f")) || (rc = rd(lmh_norm, "lm_head.norm")) ||
        (rc = rd(lm_head, "lm_head")))
        return rc;
    // shape and type checks (src/model.c:630-783)
    const size_t di = (size_t)dm * EXPAND;
    auto bad = [&](const std::string &m) { return mfail(BM_ERR_INVALID_ARG, m); };
    if (norm_f->n < (size_t)dm) return bad("norm_f smaller than d_model");
    if (lmh_norm->n < (size_t)dm) return bad("lm_head_norm smaller than d_model");
    for (int i = 0; i < nl; ++i)
        if (L[(size_t)i].in_norm.n < (size_t)dm)
            return bad("layer " + std::to_string(i) + " in_proj_norm smaller than d_model");
    if (embed.n < (size_t)vocab * (size_t)dm) return bad("embed smaller than vocab * d_model");
    if (lm_head->rows != vocab || lm_head->cols != dm)
        return bad("lm_head shape mismatch (have " + std::to_string(lm_head->rows) + "x" +
                   std::to_string(lm_head->cols) + ", need " + std::to_string(vocab) + "x" +
                   std::to_string(dm) + ")");
    if (di % (size_t)nh != 0) return bad("d_inner not divisible by n_heads");
    const int exp_proj = (int)(2 * di) + 3 * nh;
    for (int i = 0; i < nl; ++i) {
        const Layer &l = L[(size_t)i];
        const std::string li = "layer " + std::to_string(i) + " ";
        if (l.in_proj.cols != dm) return bad(li + "in_proj.cols != d_model");
        if (l.in_proj.rows != exp_proj) return bad(li + "in_proj.rows != 2 d_inner + 3 n_heads");
        if (l.out_proj.rows != dm || (size_t)l.out_proj.cols != di)
            return bad(li + "out_proj shape != d_model x d_inner");
        if (l.conv_w.n < di * CONV || l.conv_b.n < di || l.dt_bias.n < (size_t)nh ||
            l.a_log.n < (size_t)nh || l.d.n < di || l.out_norm.n < di)
            return bad(li + "float tensor smaller than its shape");
    }
    if (embed.bitnet || norm_f->bitnet || lmh_norm->bitnet)
        return bad("embed/norm_f/lm_head_norm must be float, not bitnet");
    if (!lm_head->bitnet) return bad("lm_head must be bitnet-packed");
    for (int i = 0; i < nl; ++i) {
        const Layer &l = L[(size_t)i];
        if (!l.in_proj.bitnet || !l.out_proj.bitnet)
            return bad("layer " + std::to_string(i) + " in_proj/out_proj must be bitnet-packed");
        if (l.in_norm.bitnet || l.out_norm.bitnet || l.conv_w.bitnet || l.conv_b.bitnet ||
            l.dt_bias.bitnet || l.a_log.bitnet || l.d.bitnet)
            return bad("layer " + std::to_string(i) + " float tensors must not be bitnet-packed");
    }
    return BM_OK;
}

struct Mapped {
    void *addr = nullptr;
    size_t size = 0;
    ~Mapped() {
        if (addr) munmap(addr, size);
    }
};

int map_file(const char *path, Mapped *m) {
    if (!path) return mfail(BM_ERR_INVALID_ARG, "path is NULL");
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return mfail(BM_ERR_INVALID_ARG, std::string("cannot open model file ") + path);
    struct stat sb;
    if (fstat(fd, &sb) < 0 || sb.st_size <= 0) {
        close(fd);
        return mfail(BM_ERR_INVALID_ARG, "model file too small");
    }
    m->size = (size_t)sb.st_size;
    void *a = mmap(nullptr, m->size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (a == MAP_FAILED) return mfail(BM_ERR_INVALID_ARG, "mmap failed");
    m->addr = a;
    return BM_OK;
}

int read_head(const char *path, bm_model_head_host_t *h) {
    memset(h, 0, sizeof(*h));
    Mapped m;
    int rc = map_file(path, &m);
    if (rc) return rc;
    int cfg[4];
    Tensor nf, nl, lm;
    rc = parse(static_cast<const uint8_t *>(m.addr), m.size, cfg, &nf, &nl, &lm);
    if (rc) return rc;
    const int dm = cfg[1];
    const size_t pk = (size_t)lm.rows * (size_t)((lm.cols + 3) / 4);
    h->norm_f = static_cast<float *>(malloc((size_t)dm * 4));
    h->lm_head_norm = static_cast<float *>(malloc((size_t)dm * 4));
    h->packed = static_cast<uint8_t *>(malloc(pk));
    if (!h->norm_f || !h->lm_head_norm || !h->packed) {
        bm_model_head_host_free(h);
        return mfail(BM_ERR_OOM, "host allocation");
    }
    memcpy(h->norm_f, nf.data, (size_t)dm * 4);  // the first d_model values are used
    memcpy(h->lm_head_norm, nl.data, (size_t)dm * 4);
    memcpy(h->packed, lm.data, pk);
    h->vocab_size = cfg[0];
    h->d_model = dm;
    h->n_layers = cfg[2];
    h->n_heads = cfg[3];
    h->w_scale = lm.scale;
    return BM_OK;
}

}  // namespace

struct bm_model_head {
    bm_model_head_info_t info;
    int device;
};

extern "C" {

int bm_model_head_read(const char *path, bm_model_head_host_t *out) {
    if (!out) return mfail(BM_ERR_INVALID_ARG, "out is NULL");
    return read_head(path, out);
}

void bm_model_head_host_free(bm_model_head_host_t *h) {
    if (!h) return;
    free(h->norm_f);
    free(h->lm_head_norm);
    free(h->packed);
    h->norm_f = h->lm_head_norm = nullptr;
    h->packed = nullptr;
}

int bm_model_head_load(bm_ctx_t *ctx, const char *path, bm_model_head_t **out) {
    if (!out) return mfail(BM_ERR_INVALID_ARG, "out is NULL");
    *out = nullptr;
    if (!ctx) return mfail(BM_ERR_INVALID_ARG, "ctx is NULL");
    bm_model_head_host_t h;
    int rc = read_head(path, &h);
    if (rc) return rc;
    const int V = h.vocab_size, dm = h.d_model;
    if (dm % 32 || dm > 4096) {
        bm_model_head_host_free(&h);
        return mfail(BM_ERR_UNSUPPORTED, "d_model " + std::to_string(dm) +
                                             " (the GPU lm_head needs a multiple of 32, <= 4096)");
    }
    int dev = 0;
    if ((rc = bm_ctx_device(ctx, &dev)) != BM_OK) {
        bm_model_head_host_free(&h);
        return rc;
    }
    bm_model_head_t *m = static_cast<bm_model_head_t *>(calloc(1, sizeof(bm_model_head_t)));
    if (!m) {
        bm_model_head_host_free(&h);
        return mfail(BM_ERR_OOM, "calloc");
    }
    m->device = dev;
    bm_model_head_info_t &I = m->info;
    I.vocab_size = V;
    I.d_model = dm;
    I.n_layers = h.n_layers;
    I.n_heads = h.n_heads;
    I.w_scale = h.w_scale;
    const size_t pk = (size_t)V * (size_t)(dm / 4);
    cudaError_t e = cudaSetDevice(dev);
    float *nf = nullptr, *nl = nullptr;
    int8_t *w8 = nullptr;
    uint8_t *pd = nullptr;
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void **>(&nf), (size_t)dm * 4);
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void **>(&nl), (size_t)dm * 4);
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void **>(&pd), pk);
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void **>(&w8), (size_t)V * dm);
    if (e == cudaSuccess) e = cudaMemcpy(nf, h.norm_f, (size_t)dm * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(nl, h.lm_head_norm, (size_t)dm * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(pd, h.packed, pk, cudaMemcpyHostToDevice);
    bm_model_head_host_free(&h);
    I.d_norm_f = nf;
    I.d_lmh_norm = nl;
    I.d_packed = pd;
    I.d_w8 = w8;
    if (e != cudaSuccess) {
        bm_model_head_free(m);
        char buf[200];
        snprintf(buf, sizeof(buf), "model head upload: %s", cudaGetErrorString(e));
        return bm_detail_fail(e == cudaErrorMemoryAllocation ? BM_ERR_OOM : BM_ERR_CUDA, buf);
    }
    rc = bm_ternary_unpack(ctx, pd, V, dm, w8, nullptr);
    if (rc == BM_OK) {
        e = cudaStreamSynchronize(static_cast<cudaStream_t>(bm_ctx_stream(ctx)));
        if (e != cudaSuccess) rc = bm_detail_fail(BM_ERR_CUDA, cudaGetErrorString(e));
    }
    if (rc != BM_OK) {
        bm_model_head_free(m);
        return rc;
    }
    *out = m;
    return BM_OK;
}

int bm_model_head_info(const bm_model_head_t *m, bm_model_head_info_t *info) {
    if (!m || !info) return mfail(BM_ERR_INVALID_ARG, "head or info is NULL");
    *info = m->info;
    return BM_OK;
}

void bm_model_head_free(bm_model_head_t *m) {
    if (!m) return;
    cudaSetDevice(m->device);
    cudaFree(const_cast<float *>(m->info.d_norm_f));
    cudaFree(const_cast<float *>(m->info.d_lmh_norm));
    cudaFree(const_cast<int8_t *>(m->info.d_w8));
    cudaFree(const_cast<uint8_t *>(m->info.d_packed));
    free(m);
}

}  // extern "C"
