// Host engine behind include/cuda_inference.h: model/cache lifetime, weight repacking and upload,
// launches of the persistent decode kernel (decode_kernel.cuh), token streaming to the host, and
// the standalone GEMV / argmax / read-probe kernels.
//
// Replaces metal_infrence_engine/src/metal_inference.rs. Differences that follow from the
// hardware: B200 has no unified memory, so load_model copies the weights to HBM (repacking q|k|v
// into one matrix and interleaving gate/up rows, so one streaming pass per phase reads them);
// a whole token, and a whole greedy decode, is one cooperative kernel launch instead of ~424
// dispatches per token.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/cuda_inference.h"
#include "cluster_decode.cuh"
#include "decode_kernel.cuh"
#include "batch_kernel.cuh"
#include "model_file.h"
#include "prefill.h"

using namespace qw;

namespace {

thread_local std::string g_err;

int set_err(int code, const std::string& msg) {
    g_err = msg;
    return code;
}

int cuda_err(cudaError_t e, const char* what) {
    return set_err(QW_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

#define QW_CUDA(call)                                            \
    do {                                                         \
        cudaError_t e_ = (call);                                 \
        if (e_ != cudaSuccess) return cuda_err(e_, #call);       \
    } while (0)

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

long long timeout_ns_from_env() {
    const char* s = std::getenv("QW_WAIT_TIMEOUT_MS");
    long long ms = s ? std::atoll(s) : 4000;
    if (ms < 50) ms = 50;
    return ms * 1000000LL;
}

const char* derr_name(int code) {
    switch (code) {
        case DERR_TIMEOUT_GRID: return "grid barrier wait expired";
        case DERR_TIMEOUT_FULL: return "ring-slot data wait expired";
        case DERR_TIMEOUT_EMPTY: return "ring-slot release wait expired";
        case DERR_TIMEOUT_KV: return "KV visibility wait expired";
        case DERR_BAD_TOKEN: return "input token id >= vocab_size";
        case DERR_TIMEOUT_DRAIN: return "bulk-copy drain wait expired";
        case DERR_TIMEOUT_DATA: return "activation hand-off wait expired";
        case DERR_SHAPE: return "decode kernel variant does not cover the model's shapes";
        default: return "unknown device error";
    }
}

}  // namespace

namespace qw {

int set_error(int code, const char* msg) { return set_err(code, msg); }

// lazily allocated 16-byte error word per device, for the standalone kernels
int* device_err_word_for(int device) {
    static std::mutex mu;
    static std::vector<int*> words;
    std::lock_guard<std::mutex> lock(mu);
    if ((int)words.size() <= device) words.resize(device + 1, nullptr);
    if (!words[device]) {
        int* p = nullptr;
        if (cudaMalloc(&p, 16) != cudaSuccess) return nullptr;
        cudaMemset(p, 0, 16);
        words[device] = p;
    }
    return words[device];
}

}  // namespace qw

namespace qw {

// the persistent decode kernel (device code in decode_kernel.cuh), in four variants: with or without
// the phase-timeline stamps, with or without the GEMV routine for shapes that are not whole
// 1024-column segments (kernel_for picks one per launch)
// 13 warps: one SM sub-partition holds 4 of them, so 16K registers / 128 threads caps it at 128 each
template <bool kTrace, bool kGeneric>
__global__ void __launch_bounds__(NTHREADS, 1) decode_kernel(const __grid_constant__ DecodeParams p) {
    using Decoder = DecoderT<kTrace, kGeneric>;
    if (threadIdx.x == 0) {
        for (int i = 0; i < NSLOT; i++) {
            mbar_init(&qw_sm.full[i], 1);
            mbar_init(&qw_sm.empty[i], NCW);
        }
        qw_sm.progress = 0;
        qw_sm.abort = 0;
        qw_sm.token = 0;
        qw_sm.prm = p;
        for (int w = 0; w <= NCW; w++) qw_sm.ring_it[w] = 0;
        qw_sm.n_issued = 0;
        Decoder::init_geometry(p);
        fence_mbar_init();
    }
    __syncthreads();
    if (Decoder::warp() == NCW) {
        if (Decoder::lane() == 0) Decoder::produce();
        return;
    }
    Decoder::consume();
}

// the decode kernel variant for a launch: stamps only when tracing, the generic GEMV routine only
// for shapes that need it
inline const void* kernel_for(bool trace, bool generic) {
    if (trace) return generic ? (const void*)decode_kernel<true, true> : (const void*)decode_kernel<true, false>;
    return generic ? (const void*)decode_kernel<false, true> : (const void*)decode_kernel<false, false>;
}

}  // namespace qw

struct qw_model {
    uint64_t id = 0;  // unique per load, so a cache can tell its model from a later one at the same address
    int device = 0;
    cudaStream_t stream = nullptr;
    int nctas = 0;    // grid of the decode kernel in use
    int kind = 0;     // QW_DECODER_GRID (decode_kernel.cuh) or QW_DECODER_CLUSTER (cluster_decode.cuh)
    bool generic = true;  // grid kernel: the shapes need the generic GEMV routine (full_segment_shapes)
    // persistent batch kernel (batch_kernel.cuh): 0 unchecked, 1 usable, -1 not for this model;
    // bk_use: qw_decode_batch runs it for batches of at most 8 rows (QW_BATCH_DECODER)
    int bk_state = 0;
    bool bk_use = false;
    uint8_t* d_bk = nullptr;     // its scratch: tagged x, q|k|v, h, att, partials, then argmax partials and flags
    u64 *bk_x = nullptr, *bk_qkv = nullptr, *bk_h = nullptr, *bk_att = nullptr, *bk_apart = nullptr, *bk_flags = nullptr;
    float* bk_am_val = nullptr;
    unsigned* bk_am_idx = nullptr;
    int* bk_nan0 = nullptr;
    size_t bk_tagged_bytes = 0;
    unsigned bk_epoch = 0;
    int bk_S = 1;
    bool cl_coop = true;          // cluster launches also ask for co-residency (cooperative) until refused
    uint16_t* d_clw = nullptr;    // cluster kernel: o_proj and down_proj repacked per (layer, cluster, rank)
    u64 *d_po = nullptr, *d_pd = nullptr;  // cluster kernel: [8][hidden] partial residual updates (tagged words)
    ModelConfig cfg;
    uint64_t wbytes = 0;
    // weights
    uint16_t* d_weights = nullptr;  // one allocation: layers | norms | final norm | embed | lm_head
    uint16_t *d_layer_w = nullptr, *d_layer_n = nullptr, *d_final_norm = nullptr, *d_embed = nullptr, *d_lm_head = nullptr;
    long long layer_stride = 0, norm_stride = 0;
    // scratch (one allocation)
    uint8_t* d_scratch = nullptr;
    u64 *d_x = nullptr, *d_qkv = nullptr, *d_att = nullptr, *d_h = nullptr, *d_apart = nullptr;  // tagged words
    float *d_am_val = nullptr, *d_logits = nullptr;
    unsigned* d_am_idx = nullptr;
    int *d_nan0 = nullptr, *d_err = nullptr;
    u64* d_flags = nullptr;
    // token ring (device) and its mapped host mirror
    uint32_t* d_tok = nullptr;
    size_t tok_cap = 0;
    uint32_t* h_tok = nullptr;   // mapped pinned [cap]
    unsigned* h_count = nullptr; // mapped pinned
    uint32_t* h_tok_dev = nullptr;
    unsigned* h_count_dev = nullptr;
    size_t h_cap = 0;
    uint32_t* h_stage = nullptr; // pinned, 1 token
    float* h_logits = nullptr;   // pinned [vocab]
    // staged copy-out of large results to pageable host memory (copy_to_host): two pinned stages
    uint8_t* h_out_stage = nullptr;
    cudaEvent_t out_ev[2] = {nullptr, nullptr};
    // batched prefill: scratch for up to pf.cap tokens, their ids and (when asked for) logits
    qw::pf::Scratch pf;
    uint32_t* d_pf_ids = nullptr;
    float* d_pf_logits = nullptr;
    size_t pf_logits_cap = 0;    // tokens d_pf_logits holds
    // batch decode (row mode): row views, current tokens, the [steps][B] token record, and the
    // captured graph of one step with the configuration it was captured for
    qw::pf::RowView* d_rows = nullptr;   // [ROWS_MAX]
    uint32_t* d_btok = nullptr;          // [ROWS_MAX]
    qw::pf::ArgmaxScratch* d_am = nullptr;
    uint32_t* d_bout = nullptr;
    size_t bout_cap = 0;                 // entries of d_bout
    // captured row-mode step graphs, by what they were captured for (kind 0: greedy batch step,
    // kind 1: lookup verify pass) and the buffers they bake in
    struct GraphKey {
        int kind, B, splits;
        const void *X, *Y, *attp, *logits, *out;
        bool operator==(const GraphKey& o) const {
            return kind == o.kind && B == o.B && splits == o.splits && X == o.X && Y == o.Y && attp == o.attp &&
                   logits == o.logits && out == o.out;
        }
    };
    std::vector<std::pair<GraphKey, cudaGraphExec_t>> graphs;
    unsigned epoch = 0;
    int S = 0, part_cap = 0, xs_cap = 0, xloc_cap = 0;
    u64* d_trace = nullptr;      // phase timeline of the most recent launch's first step, if enabled
    size_t dyn_smem = 0;
    long long timeout_ns = 0;
    int poll_ns = 0;
    int min_chunk = MIN_CHUNK;
    int stall_cta = -1;          // QW_TEST_STALL_CTA: consumed by the next launch only (timeout test hook)
};

// A cache never dereferences its model after qw_cache_new: it keeps what it needs (device,
// geometry), so caches and models may be freed in either order. `m` is only compared.
struct qw_cache {
    const qw_model* m = nullptr;
    uint64_t model_id = 0;
    int device = 0;
    uint64_t layers = 0, kv_heads = 0, head_dim = 0;
    size_t max_seq = 0;
    float* d_k = nullptr;
    float* d_v = nullptr;
    float2* d_rope = nullptr;
};

namespace {

int ensure_token_capacity(qw_model* m, size_t n) {
    if (n > m->tok_cap) {
        size_t cap = std::max<size_t>(n, 2 * m->tok_cap);
        uint32_t* d = nullptr;
        if (cudaMalloc(&d, cap * 4) != cudaSuccess) return set_err(QW_ERR_NOMEM, "token ring allocation failed");
        if (m->d_tok) cudaFree(m->d_tok);
        m->d_tok = d;
        m->tok_cap = cap;
    }
    if (n > m->h_cap) {
        size_t cap = std::max<size_t>(n, 2 * m->h_cap);
        void* h = nullptr;
        if (cudaHostAlloc(&h, cap * 4 + 64, cudaHostAllocMapped) != cudaSuccess)
            return set_err(QW_ERR_NOMEM, "pinned token ring allocation failed");
        if (m->h_tok) cudaFreeHost(m->h_tok);
        m->h_tok = static_cast<uint32_t*>(h);
        m->h_count = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(h) + cap * 4 + 32);
        QW_CUDA(cudaHostGetDevicePointer((void**)&m->h_tok_dev, m->h_tok, 0));
        QW_CUDA(cudaHostGetDevicePointer((void**)&m->h_count_dev, m->h_count, 0));
        m->h_cap = cap;
    }
    return QW_OK;
}

// The epoch of the next launch. Tagged hand-off words carry the low 12 bits of it, so a word left by
// a launch 4096 launches earlier (e.g. a longer decode, whose later steps' words nothing has
// overwritten since) could carry a tag that matches again: whenever those bits wrap, the tagged
// buffers are cleared first (stream-ordered, before the launch).
int next_epoch(qw_model* m, cudaStream_t s) {
    const unsigned e = ++m->epoch;
    if ((e & 0xFFFu) == 0 && e != 0) {
        // the grid kernel's tagged buffers (x, q|k|v, att, h, attention partials) lead the scratch block
        const size_t tagged_bytes = (size_t)(reinterpret_cast<uint8_t*>(m->d_am_val) - m->d_scratch);
        QW_CUDA(cudaMemsetAsync(m->d_scratch, 0, tagged_bytes, s));
        QW_CUDA(cudaMemsetAsync(m->d_po, 0, (size_t)cl::NKV * m->cfg.hidden * 8, s));
        QW_CUDA(cudaMemsetAsync(m->d_pd, 0, (size_t)cl::NKV * m->cfg.hidden * 8, s));
    }
    return QW_OK;
}

// the cluster decode kernel (cluster_decode.cuh): 8 clusters of 16 CTAs, one per KV head
int launch_cluster(qw_model* m, qw_cache* c, const uint32_t* tok_in, uint32_t* tok_out, bool stream_to_host,
                   float* logits, size_t start_pos, size_t steps, cudaStream_t s) {
    const ModelConfig& g = m->cfg;
    cl::Params p{};
    p.layer_w = m->d_layer_w;
    p.o_blk = m->d_clw;
    p.d_blk = m->d_clw + (size_t)g.layers * cl::NKV * cl::CL * cl::XO * cl::OK;
    p.layer_n = m->d_layer_n;
    p.final_norm = m->d_final_norm;
    p.embed = m->d_embed;
    p.lm_head = m->d_lm_head;
    p.kc = c->d_k;
    p.vc = c->d_v;
    p.rope = c->d_rope;
    p.po = m->d_po;
    p.pd = m->d_pd;
    p.am_val = m->d_am_val;
    p.am_idx = m->d_am_idx;
    p.nan0 = m->d_nan0;
    p.flags = m->d_flags;
    p.err = m->d_err;
    p.logits = logits;
    p.trace = m->d_trace;
    p.tok_in = tok_in;
    p.tok_out = tok_out;
    p.host_tok = stream_to_host ? m->h_tok_dev : nullptr;
    p.host_count = stream_to_host ? m->h_count_dev : nullptr;
    p.layer_stride = m->layer_stride;
    p.norm_stride = m->norm_stride;
    p.L = (int)g.layers;
    p.V = (int)g.vocab;
    p.max_seq = (int)c->max_seq;
    p.start_pos = (int)start_pos;
    p.steps = (int)steps;
    p.eps = g.eps;
    p.scale = 1.0f / sqrtf((float)g.head_dim);  // cpu_inference.rs:144
    p.timeout_ns = m->timeout_ns;
    p.stall_cta = m->stall_cta;
    m->stall_cta = -1;
    if (int e = next_epoch(m, s)) return e;
    p.epoch = m->epoch;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(m->nctas);
    cfg.blockDim = dim3(cl::NTHREADS);
    cfg.dynamicSmemBytes = cl::DYN_BYTES;
    cfg.stream = s;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = cl::CL;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeCooperative;
    at[1].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = m->cl_coop ? 2 : 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, cl::cluster_decode_kernel, p);
    if (e != cudaSuccess && m->cl_coop) {
        // a driver that does not combine cooperative and cluster launches: the load-time occupancy
        // check (every cluster fits at once on an otherwise idle GPU) stands in for it
        (void)cudaGetLastError();
        m->cl_coop = false;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, cl::cluster_decode_kernel, p);
    }
    if (e != cudaSuccess) return cuda_err(e, "cluster decode kernel launch");
    return QW_OK;
}

int launch_decode(qw_model* m, qw_cache* c, const uint32_t* tok_in, uint32_t* tok_out, bool stream_to_host,
                  float* logits, size_t start_pos, size_t steps, cudaStream_t s) {
    if (m->kind == QW_DECODER_CLUSTER) return launch_cluster(m, c, tok_in, tok_out, stream_to_host, logits, start_pos, steps, s);
    const ModelConfig& g = m->cfg;
    DecodeParams p{};
    p.layer_w = m->d_layer_w;
    p.layer_n = m->d_layer_n;
    p.final_norm = m->d_final_norm;
    p.embed = m->d_embed;
    p.lm_head = m->d_lm_head;
    p.kc = c->d_k;
    p.vc = c->d_v;
    p.rope = c->d_rope;
    p.x = m->d_x;
    p.qkv = m->d_qkv;
    p.hbuf = m->d_h;
    p.att = m->d_att;
    p.apart = m->d_apart;
    p.am_val = m->d_am_val;
    p.am_idx = m->d_am_idx;
    p.nan0 = m->d_nan0;
    p.flags = m->d_flags;
    p.err = m->d_err;
    p.logits = logits;
    p.trace = m->d_trace;
    p.tok_in = tok_in;
    p.tok_out = tok_out;
    p.host_tok = stream_to_host ? m->h_tok_dev : nullptr;
    p.host_count = stream_to_host ? m->h_count_dev : nullptr;
    p.layer_stride = m->layer_stride;
    p.norm_stride = m->norm_stride;
    p.H = (int)g.hidden;
    p.I = (int)g.inter;
    p.L = (int)g.layers;
    p.NQ = (int)g.heads;
    p.NKV = (int)g.kv_heads;
    p.V = (int)g.vocab;
    p.max_seq = (int)c->max_seq;
    p.start_pos = (int)start_pos;
    p.steps = (int)steps;
    if (int e = next_epoch(m, s)) return e;
    p.epoch = m->epoch;
    p.eps = g.eps;
    p.scale = 1.0f / sqrtf((float)g.head_dim);  // cpu_inference.rs:144
    p.S = m->S;
    p.part_cap = m->part_cap;
    p.xs_cap = m->xs_cap;
    p.xloc_cap = m->xloc_cap;
    p.timeout_ns = m->timeout_ns;
    p.poll_ns = m->poll_ns;
    p.min_chunk = m->min_chunk;
    p.stall_cta = m->stall_cta;
    m->stall_cta = -1;
    void* args[] = {&p};
    cudaError_t e = cudaLaunchCooperativeKernel(kernel_for(m->d_trace != nullptr, m->generic), dim3(m->nctas), dim3(NTHREADS), args,
                                                m->dyn_smem, s);
    if (e != cudaSuccess) return cuda_err(e, "decode kernel launch");
    return QW_OK;
}

// reads and clears the device error word after a synchronisation
int check_device_err(qw_model* m) {
    int err[4] = {0, 0, 0, 0};
    QW_CUDA(cudaMemcpy(err, m->d_err, sizeof err, cudaMemcpyDeviceToHost));
    if (err[0] == 0 && err[3] == 0) return QW_OK;
    QW_CUDA(cudaMemset(m->d_err, 0, sizeof err));
    char buf[256];
    std::snprintf(buf, sizeof buf, "device: %s (cta %d, at %d)%s", derr_name(err[0]), err[1], err[2],
                  err[3] ? "; a bulk-copy drain also expired" : "");
    return set_err(err[0] == DERR_BAD_TOKEN ? QW_ERR_ARG : QW_ERR_DEVICE_TIMEOUT, buf);
}

cudaStream_t pick_stream(qw_model* m, void* s) { return s ? static_cast<cudaStream_t>(s) : m->stream; }

// whether NKV clusters of 16 CTAs of the cluster kernel can be resident at once (`fit`: how many)
bool cluster_kernel_fits(int& fit) {
    fit = 0;
    if (cudaFuncSetAttribute(cl::cluster_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)cl::DYN_BYTES) !=
            cudaSuccess ||
        cudaFuncSetAttribute(cl::cluster_decode_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
        (void)cudaGetLastError();
        return false;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cl::NKV * cl::CL);
    cfg.blockDim = dim3(cl::NTHREADS);
    cfg.dynamicSmemBytes = cl::DYN_BYTES;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = cl::CL;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&fit, cl::cluster_decode_kernel, &cfg) != cudaSuccess) {
        (void)cudaGetLastError();
        fit = 0;
        return false;
    }
    return fit >= cl::NKV;
}

}  // namespace

extern "C" {

const char* qw_last_error(void) { return g_err.c_str(); }

int qw_inspect(const char* path, qw_config* out) {
    if (!path || !out) return set_err(QW_ERR_ARG, "null argument");
    ModelFile f;
    std::string msg;
    int rc = f.open(path, msg);
    if (rc) return set_err(rc, msg);
    const ModelConfig& c = f.config();
    *out = qw_config{c.hidden, c.inter, c.layers, c.heads, c.kv_heads, c.head_dim, c.vocab, c.eps, c.theta, c.eos};
    return QW_OK;
}

int qw_load(const char* path, int device, qw_model** out) {
    if (!path || !out) return set_err(QW_ERR_ARG, "null argument");
    *out = nullptr;
    ModelFile f;
    std::string msg;
    int rc = f.open(path, msg);
    if (rc) return set_err(rc, msg);
    const ModelConfig& c = f.config();

    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return set_err(QW_ERR_CUDA, "no CUDA device");
    if (device < 0 || device >= ndev) return set_err(QW_ERR_ARG, "device index out of range");
    QW_CUDA(cudaSetDevice(device));
    cudaDeviceProp prop;
    QW_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major < 10) return set_err(QW_ERR_UNSUPPORTED, "the kernels are built for sm_100a (B200)");
    if (!prop.cooperativeLaunch) return set_err(QW_ERR_UNSUPPORTED, "device lacks cooperative launch");

    static std::atomic<uint64_t> next_id{1};
    auto m = new qw_model();
    m->id = next_id.fetch_add(1);
    m->device = device;
    m->cfg = c;
    m->wbytes = f.weight_bytes_per_token();
    m->timeout_ns = timeout_ns_from_env();
    if (const char* e = std::getenv("QW_POLL_NS")) m->poll_ns = std::max(0, std::min(10000, std::atoi(e)));
    if (const char* e = std::getenv("QW_MIN_CHUNK")) m->min_chunk = std::max(1, std::min(1 << 20, std::atoi(e)));
    // test hook: the first launch of this model has CTA QW_TEST_STALL_CTA skip its end-of-token flag
    if (const char* e = std::getenv("QW_TEST_STALL_CTA")) m->stall_cta = std::atoi(e);
    int nctas = prop.multiProcessorCount;
    if (const char* e = std::getenv("QW_CTAS")) nctas = std::max(1, std::min(nctas, std::atoi(e)));
    // Buffers are reused across phases on the premise that a phase's input is complete only after
    // every CTA has finished reading the previous contents of the buffer it overwrites; the chain
    // that guarantees it passes through phase A (q|k|v), so every CTA must own q|k|v rows (the
    // o/down and gate|up partitions in 64-byte units may leave some CTAs without rows).
    nctas = (int)std::min<uint64_t>({(uint64_t)nctas, c.hidden, c.inter, c.heads * c.head_dim + 2 * c.kv_heads * c.head_dim});
    if ((uint64_t)nctas < c.kv_heads) { delete m; return set_err(QW_ERR_UNSUPPORTED, "fewer SMs than KV heads"); }
    m->nctas = nctas;
    m->S = std::min(MAX_S, nctas / (int)c.kv_heads);

    const uint64_t H = c.hidden, I = c.inter, QD = c.heads * c.head_dim, KVD = c.kv_heads * c.head_dim;
    const uint64_t QKVR = QD + 2 * KVD;
    m->layer_stride = (long long)(QKVR * H + H * QD + 2 * I * H + H * I);
    m->norm_stride = (long long)align_up(2 * H + 2 * c.head_dim, 64);
    const size_t n_layer_w = (size_t)m->layer_stride * c.layers;
    const size_t n_layer_n = (size_t)m->norm_stride * c.layers;
    const size_t off_n = align_up(n_layer_w, 128);
    const size_t off_f = off_n + align_up(n_layer_n, 128);
    const size_t off_e = off_f + align_up(H, 128);
    const size_t off_l = off_e + align_up(c.vocab * H, 128);
    const size_t total = off_l + c.vocab * H;

    auto fail = [&](int code, const std::string& why) {
        qw_free(m);
        return set_err(code, why);
    };
    if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess) return fail(QW_ERR_CUDA, "stream creation failed");
    if (cudaMalloc(&m->d_weights, total * 2) != cudaSuccess) return fail(QW_ERR_NOMEM, "weight allocation failed");
    m->d_layer_w = m->d_weights;
    m->d_layer_n = m->d_weights + off_n;
    m->d_final_norm = m->d_weights + off_f;
    m->d_embed = m->d_weights + off_e;
    m->d_lm_head = m->d_weights + off_l;

    // repack each layer into one block: q|k|v rows, o, gate/up interleaved by row, down
    {
        std::vector<uint16_t> blk((size_t)m->layer_stride);
        std::vector<uint16_t> nb((size_t)m->norm_stride * c.layers, 0);
        for (uint64_t l = 0; l < c.layers; l++) {
            const std::string p = "model.layers." + std::to_string(l) + ".";
            auto w = [&](const char* n) { return reinterpret_cast<const uint16_t*>(f.data(p + n)); };
            uint16_t* d = blk.data();
            std::memcpy(d, w("self_attn.q_proj.weight"), QD * H * 2);
            d += QD * H;
            std::memcpy(d, w("self_attn.k_proj.weight"), KVD * H * 2);
            d += KVD * H;
            std::memcpy(d, w("self_attn.v_proj.weight"), KVD * H * 2);
            d += KVD * H;
            std::memcpy(d, w("self_attn.o_proj.weight"), H * QD * 2);
            d += H * QD;
            const uint16_t* gt = w("mlp.gate_proj.weight");
            const uint16_t* up = w("mlp.up_proj.weight");
            for (uint64_t i = 0; i < I; i++) {
                std::memcpy(d + (2 * i) * H, gt + i * H, H * 2);
                std::memcpy(d + (2 * i + 1) * H, up + i * H, H * 2);
            }
            d += 2 * I * H;
            std::memcpy(d, w("mlp.down_proj.weight"), H * I * 2);
            if (cudaMemcpy(m->d_layer_w + l * m->layer_stride, blk.data(), blk.size() * 2, cudaMemcpyHostToDevice) != cudaSuccess)
                return fail(QW_ERR_CUDA, "weight upload failed");
            uint16_t* n = nb.data() + l * m->norm_stride;
            std::memcpy(n, w("input_layernorm.weight"), H * 2);
            std::memcpy(n + H, w("post_attention_layernorm.weight"), H * 2);
            std::memcpy(n + 2 * H, w("self_attn.q_norm.weight"), c.head_dim * 2);
            std::memcpy(n + 2 * H + c.head_dim, w("self_attn.k_norm.weight"), c.head_dim * 2);
        }
        if (cudaMemcpy(m->d_layer_n, nb.data(), nb.size() * 2, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(m->d_final_norm, f.data("model.norm.weight"), H * 2, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(m->d_embed, f.data("model.embed_tokens.weight"), c.vocab * H * 2, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(m->d_lm_head, f.data("lm_head.weight"), c.vocab * H * 2, cudaMemcpyHostToDevice) != cudaSuccess)
            return fail(QW_ERR_CUDA, "weight upload failed");
    }

    // The single-grid kernel (decode_kernel.cuh) runs every shape and is the default: on B200 one SM
    // takes in weights at only ~40 GB/s, so reaching HBM bandwidth needs every SM streaming.
    // QW_DECODER=cluster selects the cluster kernel (cluster_decode.cuh: 8 clusters of 8 CTAs, one per
    // KV head, activations exchanged through distributed shared memory) for the Qwen3-0.6B layer
    // shape; it streams on 64 SMs only, which bounds it below the grid kernel here.
    {
        const bool shape = H == (uint64_t)cl::H && I == (uint64_t)cl::I && c.heads == (uint64_t)cl::NQ &&
                           c.kv_heads == (uint64_t)cl::NKV && c.head_dim == (uint64_t)cl::HD;
        const char* bd = std::getenv("QW_BATCH_DECODER");
        m->bk_use = bd && std::strcmp(bd, "persistent") == 0;
        const char* dec = std::getenv("QW_DECODER");
        if (dec && std::strcmp(dec, "cluster") == 0) {
            if (!shape || std::getenv("QW_CTAS"))
                return fail(QW_ERR_UNSUPPORTED, "QW_DECODER=cluster: the cluster kernel needs the Qwen3-0.6B layer "
                                                "shape and no QW_CTAS");
            int fit = 0;
            if (!cluster_kernel_fits(fit))
                return fail(QW_ERR_UNSUPPORTED, "QW_DECODER=cluster: " + std::to_string(fit) + " clusters of " +
                                                    std::to_string(cl::CL) + " CTAs fit at once, " +
                                                    std::to_string(cl::NKV) + " are needed");
            m->kind = QW_DECODER_CLUSTER;
            m->nctas = cl::NKV * cl::CL;
        }
    }
    if (m->kind == QW_DECODER_CLUSTER) {
        // o_proj and down_proj once more, as the contiguous block of each (layer, cluster g, rank r):
        // rows [64r, 64r+64) over o's columns [256g, +256) and down's columns [384g, +384)
        const size_t per_o = (size_t)cl::NKV * cl::CL * cl::XO * cl::OK, per_d = (size_t)cl::NKV * cl::CL * cl::XO * cl::DK;
        if (cudaMalloc(&m->d_clw, (per_o + per_d) * c.layers * 2) != cudaSuccess)
            return fail(QW_ERR_NOMEM, "cluster weight allocation failed");
        std::vector<uint16_t> ob(per_o), db(per_d);
        for (uint64_t l = 0; l < c.layers; l++) {
            const std::string pre = "model.layers." + std::to_string(l) + ".";
            const uint16_t* o = reinterpret_cast<const uint16_t*>(f.data(pre + "self_attn.o_proj.weight"));
            const uint16_t* d = reinterpret_cast<const uint16_t*>(f.data(pre + "mlp.down_proj.weight"));
            for (int g = 0; g < cl::NKV; g++)
                for (int r = 0; r < cl::CL; r++)
                    for (int i = 0; i < cl::XO; i++) {
                        const size_t row = (size_t)cl::XO * r + i, blk = ((size_t)g * cl::CL + r) * cl::XO + i;
                        std::memcpy(&ob[blk * cl::OK], o + row * QD + (size_t)cl::OK * g, cl::OK * 2);
                        std::memcpy(&db[blk * cl::DK], d + row * I + (size_t)cl::DK * g, cl::DK * 2);
                    }
            if (cudaMemcpy(m->d_clw + l * per_o, ob.data(), per_o * 2, cudaMemcpyHostToDevice) != cudaSuccess ||
                cudaMemcpy(m->d_clw + c.layers * per_o + l * per_d, db.data(), per_d * 2, cudaMemcpyHostToDevice) != cudaSuccess)
                return fail(QW_ERR_CUDA, "cluster weight upload failed");
        }
    }

    // scratch
    const int G = (int)(c.heads / c.kv_heads);
    auto ceil_div = [](uint64_t a, uint64_t b) { return (a + b - 1) / b; };
    // most rows a CTA owns when rows are dealt out in units (the kernel's make_geo): x rows and h
    // values go in units of 8 where the widths allow
    const uint64_t ux = H % 8 == 0 ? 8 : 1, uh = I % 8 == 0 ? 8 : 1, uq = QKVR % 8 == 0 && QKVR / 8 >= (uint64_t)nctas ? 8 : 1;
    auto max_rows = [&](uint64_t rows, uint64_t unit) { return unit * ceil_div(rows / unit, nctas); };
    auto phase_cap = [&](uint64_t rows_per_cta, uint64_t K) { return (uint64_t)seg_count((int)K) * (rows_per_cta + 2); };
    uint64_t pc = std::max({phase_cap(max_rows(QKVR, uq), H), phase_cap(max_rows(H, ux), QD),
                            phase_cap(2 * max_rows(I, uh), H) + 2, phase_cap(max_rows(H, ux), I), phase_cap(ceil_div(c.vocab, nctas), H)});
    // part also stages the attention merge's partials: (S - 1) chunks x G heads x 128
    // and the 12 consumer warps' attention softmax states: NCW x G x ATT_WST
    m->part_cap = (int)align_up(std::max<uint64_t>({pc, (uint64_t)(m->S - 1) * G * HD, (uint64_t)NCW * G * ATT_WST}), 4);
    m->xs_cap = (int)align_up(std::max({H, QD, I}), 4);
    m->xloc_cap = (int)align_up(max_rows(H, ux) + 2, 4);
    m->dyn_smem = (size_t)NSLOT * SLOT_BYTES + ((size_t)m->part_cap + m->xs_cap + m->xloc_cap) * 4;
    if (m->dyn_smem + sizeof(Smem) > (size_t)prop.sharedMemPerBlockOptin)
        return fail(QW_ERR_UNSUPPORTED, "model too large for the kernel's shared-memory plan (vocab or widths)");
    m->generic = !full_segment_shapes((int)H, (int)QD, (int)I);
    for (int t = 0; t < 2; t++) {
        const void* k = kernel_for(t == 1, m->generic);
        if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)m->dyn_smem) != cudaSuccess)
            return fail(QW_ERR_CUDA, "cannot raise the decode kernel's shared-memory limit");
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, NTHREADS, m->dyn_smem) != cudaSuccess || per_sm < 1)
            return fail(QW_ERR_UNSUPPORTED, "decode kernel does not fit on an SM");
    }

    struct Piece { size_t bytes; void** dst; };
    const size_t sz_apart = (size_t)c.kv_heads * m->S * G * APART_STRIDE * 8;
    std::vector<Piece> pieces = {
        {H * 8, (void**)&m->d_x}, {QKVR * 8, (void**)&m->d_qkv}, {QD * 8, (void**)&m->d_att},
        {I * 8, (void**)&m->d_h}, {sz_apart, (void**)&m->d_apart},
        {(size_t)nctas * 4, (void**)&m->d_am_val}, {(size_t)nctas * 4, (void**)&m->d_am_idx}, {16, (void**)&m->d_nan0},
        {(size_t)nctas * 8, (void**)&m->d_flags}, {16, (void**)&m->d_err}, {c.vocab * 4, (void**)&m->d_logits},
        {(size_t)cl::NKV * H * 8, (void**)&m->d_po}, {(size_t)cl::NKV * H * 8, (void**)&m->d_pd}};
    size_t scratch = 0;
    for (auto& pc2 : pieces) scratch += align_up(pc2.bytes, 256);
    if (cudaMalloc(&m->d_scratch, scratch) != cudaSuccess) return fail(QW_ERR_NOMEM, "scratch allocation failed");
    if (cudaMemset(m->d_scratch, 0, scratch) != cudaSuccess) return fail(QW_ERR_CUDA, "scratch memset failed");
    size_t off = 0;
    for (auto& pc2 : pieces) {
        *pc2.dst = m->d_scratch + off;
        off += align_up(pc2.bytes, 256);
    }
    if (cudaHostAlloc(&m->h_stage, 64, cudaHostAllocDefault) != cudaSuccess ||
        cudaHostAlloc(&m->h_logits, c.vocab * 4, cudaHostAllocDefault) != cudaSuccess)
        return fail(QW_ERR_NOMEM, "pinned host allocation failed");
    if (int e = ensure_token_capacity(m, 1024)) { qw_free(m); return e; }
    if (cudaDeviceSynchronize() != cudaSuccess) return fail(QW_ERR_CUDA, "device synchronisation failed after load");
    *out = m;
    return QW_OK;
}

void qw_free(qw_model* m) {
    if (!m) return;
    cudaSetDevice(m->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    cudaFree(m->d_weights);
    cudaFree(m->d_clw);
    cudaFree(m->d_bk);
    cudaFree(m->d_scratch);
    cudaFree(m->d_tok);
    cudaFree(m->d_trace);
    cudaFree(m->pf.X);
    cudaFree(m->pf.Y);
    cudaFree(m->pf.Q);
    cudaFree(m->pf.att);
    cudaFree(m->pf.ahi);
    cudaFree(m->pf.alo);
    cudaFree(m->pf.attp);
    cudaFree(m->pf.att_tickets);
    cudaFree(m->pf.row_ssq);
    for (auto& g : m->graphs) cudaGraphExecDestroy(g.second);
    cudaFree(m->d_rows);
    cudaFree(m->d_btok);
    cudaFree(m->d_am);
    cudaFree(m->d_bout);
    cudaFree(m->d_pf_ids);
    cudaFree(m->d_pf_logits);
    if (m->h_tok) cudaFreeHost(m->h_tok);
    if (m->h_stage) cudaFreeHost(m->h_stage);
    if (m->h_logits) cudaFreeHost(m->h_logits);
    if (m->h_out_stage) cudaFreeHost(m->h_out_stage);
    for (cudaEvent_t e : m->out_ev)
        if (e) cudaEventDestroy(e);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

int qw_config_get(const qw_model* m, qw_config* out) {
    if (!m || !out) return set_err(QW_ERR_ARG, "null argument");
    const ModelConfig& c = m->cfg;
    *out = qw_config{c.hidden, c.inter, c.layers, c.heads, c.kv_heads, c.head_dim, c.vocab, c.eps, c.theta, c.eos};
    return QW_OK;
}

uint64_t qw_weight_bytes_per_token(const qw_model* m) { return m ? m->wbytes : 0; }

int qw_num_ctas(const qw_model* m) { return m ? m->nctas : 0; }

int qw_decoder_kind(const qw_model* m) { return m ? m->kind : -1; }

namespace {
int bk_setup(qw_model* m);  // below, with the batch decode host code
}

int qw_batch_decoder_kind(qw_model* m) {
    if (!m) return -1;
    if (!m->bk_use) return QW_BATCH_ROWS;
    if (cudaSetDevice(m->device) != cudaSuccess || bk_setup(m) != QW_OK) return -1;
    return m->bk_state == 1 ? QW_BATCH_PERSISTENT : QW_BATCH_ROWS;
}

void* qw_model_stream(const qw_model* m) { return m ? static_cast<void*>(m->stream) : nullptr; }

size_t qw_trace_stride(const qw_model* m) { return m ? (size_t)TRACE_PER_LAYER * m->cfg.layers + 4 : 0; }

static size_t trace_words(const qw_model* m) { return (size_t)m->nctas * qw_trace_stride(m); }

int qw_set_trace(qw_model* m, int enable) {
    if (!m) return set_err(QW_ERR_ARG, "null handle");
    QW_CUDA(cudaSetDevice(m->device));
    if (enable && !m->d_trace) {
        const size_t bytes = trace_words(m) * 8;
        if (cudaMalloc(&m->d_trace, bytes) != cudaSuccess) return set_err(QW_ERR_NOMEM, "trace allocation failed");
        QW_CUDA(cudaMemset(m->d_trace, 0, bytes));
    } else if (!enable && m->d_trace) {
        QW_CUDA(cudaStreamSynchronize(m->stream));
        cudaFree(m->d_trace);
        m->d_trace = nullptr;
    }
    return QW_OK;
}

int qw_read_trace(qw_model* m, uint64_t* out, size_t capacity) {
    if (!m || !out) return set_err(QW_ERR_ARG, "null argument");
    if (!m->d_trace) return set_err(QW_ERR_ARG, "tracing is not enabled");
    const size_t n = trace_words(m);
    if (capacity < n) return set_err(QW_ERR_ARG, "trace buffer too small");
    QW_CUDA(cudaSetDevice(m->device));
    QW_CUDA(cudaStreamSynchronize(m->stream));
    QW_CUDA(cudaMemcpy(out, m->d_trace, n * 8, cudaMemcpyDeviceToHost));
    return QW_OK;
}

int qw_cache_new(qw_model* m, size_t max_seq, qw_cache** out) {
    if (!m || !out) return set_err(QW_ERR_ARG, "null argument");
    *out = nullptr;
    if (max_seq == 0 || max_seq > (1u << 30)) return set_err(QW_ERR_ARG, "max_seq out of range");
    QW_CUDA(cudaSetDevice(m->device));
    const ModelConfig& c = m->cfg;
    auto cc = new qw_cache();
    cc->m = m;
    cc->model_id = m->id;
    cc->device = m->device;
    cc->layers = c.layers;
    cc->kv_heads = c.kv_heads;
    cc->head_dim = c.head_dim;
    cc->max_seq = max_seq;
    const size_t kv = c.layers * c.kv_heads * max_seq * c.head_dim * 4;
    const size_t half = c.head_dim / 2;
    if (cudaMalloc(&cc->d_k, kv) != cudaSuccess || cudaMalloc(&cc->d_v, kv) != cudaSuccess ||
        cudaMalloc(&cc->d_rope, max_seq * half * sizeof(float2)) != cudaSuccess) {
        qw_cache_free(cc);
        return set_err(QW_ERR_NOMEM, "KV cache allocation failed");
    }
    cudaMemset(cc->d_k, 0, kv);
    cudaMemset(cc->d_v, 0, kv);
    // RoPE table, same math as the reference's (metal_inference.rs:141-154 == cpu_inference.rs:204-215):
    // freq_i = theta^(-2i/head_dim) in f32, then sin/cos of (pos as f32) * freq_i
    std::vector<float> freqs(half);
    for (size_t i = 0; i < half; i++) freqs[i] = powf(c.theta, -2.0f * (float)i / (float)c.head_dim);
    std::vector<float2> tab(max_seq * half);
    for (size_t pos = 0; pos < max_seq; pos++)
        for (size_t i = 0; i < half; i++) {
            const float a = (float)pos * freqs[i];
            tab[pos * half + i] = make_float2(cosf(a), sinf(a));
        }
    if (cudaMemcpy(cc->d_rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice) != cudaSuccess) {
        qw_cache_free(cc);
        return set_err(QW_ERR_CUDA, "RoPE table upload failed");
    }
    *out = cc;
    return QW_OK;
}

void qw_cache_free(qw_cache* c) {
    if (!c) return;
    cudaSetDevice(c->device);
    cudaFree(c->d_k);  // cudaFree synchronises with work still using the buffers
    cudaFree(c->d_v);
    cudaFree(c->d_rope);
    delete c;
}

size_t qw_cache_max_seq(const qw_cache* c) { return c ? c->max_seq : 0; }

namespace {

// grow the prefill scratch to hold n tokens (and, with logits, n rows of logits)
int ensure_prefill(qw_model* m, size_t n, size_t start, bool logits, size_t row_attp = 0) {
    const ModelConfig& c = m->cfg;
    const size_t H = c.hidden, I = c.inter, QD = c.heads * c.head_dim;
    if ((int)n > m->pf.cap) {
        const size_t cap = std::max<size_t>(n, 2 * (size_t)m->pf.cap);
        qw::pf::Scratch sc;
        const size_t acols = std::max({H, QD, I});
        bool ok = cudaMalloc(&sc.X, cap * H * 4) == cudaSuccess &&
                  cudaMalloc(&sc.Q, cap * QD * 4) == cudaSuccess && cudaMalloc(&sc.att, cap * QD * 4) == cudaSuccess &&
                  cudaMalloc(&sc.ahi, cap * acols * 2) == cudaSuccess && cudaMalloc(&sc.alo, cap * acols * 2) == cudaSuccess;
        uint32_t* ids = nullptr;
        ok = ok && cudaMalloc(&ids, cap * 4) == cudaSuccess;
        if (!ok) {
            cudaFree(sc.X); cudaFree(sc.Q); cudaFree(sc.att); cudaFree(sc.ahi); cudaFree(sc.alo); cudaFree(ids);
            return set_err(QW_ERR_NOMEM, "prefill scratch allocation failed");
        }
        cudaFree(m->pf.X); cudaFree(m->pf.Q); cudaFree(m->pf.att); cudaFree(m->pf.ahi); cudaFree(m->pf.alo);
        cudaFree(m->d_pf_ids);
        sc.cap = (int)cap;
        sc.Y = m->pf.Y;
        sc.ycap = m->pf.ycap;
        sc.attp = m->pf.attp;
        sc.attp_cap = m->pf.attp_cap;
        sc.att_tickets = m->pf.att_tickets;
        sc.row_ssq = m->pf.row_ssq;
        m->pf = sc;
        m->d_pf_ids = ids;
    }
    const size_t ycap = qw::pf::y_floats((int)n, (int)H, (int)I, (int)c.heads, (int)c.kv_heads);
    if (ycap > m->pf.ycap) {
        float* d = nullptr;
        const size_t cap = std::max(ycap, 2 * m->pf.ycap);
        if (cudaMalloc(&d, cap * 4) != cudaSuccess) return set_err(QW_ERR_NOMEM, "prefill GEMM scratch allocation failed");
        cudaFree(m->pf.Y);
        m->pf.Y = d;
        m->pf.ycap = cap;
    }
    const size_t attp = std::max(qw::pf::attention_partial_floats((int)n, (int)start, (int)c.heads, (int)c.kv_heads),
                                 row_attp);
    if (attp > m->pf.attp_cap) {
        float* d = nullptr;
        const size_t cap = std::max(attp, 2 * m->pf.attp_cap);
        if (cudaMalloc(&d, cap * 4) != cudaSuccess) return set_err(QW_ERR_NOMEM, "prefill attention scratch allocation failed");
        cudaFree(m->pf.attp);
        m->pf.attp = d;
        m->pf.attp_cap = cap;
    }
    if (logits && n > m->pf_logits_cap) {
        float* d = nullptr;
        if (cudaMalloc(&d, n * c.vocab * 4) != cudaSuccess) return set_err(QW_ERR_NOMEM, "prefill logits allocation failed");
        cudaFree(m->d_pf_logits);
        m->d_pf_logits = d;
        m->pf_logits_cap = n;
    }
    return QW_OK;
}

}  // namespace

namespace {

// Device -> caller host memory for large results (the prefill's per-position logits, 311 MB for
// 512 positions of a 151,936-token vocabulary), enqueued on the model's stream after the work that
// produces them; returns once the data is in `dst`. A page-locked (or managed) destination takes
// one DMA; device memory is refused (QW_ERR_ARG). A pageable one goes through two pinned stages of OUT_STAGE bytes: the DMA into one stage runs
// while host threads copy the other out to the caller's pages, and those threads also take the
// page faults of freshly allocated memory in parallel. (One pageable cudaMemcpy of 311 MB measured
// 18 ms into memory touched before and 65 ms into fresh pages on the B200 hosts, against 6 ms for
// the DMA alone.)
constexpr size_t OUT_STAGE = 16u << 20;

int copy_to_host(qw_model* m, void* dst, const void* src, size_t bytes) {
    cudaPointerAttributes at{};
    const cudaError_t pe = cudaPointerGetAttributes(&at, dst);
    if (pe != cudaSuccess) cudaGetLastError();  // not known to CUDA: treated as pageable
    if (pe == cudaSuccess && at.type == cudaMemoryTypeDevice) return set_err(QW_ERR_ARG, "copy-out to device memory");
    const bool direct = pe == cudaSuccess && (at.type == cudaMemoryTypeHost || at.type == cudaMemoryTypeManaged);
    if (direct || bytes < 2 * OUT_STAGE) {
        QW_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, m->stream));
        QW_CUDA(cudaStreamSynchronize(m->stream));
        return QW_OK;
    }
    if (!m->h_out_stage) {
        if (cudaHostAlloc(&m->h_out_stage, 2 * OUT_STAGE, cudaHostAllocDefault) != cudaSuccess) {
            m->h_out_stage = nullptr;
            return set_err(QW_ERR_NOMEM, "pinned staging allocation failed");
        }
    }
    for (cudaEvent_t& e : m->out_ev)
        if (!e) QW_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    const size_t nch = (bytes + OUT_STAGE - 1) / OUT_STAGE;
    auto chunk_len = [&](size_t k) { return std::min(OUT_STAGE, bytes - k * OUT_STAGE); };
    auto enqueue = [&](size_t k) -> int {
        uint8_t* st = m->h_out_stage + (k & 1) * OUT_STAGE;
        QW_CUDA(cudaMemcpyAsync(st, static_cast<const uint8_t*>(src) + k * OUT_STAGE, chunk_len(k), cudaMemcpyDeviceToHost,
                                m->stream));
        QW_CUDA(cudaEventRecord(m->out_ev[k & 1], m->stream));
        return QW_OK;
    };
    // host threads: the caller's plus helpers, each copying one slice of every chunk
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    const int nthr = (int)std::min(8u, std::max(1u, hw / 2));
    std::atomic<long long> ready{-1};  // chunk whose stage may be copied out
    std::atomic<int> finished{0};      // helper slices of that chunk copied
    std::atomic<bool> quit{false};
    auto copy_slice = [&](size_t k, int t) {
        const size_t len = chunk_len(k), a = len * t / nthr, b = len * (t + 1) / nthr;
        std::memcpy(static_cast<uint8_t*>(dst) + k * OUT_STAGE + a, m->h_out_stage + (k & 1) * OUT_STAGE + a, b - a);
    };
    std::vector<std::thread> helpers;
    try {
        for (int t = 1; t < nthr; t++)
            helpers.emplace_back([&, t] {
                for (size_t k = 0; k < nch; k++) {
                    while (ready.load(std::memory_order_acquire) < (long long)k) {
                        if (quit.load(std::memory_order_relaxed)) return;
                        std::this_thread::yield();
                    }
                    copy_slice(k, t);
                    finished.fetch_add(1, std::memory_order_acq_rel);
                }
            });
    } catch (...) {  // no threads to be had: stop those started, then one pageable copy
        quit.store(true);
        for (auto& h : helpers) h.join();
        QW_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, m->stream));
        QW_CUDA(cudaStreamSynchronize(m->stream));
        return QW_OK;
    }
    int rc = QW_OK;
    for (size_t k = 0; k < std::min<size_t>(2, nch) && rc == QW_OK; k++) rc = enqueue(k);
    for (size_t k = 0; k < nch && rc == QW_OK; k++) {
        if (cudaEventSynchronize(m->out_ev[k & 1]) != cudaSuccess) {
            rc = set_err(QW_ERR_CUDA, std::string("copy-out: ") + cudaGetErrorString(cudaGetLastError()));
            break;
        }
        finished.store(0, std::memory_order_relaxed);
        ready.store((long long)k, std::memory_order_release);
        copy_slice(k, 0);
        while (finished.load(std::memory_order_acquire) < nthr - 1) std::this_thread::yield();
        if (k + 2 < nch) rc = enqueue(k + 2);
    }
    quit.store(true);
    for (auto& h : helpers) h.join();
    return rc;
}

}  // namespace

int qw_prefill(qw_model* m, qw_cache* c, const uint32_t* ids, size_t n, size_t start_pos, float* logits_out) {
    if (!m || !c || !ids || c->m != m || c->model_id != m->id) return set_err(QW_ERR_ARG, "null or mismatched handle");
    if (n == 0) return QW_OK;
    if (n > (1u << 20) || start_pos + n > c->max_seq) return set_err(QW_ERR_ARG, "start_pos + n exceeds the KV cache size");
    for (size_t i = 0; i < n; i++)
        if (ids[i] >= m->cfg.vocab) return set_err(QW_ERR_ARG, "token id >= vocab_size");
    QW_CUDA(cudaSetDevice(m->device));
    if (logits_out) {  // host memory only (the _device call takes device buffers); refused before any work
        cudaPointerAttributes at{};
        const cudaError_t pe = cudaPointerGetAttributes(&at, logits_out);
        if (pe != cudaSuccess) cudaGetLastError();
        else if (at.type == cudaMemoryTypeDevice)
            return set_err(QW_ERR_ARG, "logits_out is device memory: qw_prefill writes host memory (qw_prefill_device takes device buffers)");
    }
    if (int e = ensure_prefill(m, n, start_pos, logits_out != nullptr)) return e;
    int* ew = qw::device_err_word_for(m->device);
    if (!ew) return set_err(QW_ERR_NOMEM, "error word allocation failed");
    QW_CUDA(cudaMemsetAsync(ew, 0, 2 * sizeof(int), m->stream));
    QW_CUDA(cudaMemcpyAsync(m->d_pf_ids, ids, n * 4, cudaMemcpyHostToDevice, m->stream));
    const ModelConfig& cf = m->cfg;
    qw::pf::Weights w{m->d_layer_w, m->d_layer_n, m->d_final_norm, m->d_embed, m->d_lm_head, m->layer_stride, m->norm_stride,
                      (int)cf.hidden, (int)cf.inter, (int)cf.layers, (int)cf.heads, (int)cf.kv_heads, (int)cf.vocab, cf.eps};
    qw::pf::CacheView cv{c->d_k, c->d_v, c->d_rope, (int)c->max_seq};
    std::string err;
    if (int e = qw::pf::run(w, cv, m->d_pf_ids, (int)n, (int)start_pos, logits_out ? m->d_pf_logits : nullptr, m->pf, ew,
                            m->stream, err))
        return set_err(e, err);
    int h[2] = {0, 0};
    QW_CUDA(cudaMemcpyAsync(h, ew, sizeof h, cudaMemcpyDeviceToHost, m->stream));
    if (logits_out) {
        if (int e = copy_to_host(m, logits_out, m->d_pf_logits, n * cf.vocab * 4)) return e;
    }
    QW_CUDA(cudaStreamSynchronize(m->stream));
    if (h[0]) return set_err(QW_ERR_DEVICE_TIMEOUT, "prefill: a GEMM pipeline wait expired on the device");
    return QW_OK;
}

int qw_prefill_device(qw_model* m, qw_cache* c, const uint32_t* d_ids, size_t n, size_t start_pos, float* d_logits,
                      void* stream) {
    if (!m || !c || !d_ids || c->m != m || c->model_id != m->id) return set_err(QW_ERR_ARG, "null or mismatched handle");
    if (n == 0) return QW_OK;
    if (n > (1u << 20) || start_pos + n > c->max_seq) return set_err(QW_ERR_ARG, "start_pos + n exceeds the KV cache size");
    QW_CUDA(cudaSetDevice(m->device));
    if (int e = ensure_prefill(m, n, start_pos, false)) return e;
    int* ew = qw::device_err_word_for(m->device);
    if (!ew) return set_err(QW_ERR_NOMEM, "error word allocation failed");
    cudaStream_t s = pick_stream(m, stream);
    QW_CUDA(cudaMemsetAsync(ew, 0, 2 * sizeof(int), s));
    const ModelConfig& cf = m->cfg;
    qw::pf::Weights w{m->d_layer_w, m->d_layer_n, m->d_final_norm, m->d_embed, m->d_lm_head, m->layer_stride, m->norm_stride,
                      (int)cf.hidden, (int)cf.inter, (int)cf.layers, (int)cf.heads, (int)cf.kv_heads, (int)cf.vocab, cf.eps};
    qw::pf::CacheView cv{c->d_k, c->d_v, c->d_rope, (int)c->max_seq};
    std::string err;
    if (int e = qw::pf::run(w, cv, d_ids, (int)n, (int)start_pos, d_logits, m->pf, ew, s, err)) return set_err(e, err);
    return QW_OK;
}

namespace {

// Row views of a batch over `caches` (distinct, all of model m) with rows at pos[b], each
// running `steps` steps from there.
int batch_rows(qw_model* m, qw_cache* const* caches, size_t B, const size_t* pos, size_t steps,
               std::vector<qw::pf::RowView>& rows, int& splits) {
    if (!caches || !pos || B == 0 || B > (size_t)qw::pf::ROWS_MAX)
        return set_err(QW_ERR_ARG, "batch: 1 <= rows <= 16 caches and positions required");
    rows.resize(B);
    size_t last = 0;
    for (size_t b = 0; b < B; b++) {
        const qw_cache* c = caches[b];
        if (!c || c->m != m || c->model_id != m->id) return set_err(QW_ERR_ARG, "batch: null or mismatched cache");
        for (size_t j = 0; j < b; j++)
            if (caches[j] == c) return set_err(QW_ERR_ARG, "batch: a cache appears twice");
        if (pos[b] + steps > c->max_seq) return set_err(QW_ERR_ARG, "batch: position + steps exceeds the KV cache size");
        rows[b] = qw::pf::RowView{c->d_k, c->d_v, c->d_rope, (int)c->max_seq, (int)pos[b], (int)pos[b], 0};
        last = std::max(last, pos[b] + steps - 1);
    }
    splits = (int)(last / qw::pf::ROW_SPLIT + 1);
    return QW_OK;
}

int ensure_batch(qw_model* m, size_t B, int splits, size_t out_entries) {
    if (!m->d_rows) QW_CUDA(cudaMalloc(&m->d_rows, qw::pf::ROWS_MAX * sizeof(qw::pf::RowView)));
    if (!m->d_btok) QW_CUDA(cudaMalloc(&m->d_btok, qw::pf::ROWS_MAX * 4));
    if (!m->d_am) {
        QW_CUDA(cudaMalloc(&m->d_am, sizeof(qw::pf::ArgmaxScratch)));
        QW_CUDA(cudaMemset(m->d_am, 0, sizeof(qw::pf::ArgmaxScratch)));
    }
    if (!m->pf.att_tickets) {
        const size_t nb = (size_t)qw::pf::ROWS_MAX * m->cfg.kv_heads * 4;
        QW_CUDA(cudaMalloc(&m->pf.att_tickets, nb));
        QW_CUDA(cudaMemset(m->pf.att_tickets, 0, nb));
    }
    if (!m->pf.row_ssq) QW_CUDA(cudaMalloc(&m->pf.row_ssq, 2 * (size_t)qw::pf::ROWS_MAX * qw::pf::NORM_BLOCKS_MAX * 4));
    if (out_entries > m->bout_cap) {
        uint32_t* d = nullptr;
        const size_t cap = std::max(out_entries, 2 * m->bout_cap);
        if (cudaMalloc(&d, cap * 4) != cudaSuccess) return set_err(QW_ERR_NOMEM, "batch token record allocation failed");
        cudaFree(m->d_bout);
        m->d_bout = d;
        m->bout_cap = cap;
    }
    return ensure_prefill(m, B, 0, true, qw::pf::row_partial_floats((int)B, (int)m->cfg.heads, splits));
}

qw::pf::Weights weights_of(const qw_model* m) {
    const ModelConfig& cf = m->cfg;
    return qw::pf::Weights{m->d_layer_w, m->d_layer_n, m->d_final_norm, m->d_embed, m->d_lm_head, m->layer_stride,
                           m->norm_stride, (int)cf.hidden, (int)cf.inter, (int)cf.layers, (int)cf.heads,
                           (int)cf.kv_heads, (int)cf.vocab, cf.eps};
}

// The graph of one row-mode step over B rows, captured on the model's stream the first time a
// configuration is used and replayed after: kind 0 = greedy batch step (forward + argmax_rows,
// tokens recorded into `out`, rows advanced); kind 1 = lookup verify pass (forward + argmax_each
// into `out`).
int row_graph(qw_model* m, int kind, int B, int splits, uint32_t* out, int* ew, cudaGraphExec_t& exec) {
    const qw_model::GraphKey key{kind, B, splits, m->pf.X, m->pf.Y, m->pf.attp, m->d_pf_logits, out};
    for (auto& g : m->graphs)
        if (g.first == key) {
            exec = g.second;
            return QW_OK;
        }
    if (m->graphs.size() >= 32) {  // buffers moved or many shapes: start over
        for (auto& g : m->graphs) cudaGraphExecDestroy(g.second);
        m->graphs.clear();
    }
    cudaStream_t s = m->stream;
    QW_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    std::string err;
    // kind 0 rows are distinct caches (batch_rows refuses a cache twice); a lookup pass's rows share one
    int rc = qw::pf::run_rows(weights_of(m), m->d_rows, B, splits, kind == 0, m->d_btok, m->d_pf_logits, m->pf, ew, s, err);
    if (!rc)
        rc = kind == 0 ? qw::pf::argmax_rows(m->d_pf_logits, (int)m->cfg.vocab, B, m->d_rows, m->d_btok, out, m->d_am, s, err)
                       : qw::pf::argmax_each(m->d_pf_logits, (int)m->cfg.vocab, B, out, m->d_am, s, err);
    cudaGraph_t graph = nullptr;
    const cudaError_t ce = cudaStreamEndCapture(s, &graph);
    if (rc) {
        if (graph) cudaGraphDestroy(graph);
        return set_err(rc, err);
    }
    if (ce != cudaSuccess) return cuda_err(ce, "cudaStreamEndCapture (row step)");
    const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ie != cudaSuccess) return cuda_err(ie, "cudaGraphInstantiate (row step)");
    m->graphs.emplace_back(key, exec);
    return QW_OK;
}

// The persistent batch kernel (batch_kernel.cuh), set up on first use: the shapes it covers, its
// shared-memory plan on this GPU, and its scratch. bk_state ends 1 (usable) or -1.
int bk_setup(qw_model* m) {
    if (m->bk_state != 0) return QW_OK;
    m->bk_state = -1;
    const ModelConfig& c = m->cfg;
    const uint64_t H = c.hidden, I = c.inter, QD = c.heads * c.head_dim, KVD = c.kv_heads * c.head_dim;
    const uint64_t QKVR = QD + 2 * KVD;
    const int nctas = m->nctas;
    if (m->kind != QW_DECODER_GRID || c.head_dim != 128 || H != (uint64_t)bk::KBLK || QD % bk::KBLK || I % bk::KBLK ||
        c.heads % c.kv_heads || c.heads / c.kv_heads > (uint64_t)bk::MAX_G)
        return QW_OK;
    auto ceil_div = [](uint64_t a, uint64_t b) { return (a + b - 1) / b; };
    auto max_rows = [&](uint64_t rows, uint64_t unit) { return unit * ceil_div(rows / unit, nctas); };
    const uint64_t uq = QKVR % 8 == 0 && QKVR / 8 >= (uint64_t)nctas ? 8 : 1;
    auto fits = [&](uint64_t rows, uint64_t K) {
        const uint64_t rpp = bk::SLOT_BYTES / (2 * K);
        return rows <= (uint64_t)bk::MAX_ROWS && rpp >= 1 && ceil_div(rows, rpp) <= (uint64_t)bk::NSLOT;
    };
    if (!fits(max_rows(QKVR, uq), H) || !fits(max_rows(H, 8), QD) || !fits(2 * max_rows(I, 8), H) || !fits(max_rows(H, 8), I))
        return QW_OK;
    if (cudaFuncSetAttribute(bk::batch_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bk::DYN_BYTES) !=
        cudaSuccess) {
        (void)cudaGetLastError();
        return QW_OK;
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, bk::batch_decode_kernel, bk::NTHREADS, bk::DYN_BYTES) !=
            cudaSuccess || per_sm < 1) {
        (void)cudaGetLastError();
        return QW_OK;
    }
    const size_t G = c.heads / c.kv_heads;
    const size_t nb = bk::NB;
    const size_t tagged = (nb * H + nb * QKVR + nb * I + nb * QD + nb * c.kv_heads * bk::MAX_S * G * bk::APART) * 8;
    const size_t rest = (size_t)nctas * nb * 8 + 64 + (size_t)nctas * 8;
    if (cudaMalloc(&m->d_bk, tagged + rest) != cudaSuccess) return set_err(QW_ERR_NOMEM, "batch kernel scratch allocation failed");
    QW_CUDA(cudaMemset(m->d_bk, 0, tagged + rest));
    u64* t = reinterpret_cast<u64*>(m->d_bk);
    m->bk_x = t;
    m->bk_qkv = m->bk_x + nb * H;
    m->bk_h = m->bk_qkv + nb * QKVR;
    m->bk_att = m->bk_h + nb * I;
    m->bk_apart = m->bk_att + nb * QD;
    m->bk_tagged_bytes = tagged;
    uint8_t* r = m->d_bk + tagged;
    m->bk_am_val = reinterpret_cast<float*>(r);
    m->bk_am_idx = reinterpret_cast<unsigned*>(r + (size_t)nctas * nb * 4);
    m->bk_nan0 = reinterpret_cast<int*>(r + (size_t)nctas * nb * 8);
    m->bk_flags = reinterpret_cast<u64*>(r + (size_t)nctas * nb * 8 + 64);
    m->bk_state = 1;
    return QW_OK;
}

// one launch of the persistent batch kernel over `rows` (validated by batch_rows), first tokens in
// m->d_btok, tokens recorded into m->d_bout [steps][B]
int bk_launch(qw_model* m, qw_cache* const* caches, size_t B, const size_t* start_pos, size_t steps, cudaStream_t s) {
    const ModelConfig& g = m->cfg;
    bk::BParams p{};
    p.layer_w = m->d_layer_w;
    p.layer_n = m->d_layer_n;
    p.final_norm = m->d_final_norm;
    p.embed = m->d_embed;
    p.lm_head = m->d_lm_head;
    for (size_t b = 0; b < B; b++) {
        p.kc[b] = caches[b]->d_k;
        p.vc[b] = caches[b]->d_v;
        p.rope[b] = caches[b]->d_rope;
        p.max_seq[b] = (int)caches[b]->max_seq;
        p.pos0[b] = (int)start_pos[b];
    }
    p.x = m->bk_x;
    p.qkv = m->bk_qkv;
    p.hbuf = m->bk_h;
    p.att = m->bk_att;
    p.apart = m->bk_apart;
    p.am_val = m->bk_am_val;
    p.am_idx = m->bk_am_idx;
    p.nan0 = m->bk_nan0;
    p.flags = m->bk_flags;
    p.err = m->d_err;
    p.tok_in = m->d_btok;
    p.tok_out = m->d_bout;
    p.layer_stride = m->layer_stride;
    p.norm_stride = m->norm_stride;
    p.H = (int)g.hidden;
    p.I = (int)g.inter;
    p.L = (int)g.layers;
    p.NQ = (int)g.heads;
    p.NKV = (int)g.kv_heads;
    p.V = (int)g.vocab;
    p.nb = (int)B;
    p.steps = (int)steps;
    const unsigned e = ++m->bk_epoch;
    if ((e & 0xFFFu) == 0) QW_CUDA(cudaMemsetAsync(m->d_bk, 0, m->bk_tagged_bytes, s));  // tags would repeat
    p.epoch = e;
    p.eps = g.eps;
    p.scale = 1.0f / sqrtf((float)g.head_dim);  // cpu_inference.rs:144
    p.S = std::max(1, std::min(bk::MAX_S, m->nctas / (int)(B * g.kv_heads)));
    p.min_chunk = m->min_chunk;
    p.timeout_ns = m->timeout_ns;
    p.trace = m->d_trace;  // the decode kernel's timeline buffer and layout, when tracing is on
    p.stall_cta = m->stall_cta;
    m->stall_cta = -1;
    void* args[] = {&p};
    const cudaError_t ce = cudaLaunchCooperativeKernel((const void*)bk::batch_decode_kernel, dim3(m->nctas), dim3(bk::NTHREADS),
                                                       args, bk::DYN_BYTES, s);
    if (ce != cudaSuccess) return cuda_err(ce, "batch decode kernel launch");
    return QW_OK;
}

// stream-ordered batch decode: rows from host positions, first tokens already in m->d_btok; the
// step graph records tokens into m->d_bout ([steps][B]), so one capture serves every batch of the
// same shape
int batch_decode_launch(qw_model* m, qw_cache* const* caches, size_t B, const size_t* start_pos, size_t steps,
                        cudaStream_t s) {
    std::vector<qw::pf::RowView> rows;
    int splits = 0;
    if (int e = batch_rows(m, caches, B, start_pos, steps, rows, splits)) return e;
    if (int e = ensure_batch(m, B, splits, steps * B)) return e;
    if (m->bk_use && B <= (size_t)bk::NB) {
        if (int e = bk_setup(m)) return e;
        if (m->bk_state == 1) return bk_launch(m, caches, B, start_pos, steps, s);
    }
    int* ew = qw::device_err_word_for(m->device);
    if (!ew) return set_err(QW_ERR_NOMEM, "error word allocation failed");
    cudaGraphExec_t g = nullptr;
    if (int e = row_graph(m, 0, (int)B, splits, m->d_bout, ew, g)) return e;
    QW_CUDA(cudaMemsetAsync(ew, 0, 2 * sizeof(int), s));
    QW_CUDA(cudaMemcpyAsync(m->d_rows, rows.data(), B * sizeof(qw::pf::RowView), cudaMemcpyHostToDevice, s));
    for (size_t i = 0; i < steps; i++) QW_CUDA(cudaGraphLaunch(g, s));
    return QW_OK;
}

}  // namespace

int qw_forward_batch(qw_model* m, qw_cache* const* caches, size_t B, const uint32_t* tokens, const size_t* positions,
                     float* logits_out) {
    if (!m || !tokens || !logits_out) return set_err(QW_ERR_ARG, "null argument");
    for (size_t b = 0; b < B && b < (size_t)qw::pf::ROWS_MAX; b++)
        if (tokens[b] >= m->cfg.vocab) return set_err(QW_ERR_ARG, "token id >= vocab_size");
    QW_CUDA(cudaSetDevice(m->device));
    std::vector<qw::pf::RowView> rows;
    int splits = 0;
    if (int e = batch_rows(m, caches, B, positions, 1, rows, splits)) return e;
    if (int e = ensure_batch(m, B, splits, 0)) return e;
    int* ew = qw::device_err_word_for(m->device);
    if (!ew) return set_err(QW_ERR_NOMEM, "error word allocation failed");
    cudaStream_t s = m->stream;
    QW_CUDA(cudaMemsetAsync(ew, 0, 2 * sizeof(int), s));
    QW_CUDA(cudaMemcpyAsync(m->d_rows, rows.data(), B * sizeof(qw::pf::RowView), cudaMemcpyHostToDevice, s));
    QW_CUDA(cudaMemcpyAsync(m->d_btok, tokens, B * 4, cudaMemcpyHostToDevice, s));
    std::string err;
    if (int e = qw::pf::run_rows(weights_of(m), m->d_rows, (int)B, splits, true, m->d_btok, m->d_pf_logits, m->pf, ew, s, err))
        return set_err(e, err);
    QW_CUDA(cudaMemcpyAsync(logits_out, m->d_pf_logits, B * m->cfg.vocab * 4, cudaMemcpyDeviceToHost, s));
    int h = 0;
    QW_CUDA(cudaMemcpyAsync(&h, ew, sizeof(int), cudaMemcpyDeviceToHost, s));
    QW_CUDA(cudaStreamSynchronize(s));
    if (h) return set_err(QW_ERR_DEVICE_TIMEOUT, "forward_batch: a GEMM pipeline wait expired on the device");
    return QW_OK;
}

int qw_decode_batch(qw_model* m, qw_cache* const* caches, size_t B, const uint32_t* firsts, const size_t* start_pos,
                    size_t steps, uint32_t* tokens_out) {
    if (!m || !firsts || !tokens_out) return set_err(QW_ERR_ARG, "null argument");
    if (steps == 0) return QW_OK;
    for (size_t b = 0; b < B && b < (size_t)qw::pf::ROWS_MAX; b++)
        if (firsts[b] >= m->cfg.vocab) return set_err(QW_ERR_ARG, "token id >= vocab_size");
    QW_CUDA(cudaSetDevice(m->device));
    cudaStream_t s = m->stream;
    if (B >= 1 && B <= (size_t)qw::pf::ROWS_MAX && !m->d_btok) QW_CUDA(cudaMalloc(&m->d_btok, qw::pf::ROWS_MAX * 4));
    if (m->d_btok && B >= 1 && B <= (size_t)qw::pf::ROWS_MAX)
        QW_CUDA(cudaMemcpyAsync(m->d_btok, firsts, B * 4, cudaMemcpyHostToDevice, s));
    if (int e = batch_decode_launch(m, caches, B, start_pos, steps, s)) return e;
    std::vector<uint32_t> rec(steps * B);
    QW_CUDA(cudaMemcpyAsync(rec.data(), m->d_bout, steps * B * 4, cudaMemcpyDeviceToHost, s));
    int h = 0;
    int* ew = qw::device_err_word_for(m->device);
    QW_CUDA(cudaMemcpyAsync(&h, ew, sizeof(int), cudaMemcpyDeviceToHost, s));
    QW_CUDA(cudaStreamSynchronize(s));
    if (h) return set_err(QW_ERR_DEVICE_TIMEOUT, "decode_batch: a GEMM pipeline wait expired on the device");
    if (int e = check_device_err(m)) return e;  // the persistent batch kernel's error word
    for (size_t b = 0; b < B; b++)
        for (size_t i = 0; i < steps; i++) tokens_out[b * steps + i] = rec[i * B + b];
    return QW_OK;
}

int qw_decode_batch_device(qw_model* m, qw_cache* const* caches, size_t B, const uint32_t* d_firsts,
                           const size_t* start_pos, size_t steps, uint32_t* d_out, void* stream) {
    if (!m || !d_firsts || !d_out) return set_err(QW_ERR_ARG, "null argument");
    if (steps == 0) return QW_OK;
    QW_CUDA(cudaSetDevice(m->device));
    cudaStream_t s = pick_stream(m, stream);
    if (!m->d_btok) QW_CUDA(cudaMalloc(&m->d_btok, qw::pf::ROWS_MAX * 4));
    if (B >= 1 && B <= (size_t)qw::pf::ROWS_MAX)
        QW_CUDA(cudaMemcpyAsync(m->d_btok, d_firsts, B * 4, cudaMemcpyDeviceToDevice, s));
    if (int e = batch_decode_launch(m, caches, B, start_pos, steps, s)) return e;
    QW_CUDA(cudaMemcpyAsync(d_out, m->d_bout, steps * B * 4, cudaMemcpyDeviceToDevice, s));
    return QW_OK;
}

namespace {

// Prompt lookup (the draft source of the reference's proposed speculation, README.md:109-111): the
// longest n-gram, max_ngram down to 1 tokens, that ends the history and also occurs earlier; the
// k tokens that followed its most recent earlier occurrence are the draft. Where that continuation
// runs into the present (the occurrence overlaps the end of the history, as in a repeated token
// or phrase), it continues from the draft itself, like an overlapping copy: the text is assumed to
// keep repeating with the same period.
size_t lookup_draft(const std::vector<uint32_t>& h, size_t max_ngram, size_t k, std::vector<uint32_t>& draft) {
    draft.clear();
    const size_t L = h.size();
    if (L < 2 || k == 0) return 0;
    for (size_t n = std::min(max_ngram, L - 1); n >= 1; n--) {
        for (size_t i = L - n; i-- > 0;) {  // occurrences starting at i, latest first, each followed by a token
            if (std::equal(h.begin() + (long)i, h.begin() + (long)(i + n), h.end() - (long)n)) {
                for (size_t j = 0; j < k; j++) {
                    const size_t q = i + n + j;
                    draft.push_back(q < L ? h[q] : draft[q - L]);
                }
                return k;
            }
        }
    }
    return 0;
}

// drafts shorter than this are not worth a verify pass (a pass over the weights for B rows costs
// about two single-token decode steps); the token goes through the decode kernel instead
constexpr size_t LOOKUP_MIN_DRAFT = 2;

}  // namespace

int qw_decode_lookup(qw_model* m, qw_cache* c, const uint32_t* context, size_t context_len, uint32_t first,
                     size_t start_pos, size_t steps, uint32_t max_ngram, uint32_t draft_max, uint32_t* tokens_out,
                     qw_lookup_stats* stats) {
    if (!m || !c || c->m != m || c->model_id != m->id || (!context && context_len)) return set_err(QW_ERR_ARG, "null or mismatched handle");
    if (stats) *stats = qw_lookup_stats{0, 0, 0};
    if (steps == 0) return QW_OK;
    if (!tokens_out) return set_err(QW_ERR_ARG, "null tokens_out");
    if (max_ngram < 1 || draft_max < 1 || draft_max > QW_LOOKUP_DRAFT_MAX)
        return set_err(QW_ERR_ARG, "lookup: max_ngram >= 1 and 1 <= draft_max <= QW_LOOKUP_DRAFT_MAX");
    if (start_pos + steps > c->max_seq) return set_err(QW_ERR_ARG, "start_pos + steps exceeds the KV cache size");
    if (first >= m->cfg.vocab) return set_err(QW_ERR_ARG, "token id >= vocab_size");
    QW_CUDA(cudaSetDevice(m->device));
    if (int e = ensure_token_capacity(m, 2)) return e;
    // verify passes run in row mode (row t = the pass's t-th token at pos + t of this one cache),
    // as captured graphs; their attention splits cover the last position a pass can reach
    const int splits = (int)((start_pos + steps - 1) / qw::pf::ROW_SPLIT + 1);
    if (int e = ensure_batch(m, draft_max + 1, splits, 0)) return e;
    int* ew = qw::device_err_word_for(m->device);
    if (!ew) return set_err(QW_ERR_NOMEM, "error word allocation failed");
    cudaStream_t s = m->stream;
    QW_CUDA(cudaMemsetAsync(ew, 0, 2 * sizeof(int), s));
    std::vector<qw::pf::RowView> rows;
    std::vector<uint32_t> hist(context, context + context_len);
    hist.push_back(first);
    std::vector<uint32_t> draft, ids, got(draft_max + 1);
    uint32_t cur = first;
    size_t pos = start_pos, emitted = 0;
    qw_lookup_stats st{0, 0, 0};
    while (emitted < steps) {
        const size_t remaining = steps - emitted;
        lookup_draft(hist, max_ngram, std::min<size_t>(draft_max, remaining - 1), draft);
        size_t take;
        if (draft.size() < LOOKUP_MIN_DRAFT) {
            // no draft: one token through the persistent decode kernel
            m->h_stage[0] = cur;
            QW_CUDA(cudaMemcpyAsync(m->d_tok, m->h_stage, 4, cudaMemcpyHostToDevice, s));
            if (int e = launch_decode(m, c, m->d_tok, m->d_tok, false, nullptr, pos, 1, s)) return e;
            QW_CUDA(cudaMemcpyAsync(got.data(), m->d_tok + 1, 4, cudaMemcpyDeviceToHost, s));
            QW_CUDA(cudaStreamSynchronize(s));
            if (int e = check_device_err(m)) return e;
            take = 1;
        } else {
            // verify pass: cur and the drafts at pos .. pos + len in one multi-token forward
            ids.assign(1, cur);
            ids.insert(ids.end(), draft.begin(), draft.end());
            const size_t n = ids.size();
            rows.resize(n);
            for (size_t t = 0; t < n; t++)
                rows[t] = qw::pf::RowView{c->d_k, c->d_v, c->d_rope, (int)c->max_seq, (int)(pos + t), (int)(pos + t), 0};
            cudaGraphExec_t g = nullptr;
            if (int e = row_graph(m, 1, (int)n, splits, m->d_pf_ids, ew, g)) return e;
            QW_CUDA(cudaMemcpyAsync(m->d_rows, rows.data(), n * sizeof(qw::pf::RowView), cudaMemcpyHostToDevice, s));
            QW_CUDA(cudaMemcpyAsync(m->d_btok, ids.data(), n * 4, cudaMemcpyHostToDevice, s));
            QW_CUDA(cudaGraphLaunch(g, s));
            QW_CUDA(cudaMemcpyAsync(got.data(), m->d_pf_ids, n * 4, cudaMemcpyDeviceToHost, s));
            int h = 0;
            QW_CUDA(cudaMemcpyAsync(&h, ew, sizeof(int), cudaMemcpyDeviceToHost, s));
            QW_CUDA(cudaStreamSynchronize(s));
            if (h) return set_err(QW_ERR_DEVICE_TIMEOUT, "lookup verify pass: a GEMM pipeline wait expired on the device");
            // got[i] is the greedy token after ids[0..i]; draft i is right while it equals got[i]
            size_t a = 0;
            while (a < draft.size() && draft[a] == got[a]) a++;
            take = a + 1;
            st.drafted += draft.size();
            st.accepted += a;
        }
        st.passes++;
        for (size_t i = 0; i < take; i++) {
            tokens_out[emitted + i] = got[i];
            hist.push_back(got[i]);
        }
        emitted += take;
        pos += take;
        cur = got[take - 1];
    }
    if (stats) *stats = st;
    return QW_OK;
}

int qw_forward(qw_model* m, qw_cache* c, uint32_t token, size_t pos, float* logits_out) {
    if (!m || !c || !logits_out || c->m != m || c->model_id != m->id) return set_err(QW_ERR_ARG, "null or mismatched handle");
    if (token >= m->cfg.vocab) return set_err(QW_ERR_ARG, "token id >= vocab_size");
    if (pos >= c->max_seq) return set_err(QW_ERR_ARG, "pos exceeds the KV cache size");  // metal_inference.rs:321
    QW_CUDA(cudaSetDevice(m->device));
    m->h_stage[0] = token;
    QW_CUDA(cudaMemcpyAsync(m->d_tok, m->h_stage, 4, cudaMemcpyHostToDevice, m->stream));
    if (int e = launch_decode(m, c, m->d_tok, nullptr, false, m->d_logits, pos, 1, m->stream)) return e;
    QW_CUDA(cudaMemcpyAsync(m->h_logits, m->d_logits, m->cfg.vocab * 4, cudaMemcpyDeviceToHost, m->stream));
    QW_CUDA(cudaStreamSynchronize(m->stream));
    if (int e = check_device_err(m)) return e;
    std::memcpy(logits_out, m->h_logits, m->cfg.vocab * 4);
    return QW_OK;
}

int qw_decode(qw_model* m, qw_cache* c, uint32_t first, size_t start_pos, size_t steps, qw_token_fn on_token, void* user) {
    if (!m || !c || c->m != m || c->model_id != m->id) return set_err(QW_ERR_ARG, "null or mismatched handle");
    if (steps == 0) return QW_OK;
    if (first >= m->cfg.vocab) return set_err(QW_ERR_ARG, "token id >= vocab_size");
    if (start_pos + steps > c->max_seq) return set_err(QW_ERR_ARG, "start_pos + steps exceeds the KV cache size");
    QW_CUDA(cudaSetDevice(m->device));
    if (int e = ensure_token_capacity(m, steps + 1)) return e;
    m->h_stage[0] = first;
    __atomic_store_n(m->h_count, 0u, __ATOMIC_RELEASE);
    QW_CUDA(cudaMemcpyAsync(m->d_tok, m->h_stage, 4, cudaMemcpyHostToDevice, m->stream));
    if (int e = launch_decode(m, c, m->d_tok, m->d_tok, true, nullptr, start_pos, steps, m->stream)) return e;
    // hand each token to on_token as soon as the GPU publishes it
    size_t done = 0;
    unsigned polls = 0;
    for (;;) {
        const unsigned cnt = __atomic_load_n(m->h_count, __ATOMIC_ACQUIRE);
        while (done < cnt && done < steps) {
            ++done;
            if (on_token) on_token(user, m->h_tok[done]);
        }
        if (done >= steps) break;
        if ((++polls & 63) == 0) {
            cudaError_t q = cudaStreamQuery(m->stream);
            if (q != cudaErrorNotReady) {
                const unsigned fin = __atomic_load_n(m->h_count, __ATOMIC_ACQUIRE);
                while (done < fin && done < steps) {
                    ++done;
                    if (on_token) on_token(user, m->h_tok[done]);
                }
                break;
            }
        }
    }
    QW_CUDA(cudaStreamSynchronize(m->stream));
    if (int e = check_device_err(m)) return e;
    if (done != steps) return set_err(QW_ERR_CUDA, "decode ended before producing every token");
    return QW_OK;
}

int qw_forward_device(qw_model* m, qw_cache* c, const uint32_t* d_token, size_t pos, float* d_logits, void* stream) {
    if (!m || !c || !d_token || c->m != m || c->model_id != m->id) return set_err(QW_ERR_ARG, "null or mismatched handle");
    if (pos >= c->max_seq) return set_err(QW_ERR_ARG, "pos exceeds the KV cache size");
    QW_CUDA(cudaSetDevice(m->device));
    return launch_decode(m, c, d_token, nullptr, false, d_logits, pos, 1, pick_stream(m, stream));
}

int qw_decode_device(qw_model* m, qw_cache* c, uint32_t* d_tokens, size_t start_pos, size_t steps, void* stream) {
    if (!m || !c || !d_tokens || c->m != m || c->model_id != m->id) return set_err(QW_ERR_ARG, "null or mismatched handle");
    if (steps == 0) return QW_OK;
    if (start_pos + steps > c->max_seq) return set_err(QW_ERR_ARG, "start_pos + steps exceeds the KV cache size");
    QW_CUDA(cudaSetDevice(m->device));
    return launch_decode(m, c, d_tokens, d_tokens, false, nullptr, start_pos, steps, pick_stream(m, stream));
}

int qw_sync(qw_model* m, void* stream) {
    if (!m) return set_err(QW_ERR_ARG, "null handle");
    QW_CUDA(cudaSetDevice(m->device));
    QW_CUDA(cudaStreamSynchronize(pick_stream(m, stream)));
    if (int e = check_device_err(m)) return e;
    // the prefill GEMMs report an expired pipeline wait through the device's shared error word
    // (word 0) and an input id >= vocab_size in device memory (word 1, read as row 0 instead)
    if (int* ew = qw::device_err_word_for(m->device)) {
        int h[2] = {0, 0};
        QW_CUDA(cudaMemcpy(h, ew, sizeof h, cudaMemcpyDeviceToHost));
        if (h[0] || h[1]) {
            QW_CUDA(cudaMemset(ew, 0, sizeof h));
            if (h[0]) return set_err(QW_ERR_DEVICE_TIMEOUT, "prefill: a GEMM pipeline wait expired on the device");
            return set_err(QW_ERR_ARG, "device: an input token id >= vocab_size (row 0 was used instead)");
        }
    }
    return QW_OK;
}

int qw_cache_read(qw_cache* c, size_t layer, size_t n, float* k_out, float* v_out) {
    if (!c || !k_out || !v_out) return set_err(QW_ERR_ARG, "null argument");
    if (layer >= c->layers || n > c->max_seq) return set_err(QW_ERR_ARG, "layer or n out of range");
    if (n == 0) return QW_OK;
    QW_CUDA(cudaSetDevice(c->device));
    QW_CUDA(cudaDeviceSynchronize());
    const size_t D = c->head_dim, KVD = c->kv_heads * D;
    for (size_t h = 0; h < c->kv_heads; h++) {
        const size_t src = ((layer * c->kv_heads + h) * c->max_seq) * D;
        QW_CUDA(cudaMemcpy2D(k_out + h * D, KVD * 4, c->d_k + src, D * 4, D * 4, n, cudaMemcpyDeviceToHost));
        QW_CUDA(cudaMemcpy2D(v_out + h * D, KVD * 4, c->d_v + src, D * 4, D * 4, n, cudaMemcpyDeviceToHost));
    }
    return QW_OK;
}

}  // extern "C"
