// capi.cu: the extern "C" entry points of libtrmoe.so (declared in include/trmoe.h).
//
// Host side of the layer hook (tr_gpu_moe_*) and of the kernel-level API (tr_matmul*, tr_softmax,
// tr_swiglu). Plain CUDA runtime; no torch. Every host wait on the GPU polls with a deadline and
// reports a timeout as an error instead of blocking forever.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <chrono>
#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "../../include/trmoe.h"
#include "common.cuh"
#include "expf.cuh"
#include "layouts.cuh"
#include "moe_kernels.cuh"
#include "kernel_api.cuh"
#include "fused_layer.cuh"
#include "gguf_file.h"
#include "attention.cuh"
#include "prefill.cuh"
#include "ep.cuh"
#include "ffn_norm.cuh"

namespace {

thread_local std::string g_err;

void set_err(const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
}

void put_err(char *err, size_t err_len) {
    if (err != nullptr && err_len > 0) snprintf(err, err_len, "%s", g_err.c_str());
}

bool ck(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return true;
    set_err("%s: %s", what, cudaGetErrorString(e));
    return false;
}

// waits for the stream, polling; a GPU that does not finish within timeout_s is an error, not a hang
bool stream_wait(cudaStream_t s, double timeout_s = 60.0) {
    const auto t0 = std::chrono::steady_clock::now();
    for (unsigned spins = 0;; spins++) {
        const cudaError_t e = cudaStreamQuery(s);
        if (e == cudaSuccess) return true;
        if (e != cudaErrorNotReady) return ck(e, "cudaStreamQuery");
        const double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (dt > timeout_s) {
            set_err("the GPU did not finish within %.0f s", timeout_s);
            return false;
        }
        if (spins > 64) std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

int64_t align_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }


// Copies one GGUF matrix (rows x cols of type) from the host into dst in its device layout;
// tmp: a device staging buffer of at least the matrix's bytes (for the repacked types).
bool upload_matrix(int type, int64_t rows, int64_t cols, const void *host, uint8_t *dst, uint8_t *tmp,
                   cudaStream_t st) {
    const int64_t bytes = trx_row_bytes(type, cols) * rows;
    if (bytes <= 0) {
        set_err("type %d with %lld columns has no whole rows", type, (long long)cols);
        return false;
    }
    if (type == TRX_Q8_0 || type == TRX_Q6_K) {
        if (cols % 256 != 0) {
            set_err("type %d needs a multiple of 256 columns, got %lld", type, (long long)cols);
            return false;
        }
        if (!ck(cudaMemcpyAsync(tmp, host, (size_t)bytes, cudaMemcpyHostToDevice, st), "upload")) return false;
        if (type == TRX_Q8_0) trx_repack_q8l<<<(unsigned)rows, 256, 0, st>>>(tmp, dst, rows, cols);
        else trx_repack_q6l<<<(unsigned)rows, 128, 0, st>>>(tmp, dst, rows, cols);
        if (!ck(cudaGetLastError(), "repack")) return false;
    } else {
        if (!ck(cudaMemcpyAsync(dst, host, (size_t)bytes, cudaMemcpyHostToDevice, st), "upload")) return false;
    }
    return stream_wait(st, 300.0);
}

struct WorkLayout {
    int64_t off[26];
    int64_t total;
};

// carve the workspace of one context (every piece 256-byte aligned)
// whether a context can take the tensor-core road for long passes (Q8_0 gate/up and down)
bool prefill_capable(const tr_gpu_moe_config &c) { return c.gate_type == TRX_Q8_0 && c.down_type == TRX_Q8_0; }

WorkLayout work_layout(const tr_gpu_moe_config &c) {
    const int64_t T = c.max_tokens, E = c.n_expert, k = c.n_used, H = c.n_embd, F = c.n_ff, R = T * k;
    const bool pf = prefill_capable(c);
    const int64_t sizes[] = {
        T * E * 4,          // 0 logits
        R * 4,              // 1 sel_id
        R * 4,              // 2 sel_w
        (E + 1) * 4,        // 3 offsets
        R * 4,              // 4 place
        R * 4,              // 5 xmap
        E * 4,              // 6 active
        4,                  // 7 n_active
        4,                  // 8 route_cnt
        (H / TRX_DN_CHUNK) * 4 + 256, // 9 comb_cnt, then the error flag
        T * H * 4,          // 10 x_lc
        T * H * 4,          // 11 xq
        T * (H / 32) * 8,   // 12 xq_bf
        T * (H / 256) * 8,  // 13 xq_sc
        R * F * 4,          // 14 h
        R * F * 4,          // 15 hq
        R * (F / 32) * 8,   // 16 hq_bf
        R * (F / 256) * 8,  // 17 hq_sc
        R * H * 4,          // 18 h3
        T * H * 4,          // 19 host-call normed
        T * H * 4,          // 20 host-call x
        R * 8,              // 21 host-call sel_id
        R * 4,              // 22 host-call sel_w
        (int64_t)sizeof(TrxSync), // 23 the fused kernel's counters
        pf ? R * H * 4 : 0, // 24 the tensor-core road: the grouped inputs' hi plane
        pf ? R * H * 4 : 0, // 25 and lo plane
    };
    WorkLayout w{};
    int64_t o = 0;
    for (int i = 0; i < 26; i++) {
        w.off[i] = o;
        o += align_up(sizes[i], 256);
    }
    w.total = o;
    return w;
}

int64_t mat_stride(int type, int64_t rows, int64_t cols) { return align_up(trx_row_bytes(type, cols) * rows, 256); }

int64_t layer_bytes(const tr_gpu_moe_config &c) {
    const int64_t E = c.n_expert, H = c.n_embd, F = c.n_ff;
    return align_up(trx_row_bytes(c.router_type, H) * E, 256) + align_up(E * 4, 256) +
           2 * E * mat_stride(c.gate_type, F, H) + E * mat_stride(c.down_type, H, F);
}

} // namespace

struct tr_gpu_moe {
    tr_gpu_moe_config cfg;
    int device = 0, sm_count = 148;
    cudaStream_t stream = nullptr;
    std::vector<uint8_t *> layer_mem;
    std::vector<TrxLayer> layers;
    std::vector<int> layer_set;
    uint8_t *work_mem = nullptr;
    uint8_t *tmp = nullptr;
    TrxWork work{};
    int grid_gu = 0, grid_dn = 0, grid_fused = 0;
    size_t smem_gu = 0, smem_dn = 0, smem_fused = 0;
    TrxSync *sync = nullptr;
    uint64_t *trace = nullptr;
    uint32_t epoch = 0;
    // the host-pointer road's completion word: mapped pinned host memory the fused kernel writes its epoch to
    uint32_t *h_done = nullptr, *d_done = nullptr;
    // ffn_norm (tr_gpu_moe_set_ffn_norm): per layer n_embd weights on the device, the epsilon, whether set
    float *norm_w = nullptr;
    std::vector<float> norm_eps;
    std::vector<int> norm_set;
    bool fused_ok = false;
    float *d_normed = nullptr, *d_x = nullptr;
    int64_t *d_sel_id = nullptr;
    float *d_sel_w = nullptr;
    // the tensor-core road (prefill.cuh): calls of at least pf_min tokens take it (0: never)
    bool pf_ok = false;
    int64_t pf_min = 0;
    float *pf_xhi = nullptr, *pf_xlo = nullptr;
    CUtensorMap pf_map_x[2], pf_map_h[2]; // A operands of the gate/up and of the down GEMM: hi, lo planes
    // expert parallelism: per layer the device tables of the experts' gate, up and down matrices (E pointers each),
    // and the scratch of tr_gpu_moe_experts_dev (grown to the largest call)
    const uint8_t **ep_tab = nullptr;
    uint8_t *ep_buf = nullptr;
    int64_t ep_cap = 0;
    // expert parallelism over peer memory (tr_gpu_moe_ep_peer_*): this rank's exchange region, the other ranks'
    // regions as opened here, and their device table
    uint8_t *epp_region = nullptr;
    int epp_n = 0, epp_rank = 0;
    int64_t epp_cap = 0;
    std::vector<uint8_t *> epp_opened;
    TrxEpPeers *epp_dev = nullptr;
    // zone timing (tr_gpu_moe_profile): one set of events per profiled call, read when asked, so that
    // profiling never makes a call wait for the one before it
    struct EvSet {
        cudaEvent_t ev[TRMOE_ZONES + 1];
        bool used[TRMOE_ZONES];
    };
    bool prof = false;
    std::vector<EvSet> evs;   // every set created so far
    size_t ev_next = 0;       // sets [0, ev_next) hold calls not yet added to the sums
    double prof_ms[TRMOE_ZONES] = {};
    int64_t prof_calls[TRMOE_ZONES] = {};
};

#define TRMOE_PROF_SETS 4096

// adds the recorded calls' zone times to the sums (waits for their events)
static bool prof_collect(tr_gpu_moe *m) {
    for (size_t i = 0; i < m->ev_next; i++) {
        auto &e = m->evs[i];
        if (!ck(cudaEventSynchronize(e.ev[TRMOE_ZONES]), "cudaEventSynchronize")) return false;
        for (int z = 0; z < TRMOE_ZONES; z++) {
            if (!e.used[z]) continue;
            float ms = 0.0f;
            if (!ck(cudaEventElapsedTime(&ms, e.ev[z], e.ev[z + 1]), "cudaEventElapsedTime")) return false;
            m->prof_ms[z] += ms;
            m->prof_calls[z] += 1;
        }
    }
    m->ev_next = 0;
    return true;
}

// the event set of the next profiled call (collecting the recorded ones when the ring is full)
static tr_gpu_moe::EvSet *prof_slot(tr_gpu_moe *m) {
    if (m->ev_next == TRMOE_PROF_SETS && !prof_collect(m)) return nullptr;
    if (m->ev_next == m->evs.size()) {
        tr_gpu_moe::EvSet e{};
        for (auto &v : e.ev)
            if (!ck(cudaEventCreate(&v), "cudaEventCreate")) return nullptr;
        m->evs.push_back(e);
    }
    return &m->evs[m->ev_next++];
}

using GateUpFn = void (*)(TrxLayer, TrxShape, TrxWork);
using DownFn = void (*)(TrxLayer, TrxShape, TrxWork, float *, int, float *);

static GateUpFn gateup_fn(int gate_type, int down_type) {
    const bool lc = down_type != TRX_Q4_K;
    if (gate_type == TRX_Q4_K) return lc ? trx_k_gateup<TRX_Q4_K, true> : trx_k_gateup<TRX_Q4_K, false>;
    return lc ? trx_k_gateup<TRX_Q8_0, true> : trx_k_gateup<TRX_Q8_0, false>;
}

static DownFn down_fn(int down_type) {
    if (down_type == TRX_Q4_K) return trx_k_down<TRX_Q4_K>;
    if (down_type == TRX_Q8_0) return trx_k_down<TRX_Q8_0>;
    return trx_k_down<TRX_Q6_K>;
}

using LayerFn = void (*)(TrxLayer, TrxShape, const float *, int, TrxWork, TrxSync *, float *, float *, uint32_t, int,
                         int);

static LayerFn layer_fn(int gate_type, int down_type) {
    if (gate_type == TRX_Q4_K) {
        if (down_type == TRX_Q4_K) return trx_k_layer<TRX_Q4_K, TRX_Q4_K>;
        if (down_type == TRX_Q6_K) return trx_k_layer<TRX_Q4_K, TRX_Q6_K>;
        return trx_k_layer<TRX_Q4_K, TRX_Q8_0>;
    }
    if (down_type == TRX_Q4_K) return trx_k_layer<TRX_Q8_0, TRX_Q4_K>;
    if (down_type == TRX_Q6_K) return trx_k_layer<TRX_Q8_0, TRX_Q6_K>;
    return trx_k_layer<TRX_Q8_0, TRX_Q8_0>;
}

// the fused kernel: the most shared memory a CTA may take, and a cooperative grid of one CTA per SM
static bool plan_fused(tr_gpu_moe *m) {
    const tr_gpu_moe_config &c = m->cfg;
    int coop = 0, occ = 0;
    LayerFn fn = layer_fn(c.gate_type, c.down_type);
    cudaFuncAttributes fa{};
    if (!ck(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, m->device), "attribute") ||
        !ck(cudaFuncGetAttributes(&fa, fn), "cudaFuncGetAttributes"))
        return false;
    if (!coop) return true; // the multi-kernel road serves every pass
    const size_t limit = 232448; // bytes of shared memory a block may use on sm_100 (static + dynamic)
    m->smem_fused = limit - fa.sharedSizeBytes - 1024;
    if (!ck(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)m->smem_fused), "smem fused") ||
        !ck(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, TRX_FU_THREADS, m->smem_fused), "occupancy"))
        return false;
    m->grid_fused = m->sm_count; // one CTA per SM (occupancy is at least one: checked)
    m->fused_ok = occ >= 1;
    return true;
}

// the stages of a fused call of T tokens: as many as this CTA's share of the routed rows can use, within the
// shared memory; false when even two of each do not fit (the multi-kernel road then takes the call)
static bool fused_stages(const tr_gpu_moe *m, int T, int *sg, int *sd, int k_override = 0) {
    const tr_gpu_moe_config &c = m->cfg;
    const int H = (int)c.n_embd, F = (int)c.n_ff, k = k_override ? k_override : (int)c.n_used;
    const int64_t act = std::min<int64_t>(c.n_expert, (int64_t)T * k);
    const int64_t rows_g = (act * F + m->grid_fused - 1) / m->grid_fused, rows_d = (act * H + m->grid_fused - 1) / m->grid_fused;
    int g = (int)std::min<int64_t>(TRX_FU_MAXST, std::max<int64_t>(2, (rows_g + TRX_GU_CHUNK - 1) / TRX_GU_CHUNK + 1));
    int d = (int)std::min<int64_t>(TRX_FU_MAXST, std::max<int64_t>(2, (rows_d + TRX_DN_CHUNK - 1) / TRX_DN_CHUNK + 1));
    auto fits = [&](int a, int b) {
        return trx_fused_layout(c.gate_type, c.down_type, H, F, T, k, a, b, (int)c.n_expert, m->grid_fused).total <= m->smem_fused;
    };
    while (!fits(g, d)) {
        const TrxFusedSmem l = trx_fused_layout(c.gate_type, c.down_type, H, F, T, k, g, d, (int)c.n_expert, m->grid_fused);
        if (g > 2 && (g * l.gu_stage >= d * l.dn_stage || d <= 2)) g--;
        else if (d > 2) d--;
        else return false;
    }
    *sg = g;
    *sd = d;
    return true;
}

// shared memory of the streaming kernels and their persistent grids (every CTA resident at once)
static bool plan_kernels(tr_gpu_moe *m) {
    const tr_gpu_moe_config &c = m->cfg;
    const int64_t rb_gu = trx_row_bytes(c.gate_type, c.n_embd);
    const int64_t rb_dn = c.down_type == TRX_Q6_K ? c.n_ff / 256 * 208 : trx_row_bytes(c.down_type, c.n_ff);
    m->smem_gu = (size_t)(TRX_STAGES * 2 * TRX_GU_CHUNK * rb_gu + TRX_STAGES * 8);
    m->smem_dn = (size_t)(TRX_STAGES * TRX_DN_CHUNK * rb_dn + TRX_STAGES * 8);
    const size_t smem_router = (size_t)(1 + TRX_TOK_STAGE) * c.n_embd * 4;
    GateUpFn gu = gateup_fn(c.gate_type, c.down_type);
    DownFn dn = down_fn(c.down_type);
    int occ_gu = 0, occ_dn = 0;
    bool ok = ck(cudaFuncSetAttribute(gu, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)m->smem_gu), "smem gate/up") &&
              ck(cudaFuncSetAttribute(dn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)m->smem_dn), "smem down") &&
              ck(cudaFuncSetAttribute(trx_k_router_many<TRX_F32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)trx_router_many_smem(TRX_F32, TRX_MAX_EXPERTS)),
                 "smem router") &&
              ck(cudaFuncSetAttribute(trx_k_router_many<TRX_BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)trx_router_many_smem(TRX_BF16, TRX_MAX_EXPERTS)),
                 "smem router") &&
              ck(cudaFuncSetAttribute(trx_k_router, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_router),
                 "smem router") &&
              ck(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_gu, gu, 256, m->smem_gu), "occupancy") &&
              ck(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_dn, dn, 256, m->smem_dn), "occupancy");
    if (!ok) return false;
    if (occ_gu < 1 || occ_dn < 1) {
        set_err("the expert kernels do not fit on an SM (occupancy %d, %d)", occ_gu, occ_dn);
        return false;
    }
    m->grid_gu = occ_gu * m->sm_count;
    m->grid_dn = occ_dn * m->sm_count;
    return plan_fused(m);
}

extern "C" const char *trmoe_last_error(void) { return g_err.c_str(); }

extern "C" uint64_t tr_gpu_moe_bytes(const tr_gpu_moe_config *cfg) {
    if (cfg == nullptr) return 0;
    return (uint64_t)(layer_bytes(*cfg) * cfg->n_layers + work_layout(*cfg).total);
}

static bool check_config(const tr_gpu_moe_config *c) {
    if (c == nullptr) {
        set_err("no config");
        return false;
    }
    if (c->n_layers < 1 || c->n_expert < 1 || c->n_expert > TRX_MAX_EXPERTS || c->n_used < 1 ||
        c->n_used > TRX_MAX_USED || c->n_used > c->n_expert || c->max_tokens < 1) {
        set_err("unsupported counts (layers %lld, experts %lld, used %lld, max tokens %lld)", (long long)c->n_layers,
                (long long)c->n_expert, (long long)c->n_used, (long long)c->max_tokens);
        return false;
    }
    if (c->n_embd % 256 || c->n_ff % 256 || c->n_embd < 256 || c->n_ff < 256 || c->n_embd > 8192) {
        set_err("n_embd and n_ff must be multiples of 256 (n_embd <= 8192), got %lld and %lld", (long long)c->n_embd,
                (long long)c->n_ff);
        return false;
    }
    if (c->router_type != TRX_F32 && c->router_type != TRX_BF16) {
        set_err("router type %d not supported (F32, BF16)", c->router_type);
        return false;
    }
    if (c->gate_type != TRX_Q8_0 && c->gate_type != TRX_Q4_K) {
        set_err("gate/up type %d not supported (Q8_0, Q4_K)", c->gate_type);
        return false;
    }
    if (c->down_type != TRX_Q8_0 && c->down_type != TRX_Q4_K && c->down_type != TRX_Q6_K) {
        set_err("down type %d not supported (Q8_0, Q4_K, Q6_K)", c->down_type);
        return false;
    }
    if (c->gate_type == TRX_Q4_K && c->n_embd != 2048) {
        set_err("Q4_K gate/up needs n_embd 2048 (8 blocks a row), got %lld", (long long)c->n_embd);
        return false;
    }
    if (c->down_type == TRX_Q4_K && c->n_ff != 1024) {
        set_err("Q4_K down needs n_ff 1024 (4 blocks a row), got %lld", (long long)c->n_ff);
        return false;
    }
    return true;
}

// a 2-D fp32 tensor map over rows x cols (row-major), boxes of 32 columns x 128 rows, 128-byte swizzle
static bool encode_map(CUtensorMap *map, float *base, int64_t rows, int64_t cols) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (encode == nullptr) {
        cudaDriverEntryPointQueryResult q{};
        void *fn = nullptr;
        if (!ck(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q), "driver entry point") ||
            q != cudaDriverEntryPointSuccess || fn == nullptr) {
            if (g_err.empty()) set_err("cuTensorMapEncodeTiled is not available");
            return false;
        }
        encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
    }
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows}, strides[1] = {(cuuint64_t)cols * 4};
    const cuuint32_t box[2] = {TRX_PF_BK, TRX_PF_BM}, es[2] = {1, 1};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, es,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_err("cuTensorMapEncodeTiled failed (%d)", (int)r);
        return false;
    }
    return true;
}

// the tensor-core road: its kernels' shared memory and the A operands' tensor maps (the h planes reuse the h and
// hq regions, which the Q8_0 roads of the other kernels leave free during a prefill call)
static bool plan_prefill(tr_gpu_moe *m) {
    const tr_gpu_moe_config &c = m->cfg;
    const int64_t R = c.max_tokens * c.n_used;
    if (!ck(cudaFuncSetAttribute(trx_k_pf_gemm<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, TRX_PF_SMEM),
            "smem prefill") ||
        !ck(cudaFuncSetAttribute(trx_k_pf_gemm<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, TRX_PF_SMEM),
            "smem prefill"))
        return false;
    if (!encode_map(&m->pf_map_x[0], m->pf_xhi, R, c.n_embd) || !encode_map(&m->pf_map_x[1], m->pf_xlo, R, c.n_embd) ||
        !encode_map(&m->pf_map_h[0], m->work.h, R, c.n_ff) ||
        !encode_map(&m->pf_map_h[1], reinterpret_cast<float *>(m->work.hq), R, c.n_ff))
        return false;
    m->pf_ok = true;
    m->pf_min = 256;
    return true;
}

extern "C" tr_gpu_moe *tr_gpu_moe_create(const tr_gpu_moe_config *cfg, int device, char *err, size_t err_len) {
    g_err.clear();
    if (!check_config(cfg)) {
        put_err(err, err_len);
        return nullptr;
    }
    tr_gpu_moe *m = new tr_gpu_moe();
    m->cfg = *cfg;
    m->device = device;
    const WorkLayout wl = work_layout(*cfg);
    const int64_t lb = layer_bytes(*cfg);
    const int64_t tmp_bytes = std::max(std::max(trx_row_bytes(cfg->gate_type, cfg->n_embd) * cfg->n_ff,
                                                trx_row_bytes(cfg->down_type, cfg->n_ff) * cfg->n_embd),
                                       trx_row_bytes(cfg->router_type, cfg->n_embd) * cfg->n_expert);
    bool ok = ck(cudaSetDevice(device), "cudaSetDevice") &&
              ck(cudaDeviceGetAttribute(&m->sm_count, cudaDevAttrMultiProcessorCount, device), "attribute") &&
              ck(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking), "cudaStreamCreate") &&
              ck(cudaMalloc(&m->work_mem, (size_t)wl.total), "cudaMalloc(workspace)") &&
              ck(cudaMemset(m->work_mem, 0, (size_t)wl.total), "cudaMemset") &&
              ck(cudaMalloc(&m->tmp, (size_t)tmp_bytes), "cudaMalloc(staging)");
    if (ok) {
        m->layer_mem.assign((size_t)cfg->n_layers, nullptr);
        m->layers.assign((size_t)cfg->n_layers, TrxLayer{});
        m->layer_set.assign((size_t)cfg->n_layers, 0);
        for (int64_t l = 0; l < cfg->n_layers && ok; l++)
            ok = ck(cudaMalloc(&m->layer_mem[(size_t)l], (size_t)lb), "cudaMalloc(layer)");
    }
    if (ok) ok = plan_kernels(m);
    // the completion word of the host-pointer road (without it that road copies x and polls the stream)
    if (ok && cudaHostAlloc((void **)&m->h_done, 256, cudaHostAllocMapped) == cudaSuccess) {
        *(volatile uint32_t *)m->h_done = 0;
        if (cudaHostGetDevicePointer((void **)&m->d_done, m->h_done, 0) != cudaSuccess) {
            cudaFreeHost(m->h_done);
            m->h_done = m->d_done = nullptr;
        }
    }
    cudaGetLastError();
    if (!ok) {
        put_err(err, err_len);
        tr_gpu_moe_free(m);
        return nullptr;
    }
    uint8_t *b = m->work_mem;
    TrxWork &w = m->work;
    w.logits = (float *)(b + wl.off[0]);
    w.sel_id = (int32_t *)(b + wl.off[1]);
    w.sel_w = (float *)(b + wl.off[2]);
    w.offsets = (int32_t *)(b + wl.off[3]);
    w.place = (int32_t *)(b + wl.off[4]);
    w.xmap = (int32_t *)(b + wl.off[5]);
    w.active = (int32_t *)(b + wl.off[6]);
    w.n_active = (int32_t *)(b + wl.off[7]);
    w.route_cnt = (uint32_t *)(b + wl.off[8]);
    w.comb_cnt = (uint32_t *)(b + wl.off[9]);
    w.err = (int32_t *)(b + wl.off[9] + (cfg->n_embd / TRX_DN_CHUNK) * 4);
    w.x_lc = (float *)(b + wl.off[10]);
    w.xq = (uint32_t *)(b + wl.off[11]);
    w.xq_bf = (double *)(b + wl.off[12]);
    w.xq_sc = (double *)(b + wl.off[13]);
    w.h = (float *)(b + wl.off[14]);
    w.hq = (uint32_t *)(b + wl.off[15]);
    w.hq_bf = (double *)(b + wl.off[16]);
    w.hq_sc = (double *)(b + wl.off[17]);
    w.h3 = (float *)(b + wl.off[18]);
    m->d_normed = (float *)(b + wl.off[19]);
    m->d_x = (float *)(b + wl.off[20]);
    m->d_sel_id = (int64_t *)(b + wl.off[21]);
    m->d_sel_w = (float *)(b + wl.off[22]);
    m->sync = (TrxSync *)(b + wl.off[23]);
    if (prefill_capable(*cfg)) {
        m->pf_xhi = (float *)(b + wl.off[24]);
        m->pf_xlo = (float *)(b + wl.off[25]);
        if (!plan_prefill(m)) {
            put_err(err, err_len);
            tr_gpu_moe_free(m);
            return nullptr;
        }
    }
    return m;
}

extern "C" void tr_gpu_moe_free(tr_gpu_moe *m) {
    if (m == nullptr) return;
    cudaSetDevice(m->device);
    if (m->stream) stream_wait(m->stream, 60.0);
    for (uint8_t *p : m->layer_mem)
        if (p) cudaFree(p);
    if (m->work_mem) cudaFree(m->work_mem);
    if (m->tmp) cudaFree(m->tmp);
    if (m->trace) cudaFree(m->trace);
    if (m->ep_tab) cudaFree(m->ep_tab);
    if (m->ep_buf) cudaFree(m->ep_buf);
    if (m->h_done) cudaFreeHost(m->h_done);
    for (uint8_t *p : m->epp_opened)
        if (p) cudaIpcCloseMemHandle(p);
    if (m->epp_dev) cudaFree(m->epp_dev);
    if (m->epp_region) cudaFree(m->epp_region);
    if (m->norm_w) cudaFree(m->norm_w);
    for (auto &es : m->evs)
        for (cudaEvent_t e : es.ev) cudaEventDestroy(e);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

extern "C" int tr_gpu_moe_set_layer(tr_gpu_moe *m, int64_t layer, const void *router, const float *router_bias,
                                    const void *const *gate, const void *const *up, const void *const *down,
                                    char *err, size_t err_len) {
    g_err.clear();
    if (m == nullptr || layer < 0 || layer >= m->cfg.n_layers || router == nullptr || gate == nullptr ||
        up == nullptr || down == nullptr) {
        set_err("bad arguments to tr_gpu_moe_set_layer");
        put_err(err, err_len);
        return -1;
    }
    const tr_gpu_moe_config &c = m->cfg;
    const int64_t E = c.n_expert, H = c.n_embd, F = c.n_ff;
    if (!ck(cudaSetDevice(m->device), "cudaSetDevice")) {
        put_err(err, err_len);
        return -1;
    }
    uint8_t *b = m->layer_mem[(size_t)layer];
    TrxLayer L{};
    L.router_type = c.router_type;
    L.gate_type = L.up_type = c.gate_type;
    L.down_type = c.down_type;
    const int64_t router_bytes = trx_row_bytes(c.router_type, H) * E;
    int64_t o = 0;
    L.router = b + o;
    o += align_up(router_bytes, 256);
    float *bias = (float *)(b + o);
    o += align_up(E * 4, 256);
    L.router_bias = router_bias ? bias : nullptr;
    L.gate_mb = mat_stride(c.gate_type, F, H);
    L.up_mb = L.gate_mb;
    L.down_mb = mat_stride(c.down_type, H, F);
    L.gate = b + o;
    o += E * L.gate_mb;
    L.up = b + o;
    o += E * L.up_mb;
    L.down = b + o;
    // the router in lane-row order (trx_repack_lanerows), staged through the matrix buffer
    bool ok = ck(cudaMemcpyAsync(m->tmp, router, (size_t)router_bytes, cudaMemcpyHostToDevice, m->stream), "upload router");
    if (ok) {
        trx_repack_lanerows<<<(unsigned)E, 256, 0, m->stream>>>(m->tmp, (uint8_t *)L.router, E, H,
                                                                  c.router_type == TRX_F32 ? 4 : 2);
        ok = ck(cudaGetLastError(), "repack router") && stream_wait(m->stream, 300.0);
    }
    if (ok && router_bias)
        ok = ck(cudaMemcpyAsync(bias, router_bias, (size_t)E * 4, cudaMemcpyHostToDevice, m->stream), "upload bias");
    for (int64_t e = 0; e < E && ok; e++) {
        if (gate[e] == nullptr && up[e] == nullptr && down[e] == nullptr) continue; // held by another rank
        ok = upload_matrix(c.gate_type, F, H, gate[e], (uint8_t *)L.gate + e * L.gate_mb, m->tmp, m->stream) &&
             upload_matrix(c.gate_type, F, H, up[e], (uint8_t *)L.up + e * L.up_mb, m->tmp, m->stream) &&
             upload_matrix(c.down_type, H, F, down[e], (uint8_t *)L.down + e * L.down_mb, m->tmp, m->stream);
    }
    if (ok) ok = stream_wait(m->stream, 300.0);
    // the layer's matrix tables for tr_gpu_moe_experts_dev
    if (ok && m->ep_tab == nullptr)
        ok = ck(cudaMalloc(&m->ep_tab, (size_t)c.n_layers * 3 * E * sizeof(void *)), "cudaMalloc(expert tables)");
    if (ok) {
        std::vector<const uint8_t *> tab((size_t)(3 * E));
        for (int64_t e = 0; e < E; e++) {
            tab[(size_t)e] = L.gate + e * L.gate_mb;
            tab[(size_t)(E + e)] = L.up + e * L.up_mb;
            tab[(size_t)(2 * E + e)] = L.down + e * L.down_mb;
        }
        ok = ck(cudaMemcpy(m->ep_tab + (size_t)layer * 3 * E, tab.data(), tab.size() * sizeof(void *),
                           cudaMemcpyHostToDevice),
                "upload expert tables");
    }
    if (!ok) {
        put_err(err, err_len);
        return -1;
    }
    m->layers[(size_t)layer] = L;
    m->layer_set[(size_t)layer] = 1;
    return 0;
}

extern "C" int tr_gpu_moe_profile(tr_gpu_moe *m, int on) {
    g_err.clear();
    if (m == nullptr || !ck(cudaSetDevice(m->device), "cudaSetDevice")) return -1;
    if (!prof_collect(m)) return -1;
    m->prof = on != 0;
    for (int z = 0; z < TRMOE_ZONES; z++) {
        m->prof_ms[z] = 0.0;
        m->prof_calls[z] = 0;
    }
    return 0;
}

extern "C" int tr_gpu_moe_trace(tr_gpu_moe *m, int on) {
    g_err.clear();
    if (m == nullptr || !ck(cudaSetDevice(m->device), "cudaSetDevice") || !stream_wait(m->stream)) return -1;
    if (!on) {
        if (m->trace) cudaFree(m->trace);
    if (m->ep_tab) cudaFree(m->ep_tab);
    if (m->ep_buf) cudaFree(m->ep_buf);
        m->trace = nullptr;
        return 0;
    }
    const size_t bytes = (size_t)std::max(m->grid_fused, 1) * 64 * 8;
    if (m->trace == nullptr && !ck(cudaMalloc(&m->trace, bytes), "cudaMalloc(trace)")) return -1;
    return ck(cudaMemset(m->trace, 0, bytes), "cudaMemset(trace)") ? 0 : -1;
}

extern "C" int tr_gpu_moe_trace_read(tr_gpu_moe *m, uint64_t *slots, int64_t n) {
    g_err.clear();
    if (m == nullptr || m->trace == nullptr || slots == nullptr) {
        set_err("tracing is off");
        return -1;
    }
    if (!ck(cudaSetDevice(m->device), "cudaSetDevice") || !ck(cudaDeviceSynchronize(), "cudaDeviceSynchronize"))
        return -1;
    const int64_t have = (int64_t)m->grid_fused * 64;
    if (!ck(cudaMemcpy(slots, m->trace, (size_t)std::min(n, have) * 8, cudaMemcpyDeviceToHost), "copy trace")) return -1;
    return m->grid_fused;
}

extern "C" int tr_gpu_moe_profile_read(tr_gpu_moe *m, double *ms, int64_t *calls, int n_zones) {
    g_err.clear();
    if (m == nullptr || !ck(cudaSetDevice(m->device), "cudaSetDevice") || !prof_collect(m)) return -1;
    for (int z = 0; z < n_zones && z < TRMOE_ZONES; z++) {
        if (ms) ms[z] = m->prof_ms[z];
        if (calls) calls[z] = m->prof_calls[z];
    }
    return 0;
}

// after a kernel gave up: every counter and flag back to zero (the next call starts clean)
static void reset_counters(tr_gpu_moe *m, cudaStream_t st) {
    cudaMemsetAsync(m->work.err, 0, 4, st);
    cudaMemsetAsync(m->work.route_cnt, 0, 4, st);
    cudaMemsetAsync(m->work.comb_cnt, 0, (size_t)(m->cfg.n_embd / TRX_DN_CHUNK) * 4, st);
    cudaMemsetAsync(m->sync, 0, sizeof(TrxSync), st);
    m->epoch = 0;
    stream_wait(st);
}

extern "C" int tr_gpu_moe_launches(const tr_gpu_moe *m, int64_t n_tok) {
    if (m == nullptr) return 0;
    if (m->pf_ok && m->pf_min > 0 && n_tok >= m->pf_min && !m->prof) return 7; // route 3, gather, 2 GEMMs, combine
    int sg, sd;
    if (m->fused_ok && n_tok <= TRX_ROUTE_FUSED_MAX && m->cfg.n_expert + n_tok <= m->grid_fused && !m->prof &&
        fused_stages(m, (int)n_tok, &sg, &sd))
        return 1;
    return (n_tok <= TRX_ROUTE_FUSED_MAX ? 1 : 4) + 2 + (m->cfg.down_type == TRX_Q4_K ? 1 : 0);
}

extern "C" int tr_gpu_moe_check(tr_gpu_moe *m) {
    g_err.clear();
    if (m == nullptr || !ck(cudaSetDevice(m->device), "cudaSetDevice") || !stream_wait(m->stream)) return -1;
    int32_t flag = 0;
    if (!ck(cudaMemcpy(&flag, m->work.err, 4, cudaMemcpyDeviceToHost), "read error flag")) return -1;
    if (flag != 0) {
        reset_counters(m, m->stream);
        set_err("a kernel gave up on a bounded wait (device error flag %d)", flag);
        return -1;
    }
    return 0;
}

// router logits of a long pass: 16 tokens a block, every expert
static void launch_router_many(const TrxLayer &L, const TrxShape &S, const float *d_normed, int T, const TrxWork &w,
                               cudaStream_t st) {
    const unsigned blocks = (unsigned)((T + TRX_TOK_STAGE - 1) / TRX_TOK_STAGE);
    const size_t smem = trx_router_many_smem(L.router_type, S.E);
    if (L.router_type == TRX_F32) trx_k_router_many<TRX_F32><<<blocks, 256, smem, st>>>(L, S, d_normed, T, w);
    else trx_k_router_many<TRX_BF16><<<blocks, 256, smem, st>>>(L, S, d_normed, T, w);
}

// A long pass on the tensor-core road: the exact routing (router, top-k, sort), the inputs gathered as hi/lo planes,
// the gate/up and down GEMMs (3xTF32 on tcgen05), the exact combine.
static int launch_prefill(tr_gpu_moe *m, const TrxLayer &L, const TrxShape &S, const TrxWork &w, const float *d_normed,
                          int T, float *d_x, float *ffn_out, cudaStream_t st) {
    const int E = S.E, H = S.H, F = S.F, R = T * S.k;
    launch_router_many(L, S, d_normed, T, w, st);
    trx_k_route<<<(unsigned)((T + 7) / 8), 256, 0, st>>>(S, T, w);
    trx_k_sort<<<1, 1024, 0, st>>>(S, T, w);
    trx_k_pf_gather<<<(unsigned)R, 256, 0, st>>>(d_normed, w.xmap, w.offsets, E, H, m->pf_xhi, m->pf_xlo);
    const unsigned mtiles = (unsigned)((R + TRX_PF_BM - 1) / TRX_PF_BM + std::min(E, R));
    TrxPfArgs a{};
    a.offsets = w.offsets;
    a.active = w.active;
    a.n_active = w.n_active;
    a.err = w.err;
    a.wa = L.gate;
    a.wb = L.up;
    a.wa_mb = L.gate_mb;
    a.wb_mb = L.up_mb;
    a.K = H;
    a.N = F;
    a.out_hi = w.h;
    a.out_lo = reinterpret_cast<float *>(w.hq);
    trx_k_pf_gemm<true><<<dim3((unsigned)(F / 128), mtiles), TRX_PF_THREADS, TRX_PF_SMEM, st>>>(m->pf_map_x[0],
                                                                                               m->pf_map_x[1], a);
    a.wa = L.down;
    a.wb = nullptr;
    a.wa_mb = L.down_mb;
    a.wb_mb = 0;
    a.K = F;
    a.N = H;
    a.out_hi = w.h3;
    a.out_lo = nullptr;
    trx_k_pf_gemm<false><<<dim3((unsigned)(H / TRX_PF_BN), mtiles), TRX_PF_THREADS, TRX_PF_SMEM, st>>>(m->pf_map_h[0],
                                                                                                      m->pf_map_h[1], a);
    const int64_t n = (int64_t)T * H;
    trx_k_pf_combine<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(w.sel_w, w.place, w.h3, T, S.k, H, d_x, ffn_out);
    return ck(cudaGetLastError(), "prefill launch") ? 0 : -1;
}

// Enqueues parts [first, last] of one layer call on st: 0 route (router, top-k, dispatch, input preparation),
// 1 gate/up + SwiGLU, 2 the down input's Q4_K preparation, 3 down + combine + residual.
// whether a whole layer call of T tokens takes the fused kernel (launch_layer's choice)
#define TRX_HOST_ZC_MAX 16 // calls up to this many tokens may take the zero-copy host-pointer road

static bool takes_fused(const tr_gpu_moe *m, int T) {
    int sg, sd;
    return m->fused_ok && !m->prof && !(m->pf_ok && m->pf_min > 0 && T >= m->pf_min) && T <= TRX_ROUTE_FUSED_MAX &&
           (int)m->cfg.n_expert + T <= m->grid_fused && fused_stages(m, T, &sg, &sd);
}

// the fused decode kernel (fused_layer.cuh) over T rows of S's shape: one cooperative launch, a CTA an SM, with sg / sd
// stages (fused_stages) and the shared memory their layout takes
static int launch_fused(tr_gpu_moe *m, const TrxLayer &L, const TrxShape &S, const float *normed, int T, const TrxWork &w,
                        float *x_io, float *ffn_out, uint32_t epoch, int sg, int sd, cudaStream_t st, const char *what) {
    const tr_gpu_moe_config &c = m->cfg;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)m->grid_fused);
    cfg.blockDim = dim3(TRX_FU_THREADS);
    cfg.dynamicSmemBytes =
        trx_fused_layout(c.gate_type, c.down_type, S.H, S.F, T, S.k, sg, sd, S.E, m->grid_fused).total;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return ck(cudaLaunchKernelEx(&cfg, layer_fn(c.gate_type, c.down_type), L, S, normed, T, w, m->sync, x_io, ffn_out,
                                 epoch, sg, sd),
              what)
               ? 0
               : -1;
}

static int launch_ffn_norm(tr_gpu_moe *m, int64_t layer, const float *x, int64_t n_tok, float *normed, cudaStream_t st);

// done: when the fused kernel takes the call, the device address of the word it writes its epoch to when every
// output is out (*epoch_out: that epoch).
// norm_src (the ffn_norm in the hook): the call's input rows are these residual rows (device memory), normalised
// first: inside the fused kernel for short calls, else by trx_k_ffn_norm into d_normed; normed_out (optional)
// receives the normalised rows.
static int launch_layer(tr_gpu_moe *m, int64_t layer, const float *d_normed, int64_t n_tok, float *d_x,
                        const tr_gpu_moe_outputs *out, cudaStream_t st, int first = 0, int last = 3,
                        uint32_t *done = nullptr, uint32_t *epoch_out = nullptr, const float *norm_src = nullptr,
                        float *normed_out = nullptr) {
    const tr_gpu_moe_config &c = m->cfg;
    if (layer < 0 || layer >= c.n_layers || !m->layer_set[(size_t)layer]) {
        set_err("layer %lld is not set", (long long)layer);
        return -1;
    }
    if (n_tok < 1 || n_tok > c.max_tokens || d_normed == nullptr || d_x == nullptr) {
        set_err("bad token count %lld (max %lld) or input", (long long)n_tok, (long long)c.max_tokens);
        return -1;
    }
    if (first < 0 || last > 3 || first > last) {
        set_err("bad part range %d..%d", first, last);
        return -1;
    }
    TrxLayer L = m->layers[(size_t)layer];
    TrxShape S{(int)c.n_expert, (int)c.n_used, (int)c.n_embd, (int)c.n_ff, (int)c.norm_topk, 0};
    if (norm_src) {
        if (m->norm_w == nullptr || !m->norm_set[(size_t)layer]) {
            set_err("layer %lld has no ffn_norm weight (tr_gpu_moe_set_ffn_norm)", (long long)layer);
            return -1;
        }
        L.norm_w = m->norm_w + layer * c.n_embd;
        L.norm_eps = m->norm_eps[(size_t)layer];
    }
    TrxWork w = m->work;
    w.trace = m->trace;
    if (out) {
        w.out_logits = out->logits;
        w.out_sel_id = out->sel_id;
        w.out_sel_w = out->sel_w;
        w.out_offsets = out->offsets;
        w.out_place = out->place;
    }
    if ((w.out_sel_id == nullptr) != (w.out_sel_w == nullptr)) {
        set_err("sel_id and sel_w outputs go together");
        return -1;
    }
    const int T = (int)n_tok, E = S.E, R = T * S.k;
    tr_gpu_moe::EvSet *es = nullptr;
    if (m->prof && first == 0 && last == 3 && (es = prof_slot(m)) == nullptr) return -1;
    // zone z's kernels run between events z and z + 1; an unused zone's two events coincide
    auto mark = [&](int z) {
        if (es) cudaEventRecord(es->ev[z], st);
    };
    if (es) {
        for (int z = 0; z < TRMOE_ZONES; z++) es->used[z] = true;
        es->used[2] = c.down_type == TRX_Q4_K;
    }
    int sg = 0, sd = 0;
    const bool fused = first == 0 && last == 3 && !(m->pf_ok && m->pf_min > 0 && T >= m->pf_min) && m->fused_ok &&
                       T <= TRX_ROUTE_FUSED_MAX && E + T <= m->grid_fused && !es && fused_stages(m, T, &sg, &sd);
    if (norm_src) {
        // short fused calls normalise inside the kernel when the rows fit the stage area beside the router's staging
        const bool inside =
            fused && T <= TRX_FU_LOCAL_PREP && ((uintptr_t)norm_src & 15) == 0 &&
            trx_fu_norm_off(T, S.H, E) + (size_t)T * S.H * 4 <=
                trx_fused_layout(c.gate_type, c.down_type, S.H, S.F, T, S.k, sg, sd, E, m->grid_fused).bars;
        if (inside) {
            S.norm_in = 1;
            d_normed = norm_src;
            w.out_normed = normed_out;
        } else {
            float *nb = normed_out ? normed_out : m->d_normed;
            if (launch_ffn_norm(m, layer, norm_src, n_tok, nb, st) != 0) return -1;
            d_normed = nb;
        }
    }
    if (first == 0 && last == 3 && m->pf_ok && m->pf_min > 0 && T >= m->pf_min && !es)
        return launch_prefill(m, L, S, w, d_normed, T, d_x, out ? out->ffn_out : nullptr, st);
    if (fused) {
        float *ffn = out ? out->ffn_out : nullptr;
        uint32_t epoch = ++m->epoch & 0x7fffffffu;
        if (epoch == 0) epoch = ++m->epoch & 0x7fffffffu; // 0 is the completion word's initial value
        w.host_done = done;
        if (epoch_out) *epoch_out = epoch;
        return launch_fused(m, L, S, d_normed, T, w, d_x, ffn, epoch, sg, sd, st, "fused layer launch");
    }
    mark(0);
    if (first <= 0 && 0 <= last) {
        const bool fused = T <= TRX_ROUTE_FUSED_MAX;
        const size_t smem_router = (size_t)(1 + std::min(T, TRX_TOK_STAGE)) * S.H * 4;
        if (fused) {
            trx_k_router<<<(unsigned)(E + T), 256, smem_router, st>>>(L, S, d_normed, T, w, 1);
        } else {
            launch_router_many(L, S, d_normed, T, w, st);
            trx_k_prep_tokens<<<(unsigned)T, 256, 0, st>>>(L, S, d_normed, w);
            trx_k_route<<<(unsigned)((T + 7) / 8), 256, 0, st>>>(S, T, w);
            trx_k_sort<<<1, 1024, 0, st>>>(S, T, w);
        }
    }
    mark(1);
    if (first <= 1 && 1 <= last) gateup_fn(c.gate_type, c.down_type)<<<(unsigned)m->grid_gu, 256, m->smem_gu, st>>>(L, S, w);
    mark(2);
    if (first <= 2 && 2 <= last && c.down_type == TRX_Q4_K) {
        const int warps = R * (S.F / 256);
        trx_k_prep<<<(unsigned)((warps + 7) / 8), 256, 0, st>>>(S, R, w);
    }
    mark(3);
    if (first <= 3 && 3 <= last) {
        float *ffn = out ? out->ffn_out : nullptr;
        down_fn(c.down_type)<<<(unsigned)m->grid_dn, 256, m->smem_dn, st>>>(L, S, w, d_x, T, ffn);
    }
    mark(4);
    return ck(cudaGetLastError(), "launch") ? 0 : -1;
}

extern "C" int tr_gpu_moe_set_prefill(tr_gpu_moe *m, int64_t min_tokens) {
    g_err.clear();
    if (m == nullptr || min_tokens < 0) {
        set_err("bad arguments to tr_gpu_moe_set_prefill");
        return -1;
    }
    if (!m->pf_ok) {
        if (min_tokens == 0) return 0;
        set_err("this context has no tensor-core road (it needs Q8_0 gate/up and down weights)");
        return -1;
    }
    m->pf_min = min_tokens;
    return 0;
}

extern "C" int tr_gpu_moe_layer_dev(tr_gpu_moe *m, int64_t layer, const float *d_normed, int64_t n_tok,
                                    float *d_x_inout, const tr_gpu_moe_outputs *out, void *stream) {
    g_err.clear();
    if (m == nullptr) {
        set_err("no context");
        return -1;
    }
    if (!ck(cudaSetDevice(m->device), "cudaSetDevice")) return -1;
    cudaStream_t st = stream ? (cudaStream_t)stream : m->stream;
    return launch_layer(m, layer, d_normed, n_tok, d_x_inout, out, st);
}

extern "C" int tr_gpu_moe_layer_part(tr_gpu_moe *m, int64_t layer, int part, const float *d_normed, int64_t n_tok,
                                     float *d_x_inout, const tr_gpu_moe_outputs *out, void *stream) {
    g_err.clear();
    if (m == nullptr) {
        set_err("no context");
        return -1;
    }
    if (!ck(cudaSetDevice(m->device), "cudaSetDevice")) return -1;
    cudaStream_t st = stream ? (cudaStream_t)stream : m->stream;
    return launch_layer(m, layer, d_normed, n_tok, d_x_inout, out, st, part, part);
}

// normed = ffn_norm(x) of layer `layer` for n_tok rows (x: device memory, or pinned host memory mapped in)
static int launch_ffn_norm(tr_gpu_moe *m, int64_t layer, const float *x, int64_t n_tok, float *normed, cudaStream_t st) {
    if (layer < 0 || layer >= m->cfg.n_layers || m->norm_w == nullptr || !m->norm_set[(size_t)layer]) {
        set_err("layer %lld has no ffn_norm weight (tr_gpu_moe_set_ffn_norm)", (long long)layer);
        return -1;
    }
    const int H = (int)m->cfg.n_embd;
    trx_k_ffn_norm<<<(unsigned)n_tok, 128, (size_t)H * 4, st>>>(x, m->norm_w + layer * H, m->norm_eps[(size_t)layer], H,
                                                                normed);
    return ck(cudaGetLastError(), "ffn_norm launch") ? 0 : -1;
}

// The host-pointer calls. normed == NULL: the layer's ffn_norm of x first (tr_gpu_moe_ffn).
static int host_layer(tr_gpu_moe *m, int64_t layer, const float *normed, int64_t n_tok, float *x_inout,
                      float *normed_out, int64_t *sel_id_out, float *sel_w_out) {
    if (n_tok < 1 || n_tok > m->cfg.max_tokens) {
        set_err("bad token count %lld (max %lld)", (long long)n_tok, (long long)m->cfg.max_tokens);
        return -1;
    }
    if (!ck(cudaSetDevice(m->device), "cudaSetDevice")) return -1;
    const bool norm = normed == nullptr;
    const size_t xb = (size_t)(n_tok * m->cfg.n_embd) * 4;
    const int64_t R = n_tok * m->cfg.n_used;
    cudaStream_t st = m->stream;
    // Short calls on pinned x (page-locked, mapped: cudaHostAlloc, cudaHostRegister, torch pin_memory): the kernels
    // read (and the layer writes) x in place through its device mapping, and the layer posts its epoch to a pinned
    // word once every output is out; the host polls that word instead of copying x back and synchronising the stream.
    cudaPointerAttributes pa{};
    if (m->h_done && sel_id_out == nullptr && sel_w_out == nullptr && normed_out == nullptr &&
        n_tok <= TRX_HOST_ZC_MAX && takes_fused(m, (int)n_tok) && cudaPointerGetAttributes(&pa, x_inout) == cudaSuccess &&
        pa.type == cudaMemoryTypeHost && pa.devicePointer != nullptr) {
        uint32_t epoch = 0;
        float *xd = (float *)pa.devicePointer;
        // with the ffn_norm, the norm reads a device copy of x (one copy-engine transfer beats reads over the link)
        const bool in = norm ? ck(cudaMemcpyAsync(m->d_x, x_inout, xb, cudaMemcpyHostToDevice, st), "copy x")
                             : ck(cudaMemcpyAsync(m->d_normed, normed, xb, cudaMemcpyHostToDevice, st), "copy normed");
        if (!in || launch_layer(m, layer, m->d_normed, n_tok, xd, nullptr, st, 0, 3, m->d_done, &epoch,
                                norm ? m->d_x : nullptr) != 0)
            return -1;
        const volatile uint32_t *word = m->h_done;
        const auto t0 = std::chrono::steady_clock::now();
        for (unsigned spins = 1;; spins++) {
            const uint32_t v = *word;
            if (v == epoch) return 0;
            if (v == (epoch | 0x80000000u)) break; // the kernel gave up on a bounded wait
            if ((spins & 1023) == 0) {
                const double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
                if (dt > 60.0) {
                    set_err("the GPU did not finish within 60 s");
                    return -1;
                }
                if (dt > 0.002) std::this_thread::sleep_for(std::chrono::microseconds(20));
                const cudaError_t e = cudaStreamQuery(st); // a launch or device error ends the wait too
                if (e != cudaSuccess && e != cudaErrorNotReady) {
                    ck(e, "cudaStreamQuery");
                    return -1;
                }
                if (e == cudaSuccess && *word != epoch) break; // finished without posting: the error road
            }
        }
        stream_wait(st);
        reset_counters(m, st);
        int32_t flag = 0;
        cudaMemcpy(&flag, m->work.err, 4, cudaMemcpyDeviceToHost);
        set_err("a kernel gave up on a bounded wait (device error flag %d)", flag);
        return -1;
    }
    cudaGetLastError(); // a pointer the runtime does not know (pageable memory) is not an error here
    tr_gpu_moe_outputs out{};
    const bool sel = sel_id_out != nullptr || sel_w_out != nullptr;
    if (sel) {
        out.sel_id = m->d_sel_id;
        out.sel_w = m->d_sel_w;
    }
    // (with the ffn_norm the normalised rows go to a buffer of their own: the layer updates d_x while reading them)
    float *nb = normed_out ? m->d_normed : nullptr;
    bool ok = ck(cudaMemcpyAsync(m->d_x, x_inout, xb, cudaMemcpyHostToDevice, st), "copy x") &&
              (norm || ck(cudaMemcpyAsync(m->d_normed, normed, xb, cudaMemcpyHostToDevice, st), "copy normed")) &&
              launch_layer(m, layer, m->d_normed, n_tok, m->d_x, sel ? &out : nullptr, st, 0, 3, nullptr, nullptr,
                           norm ? m->d_x : nullptr, nb) == 0 &&
              ck(cudaMemcpyAsync(x_inout, m->d_x, xb, cudaMemcpyDeviceToHost, st), "copy x back");
    if (ok && normed_out)
        ok = ck(cudaMemcpyAsync(normed_out, m->d_normed, xb, cudaMemcpyDeviceToHost, st), "copy normed out");
    if (ok && sel_id_out)
        ok = ck(cudaMemcpyAsync(sel_id_out, m->d_sel_id, (size_t)R * 8, cudaMemcpyDeviceToHost, st), "copy sel_id");
    if (ok && sel_w_out)
        ok = ck(cudaMemcpyAsync(sel_w_out, m->d_sel_w, (size_t)R * 4, cudaMemcpyDeviceToHost, st), "copy sel_w");
    int32_t flag = 0;
    if (ok) ok = ck(cudaMemcpyAsync(&flag, m->work.err, 4, cudaMemcpyDeviceToHost, st), "copy error flag");
    if (ok) ok = stream_wait(st);
    if (ok && flag != 0) {
        reset_counters(m, st);
        set_err("a kernel gave up on a bounded wait (device error flag %d)", flag);
        ok = false;
    }
    return ok ? 0 : -1;
}

extern "C" int tr_gpu_moe_layer(tr_gpu_moe *m, int64_t layer, const float *normed, int64_t n_tok, float *x_inout,
                                int64_t *sel_id_out, float *sel_w_out) {
    g_err.clear();
    if (m == nullptr || normed == nullptr || x_inout == nullptr) {
        set_err("bad arguments to tr_gpu_moe_layer");
        return -1;
    }
    return host_layer(m, layer, normed, n_tok, x_inout, nullptr, sel_id_out, sel_w_out);
}

// ---------------------------------------------------------------------------------------------
// ffn_norm fused into the hook (ffn_norm.cuh)

extern "C" int tr_gpu_moe_set_ffn_norm(tr_gpu_moe *m, int64_t layer, const float *weight, float eps, char *err,
                                       size_t err_len) {
    g_err.clear();
    if (m == nullptr || layer < 0 || layer >= m->cfg.n_layers || weight == nullptr || !(eps >= 0.0f)) {
        set_err("bad arguments to tr_gpu_moe_set_ffn_norm");
        put_err(err, err_len);
        return -1;
    }
    const int64_t H = m->cfg.n_embd;
    bool ok = ck(cudaSetDevice(m->device), "cudaSetDevice");
    if (ok && m->norm_w == nullptr) {
        ok = ck(cudaMalloc(&m->norm_w, (size_t)(m->cfg.n_layers * H) * 4), "cudaMalloc(ffn_norm)");
        if (ok) {
            m->norm_eps.assign((size_t)m->cfg.n_layers, 0.0f);
            m->norm_set.assign((size_t)m->cfg.n_layers, 0);
        }
    }
    if (ok) ok = ck(cudaMemcpyAsync(m->norm_w + layer * H, weight, (size_t)H * 4, cudaMemcpyHostToDevice, m->stream),
                    "copy ffn_norm") &&
                 stream_wait(m->stream);
    if (!ok) {
        put_err(err, err_len);
        return -1;
    }
    m->norm_eps[(size_t)layer] = eps;
    m->norm_set[(size_t)layer] = 1;
    return 0;
}

extern "C" int tr_gpu_moe_ffn(tr_gpu_moe *m, int64_t layer, int64_t n_tok, float *x_inout, float *normed_out,
                              int64_t *sel_id_out, float *sel_w_out) {
    g_err.clear();
    if (m == nullptr || x_inout == nullptr) {
        set_err("bad arguments to tr_gpu_moe_ffn");
        return -1;
    }
    return host_layer(m, layer, nullptr, n_tok, x_inout, normed_out, sel_id_out, sel_w_out);
}

extern "C" int tr_gpu_moe_ffn_dev(tr_gpu_moe *m, int64_t layer, int64_t n_tok, float *d_x_inout, float *d_normed_out,
                                  const tr_gpu_moe_outputs *out, void *stream) {
    g_err.clear();
    if (m == nullptr || d_x_inout == nullptr) {
        set_err("bad arguments to tr_gpu_moe_ffn_dev");
        return -1;
    }
    if (n_tok < 1 || n_tok > m->cfg.max_tokens) {
        set_err("bad token count %lld (max %lld)", (long long)n_tok, (long long)m->cfg.max_tokens);
        return -1;
    }
    if (!ck(cudaSetDevice(m->device), "cudaSetDevice")) return -1;
    cudaStream_t st = stream ? (cudaStream_t)stream : m->stream;
    return launch_layer(m, layer, m->d_normed, n_tok, d_x_inout, out, st, 0, 3, nullptr, nullptr, d_x_inout,
                        d_normed_out);
}

// ---------------------------------------------------------------------------------------------
// the model loader: an OLMoE GGUF file straight into the context's resident layout (no expert store)

namespace {

// the MoE block's tensors of one layer (src/models/olmoe.c:605-641, 901-906)
struct GgufLayer {
    const TrxGgufTensor *router, *norm, *gate, *up, *down;
};

// a tensor of the given ggml dimensions (olmoe.c's check_shape / find_experts): NULL with the reason in err
const TrxGgufTensor *gguf_need(const TrxGguf &g, const std::string &name, uint32_t n_dims, uint64_t ne0, uint64_t ne1,
                               uint64_t ne2, std::string &err) {
    const TrxGgufTensor *t = g.tensor(name);
    if (t == nullptr) {
        err = "missing tensor '" + name + "'";
        return nullptr;
    }
    const uint64_t want[3] = {ne0, ne1, ne2};
    bool ok = t->n_dims == n_dims;
    for (uint32_t d = 0; ok && d < n_dims; d++) ok = t->ne[d] == want[d];
    if (!ok) {
        err = "tensor '" + name + "' has shape [";
        for (uint32_t d = 0; d < t->n_dims; d++) err += (d ? ", " : "") + std::to_string(t->ne[d]);
        err += "], expected [";
        for (uint32_t d = 0; d < n_dims; d++) err += (d ? ", " : "") + std::to_string(want[d]);
        err += "]";
        return nullptr;
    }
    return t;
}

// every value of an F32 tensor a bfloat16 (its low 16 bits zero), as Trochilus's tr_f32_to_bf16_exact asks
// (src/kernels/kernels.h:82-85) before it keeps an F32 router as BF16
bool gguf_bf16_exact(const TrxGgufTensor &t, const uint8_t *p) {
    for (uint64_t i = 0; i < t.n_bytes / 4; i++) {
        uint32_t v;
        memcpy(&v, p + 4 * i, 4);
        if (v & 0xffffu) return false;
    }
    return true;
}

// The file's MoE configuration (olmoe.c:541-575's metadata, the router, ffn_norm and expert tensors of every layer),
// with *eps its RMSNorm epsilon and layers[L] each layer's tensors. The context takes one gate/up type and one down
// type: a file whose layers differ is refused. The router type is BF16 when every layer's router is BF16 or an F32
// whose values are all bfloat16 (the reference keeps those as BF16, olmoe.c:391), else F32.
bool gguf_config(const TrxGguf &g, tr_gpu_moe_config &cfg, float &eps, std::vector<GgufLayer> &layers, std::string &err) {
    std::string arch;
    if (g.get_str("general.architecture", arch) && arch != "olmoe") {
        err = "general.architecture is '" + arch + "', not 'olmoe'";
        return false;
    }
    uint32_t nl = 0, H = 0, F = 0, E = 0, k = 0;
    const char *need[5] = {"olmoe.block_count", "olmoe.embedding_length", "olmoe.feed_forward_length",
                           "olmoe.expert_count", "olmoe.expert_used_count"};
    uint32_t *dst[5] = {&nl, &H, &F, &E, &k};
    for (int i = 0; i < 5; i++)
        if (!g.get_u32(need[i], *dst[i])) {
            err = std::string("missing metadata key '") + need[i] + "'";
            return false;
        }
    if (!g.get_f32("olmoe.attention.layer_norm_rms_epsilon", eps)) {
        err = "missing metadata key 'olmoe.attention.layer_norm_rms_epsilon'";
        return false;
    }
    bool norm_topk = false;
    g.get_bool("olmoe.expert_weights_norm", norm_topk);
    if (nl == 0 || H == 0 || F == 0 || E == 0 || k == 0) {
        err = "invalid (zero) hyperparameter in metadata";
        return false;
    }
    if (k > E) {
        err = "olmoe.expert_used_count exceeds olmoe.expert_count";
        return false;
    }
    layers.assign(nl, GgufLayer{});
    bool all_bf16 = true;
    for (uint32_t L = 0; L < nl; L++) {
        const std::string b = "blk." + std::to_string(L) + ".";
        GgufLayer &y = layers[L];
        if (!(y.router = gguf_need(g, b + "ffn_gate_inp.weight", 2, H, E, 0, err)) ||
            !(y.norm = gguf_need(g, b + "ffn_norm.weight", 1, H, 0, 0, err)) ||
            !(y.gate = gguf_need(g, b + "ffn_gate_exps.weight", 3, H, F, E, err)) ||
            !(y.up = gguf_need(g, b + "ffn_up_exps.weight", 3, H, F, E, err)) ||
            !(y.down = gguf_need(g, b + "ffn_down_exps.weight", 3, F, H, E, err)))
            return false;
        if (y.router->type != TRX_F32 && y.router->type != TRX_BF16) {
            err = b + "ffn_gate_inp.weight has type " + std::to_string(y.router->type) + " (F32 or BF16 taken)";
            return false;
        }
        if (y.norm->type != TRX_F32) {
            err = b + "ffn_norm.weight is not F32";
            return false;
        }
        if (y.up->type != y.gate->type || y.gate->type != layers[0].gate->type || y.down->type != layers[0].down->type) {
            err = "layer " + std::to_string(L) + "'s expert types differ from layer 0's (gate/up " +
                  std::to_string(layers[0].gate->type) + ", down " + std::to_string(layers[0].down->type) +
                  "): a context takes one gate/up type and one down type";
            return false;
        }
        if (y.router->type == TRX_F32 && all_bf16) all_bf16 = gguf_bf16_exact(*y.router, g.bytes(*y.router));
    }
    cfg.n_layers = nl;
    cfg.n_expert = E;
    cfg.n_used = k;
    cfg.n_embd = H;
    cfg.n_ff = F;
    cfg.norm_topk = norm_topk ? 1 : 0;
    cfg.router_type = all_bf16 ? TRX_BF16 : TRX_F32;
    cfg.gate_type = (int32_t)layers[0].gate->type;
    cfg.down_type = (int32_t)layers[0].down->type;
    return true;
}

} // namespace

extern "C" int tr_gpu_moe_config_from_gguf(const char *path, tr_gpu_moe_config *cfg, float *rms_eps, char *err,
                                           size_t err_len) {
    g_err.clear();
    if (path == nullptr || cfg == nullptr) {
        set_err("bad arguments to tr_gpu_moe_config_from_gguf");
        put_err(err, err_len);
        return -1;
    }
    TrxGguf g;
    std::string e;
    tr_gpu_moe_config c = *cfg;
    float eps = 0.0f;
    std::vector<GgufLayer> layers;
    if (!g.open(path, e) || !gguf_config(g, c, eps, layers, e)) {
        set_err("%s", e.c_str());
        put_err(err, err_len);
        return -1;
    }
    *cfg = c;
    if (rms_eps) *rms_eps = eps;
    return 0;
}

extern "C" int tr_gpu_moe_load_gguf(tr_gpu_moe *m, const char *path, char *err, size_t err_len) {
    g_err.clear();
    if (m == nullptr || path == nullptr) {
        set_err("bad arguments to tr_gpu_moe_load_gguf");
        put_err(err, err_len);
        return -1;
    }
    TrxGguf g;
    std::string e;
    tr_gpu_moe_config f = m->cfg;
    float eps = 0.0f;
    std::vector<GgufLayer> layers;
    if (!g.open(path, e) || !gguf_config(g, f, eps, layers, e)) {
        set_err("%s", e.c_str());
        put_err(err, err_len);
        return -1;
    }
    const tr_gpu_moe_config &c = m->cfg;
    if (f.n_layers != c.n_layers || f.n_expert != c.n_expert || f.n_used != c.n_used || f.n_embd != c.n_embd ||
        f.n_ff != c.n_ff || f.norm_topk != c.norm_topk || f.gate_type != c.gate_type || f.down_type != c.down_type ||
        (f.router_type == TRX_F32 && c.router_type == TRX_BF16)) {
        set_err("the file's MoE configuration (layers %lld, experts %lld of %lld, %lldx%lld, norm_topk %d, router %d, "
                "gate/up %d, down %d) is not the context's (tr_gpu_moe_config_from_gguf gives it)",
                (long long)f.n_layers, (long long)f.n_used, (long long)f.n_expert, (long long)f.n_embd,
                (long long)f.n_ff, f.norm_topk, f.router_type, f.gate_type, f.down_type);
        put_err(err, err_len);
        return -1;
    }
    const int64_t E = c.n_expert, H = c.n_embd, F = c.n_ff;
    const int64_t gate_bytes = trx_row_bytes(c.gate_type, H) * F, down_bytes = trx_row_bytes(c.down_type, F) * H;
    std::vector<const void *> gp((size_t)E), up((size_t)E), dp((size_t)E);
    std::vector<uint16_t> r16;
    std::vector<float> r32;
    for (int64_t L = 0; L < c.n_layers; L++) {
        const GgufLayer &y = layers[(size_t)L];
        // the router in the context's type: as stored, narrowed (bfloat16-exact F32) or widened (BF16 into F32)
        const void *router = g.bytes(*y.router);
        const int64_t nr = E * H;
        if (y.router->type == TRX_F32 && c.router_type == TRX_BF16) {
            r16.resize((size_t)nr);
            for (int64_t i = 0; i < nr; i++) {
                uint32_t v;
                memcpy(&v, (const uint8_t *)router + 4 * i, 4);
                r16[(size_t)i] = (uint16_t)(v >> 16);
            }
            router = r16.data();
        } else if (y.router->type == TRX_BF16 && c.router_type == TRX_F32) {
            r32.resize((size_t)nr);
            for (int64_t i = 0; i < nr; i++) {
                uint16_t v;
                memcpy(&v, (const uint8_t *)router + 2 * i, 2);
                const uint32_t w = (uint32_t)v << 16;
                memcpy(&r32[(size_t)i], &w, 4);
            }
            router = r32.data();
        }
        // expert e of a stacked tensor at byte e out row_bytes(in) (olmoe.c:466-472)
        for (int64_t x = 0; x < E; x++) {
            gp[(size_t)x] = g.bytes(*y.gate) + x * gate_bytes;
            up[(size_t)x] = g.bytes(*y.up) + x * gate_bytes;
            dp[(size_t)x] = g.bytes(*y.down) + x * down_bytes;
        }
        if (tr_gpu_moe_set_layer(m, L, router, nullptr, gp.data(), up.data(), dp.data(), err, err_len) != 0)
            return -1;
        float norm_host[8192];
        memcpy(norm_host, g.bytes(*y.norm), (size_t)H * 4); // (the mapping's bytes may be unaligned for floats)
        if (tr_gpu_moe_set_ffn_norm(m, L, norm_host, eps, err, err_len) != 0) return -1;
    }
    return 0;
}

// ---------------------------------------------------------------------------------------------
// expert parallelism (ep.cuh): pack, the experts of arriving rows, combine

extern "C" int tr_gpu_moe_ep_pack(tr_gpu_moe *m, const int64_t *d_sel_id, int64_t n_tok, int32_t n_ranks, int64_t cap,
                                  const float *d_normed, float *d_send_rows, int32_t *d_send_ids, int32_t *d_send_counts,
                                  int32_t *d_place, int32_t *d_scratch, void *stream) {
    g_err.clear();
    const int64_t R = n_tok * (m ? m->cfg.n_used : 0);
    if (m == nullptr || d_sel_id == nullptr || d_normed == nullptr || d_send_rows == nullptr || d_send_ids == nullptr ||
        d_send_counts == nullptr || d_place == nullptr || d_scratch == nullptr || n_tok < 1 || n_ranks < 1 ||
        n_ranks > 64 || m->cfg.n_expert % n_ranks != 0 || (cap != 0 && cap < R) || R > (1 << 24)) {
        set_err("bad arguments to tr_gpu_moe_ep_pack (ranks must divide the experts; cap 0 or at least n_tok x n_used)");
        return -1;
    }
    if (!ck(cudaSetDevice(m->device), "cudaSetDevice")) return -1;
    cudaStream_t st = stream ? (cudaStream_t)stream : m->stream;
    const int H = (int)m->cfg.n_embd;
    const int64_t div = m->cfg.n_expert / n_ranks;
    int32_t *offsets = d_scratch, *xmap = d_scratch + 72; // scratch: 72 + R int32
    if (cap > 0 && !ck(cudaMemsetAsync(d_send_ids, 0xff, (size_t)(n_ranks * cap) * 4, st), "clear ids")) return -1;
    trx_k_stable_sort<<<1, 1024, 0, st>>>(d_sel_id, nullptr, div, (int)R, n_ranks, offsets, d_place, xmap, d_send_counts);
    trx_k_gather_rows<<<(unsigned)R, 256, 0, st>>>(d_normed, xmap, offsets + n_ranks, (int)m->cfg.n_used, H, d_send_rows,
                                                   d_sel_id, d_send_ids, offsets, (int)cap, div, d_place);
    return ck(cudaGetLastError(), "ep pack launch") ? 0 : -1;
}

extern "C" int tr_gpu_moe_experts_dev(tr_gpu_moe *m, int64_t layer, const float *d_rows, const int32_t *d_ids,
                                      int64_t n_rows, float *d_out, void *stream) {
    g_err.clear();
    if (m == nullptr || layer < 0 || layer >= m->cfg.n_layers || !m->layer_set[(size_t)layer] || n_rows < 0 ||
        (n_rows > 0 && (d_rows == nullptr || d_ids == nullptr || d_out == nullptr))) {
        set_err("bad arguments to tr_gpu_moe_experts_dev (or the layer is not set)");
        return -1;
    }
    if (n_rows == 0) return 0;
    if (n_rows > (1 << 24)) {
        set_err("tr_gpu_moe_experts_dev: %lld rows is more than it takes", (long long)n_rows);
        return -1;
    }
    if (!ck(cudaSetDevice(m->device), "cudaSetDevice")) return -1;
    cudaStream_t st = stream ? (cudaStream_t)stream : m->stream;
    const tr_gpu_moe_config &c = m->cfg;
    const int64_t E = c.n_expert, H = c.n_embd, F = c.n_ff, n = n_rows, mx = std::max(H, F);
    // Up to TRX_ROUTE_FUSED_MAX rows, and no more than the context's max_tokens (its per-row work buffers): the fused
    // decode kernel with the routing given (row t to expert ids[t] alone, weight 1: its mix is the expert's row),
    // one launch
    int sg = 0, sd = 0;
    if (m->fused_ok && n <= TRX_ROUTE_FUSED_MAX && n <= c.max_tokens && n <= m->grid_fused &&
        fused_stages(m, (int)n, &sg, &sd, 1)) {
        const TrxLayer &L = m->layers[(size_t)layer];
        const TrxShape S{(int)E, 1, (int)H, (int)F, 0, 0, 1};
        TrxWork w = m->work;
        w.ext_ids = d_ids;
        const uint32_t epoch = (++m->epoch & 0x7fffffffu) | 1u;
        return launch_fused(m, L, S, d_rows, (int)n, w, nullptr, d_out, epoch, sg, sd, st, "fused experts launch");
    }
    // scratch: sort (offsets, place, xmap), grouped rows, gate and up outputs, down output, prepared inputs
    const int64_t so = align_up((E + 8 + 2 * n) * 4, 256), xb = align_up(n * H * 4, 256), gb = align_up(n * F * 4, 256),
                  qb = align_up(n * mx * 4, 256), bfb = align_up(n * (mx / 32) * 8, 256), scb = align_up(n * (mx / 256) * 8, 256),
                  need = so + 2 * xb + 2 * gb + qb + bfb + scb;
    if (need > m->ep_cap) {
        if (m->ep_buf) {
            if (!stream_wait(st)) return -1;
            cudaFree(m->ep_buf);
            m->ep_buf = nullptr;
            m->ep_cap = 0;
        }
        if (!ck(cudaMalloc(&m->ep_buf, (size_t)need), "cudaMalloc(expert scratch)")) return -1;
        m->ep_cap = need;
    }
    uint8_t *b = m->ep_buf;
    int32_t *offsets = (int32_t *)b, *place = offsets + E + 8, *xmap = place + n;
    float *xg = (float *)(b + so), *y = (float *)(b + so + xb), *g = (float *)(b + so + 2 * xb),
          *u = (float *)(b + so + 2 * xb + gb);
    uint32_t *dq = (uint32_t *)(b + so + 2 * xb + 2 * gb);
    double *dbf = (double *)(b + so + 2 * xb + 2 * gb + qb), *dsc = (double *)(b + so + 2 * xb + 2 * gb + qb + bfb);
    const uint8_t *const *tab = m->ep_tab + (size_t)layer * 3 * E;
    trx_k_stable_sort<<<1, 1024, 0, st>>>(nullptr, d_ids, 1, (int)n, (int)E, offsets, place, xmap, nullptr);
    trx_k_gather_rows<<<(unsigned)n, 256, 0, st>>>(d_rows, xmap, offsets + E, 1, (int)H, xg, nullptr, nullptr, nullptr,
                                                   0, 1, nullptr);
    bool ok = trx_kapi_grouped(c.gate_type, F, H, tab, offsets, (int)E, (int)n, xg, dq, dbf, dsc, g, st) &&
              trx_kapi_grouped(c.gate_type, F, H, tab + E, offsets, (int)E, (int)n, xg, dq, dbf, dsc, u, st) &&
              trx_kapi_swiglu(g, u, n * F, st) &&
              trx_kapi_grouped(c.down_type, H, F, tab + 2 * E, offsets, (int)E, (int)n, g, dq, dbf, dsc, y, st);
    if (!ok) {
        set_err("tr_gpu_moe_experts_dev: launch failed");
        return -1;
    }
    trx_k_scatter_rows<<<(unsigned)n, 256, 0, st>>>(y, xmap, offsets + E, (int)H, d_out);
    return ck(cudaGetLastError(), "experts launch") ? 0 : -1;
}

extern "C" int tr_gpu_moe_ep_combine(tr_gpu_moe *m, const float *d_sel_w, const int32_t *d_place, const float *d_back,
                                     int64_t n_tok, float *d_x, float *d_ffn_out, void *stream) {
    g_err.clear();
    if (m == nullptr || d_sel_w == nullptr || d_place == nullptr || d_back == nullptr || d_x == nullptr || n_tok < 1) {
        set_err("bad arguments to tr_gpu_moe_ep_combine");
        return -1;
    }
    if (!ck(cudaSetDevice(m->device), "cudaSetDevice")) return -1;
    cudaStream_t st = stream ? (cudaStream_t)stream : m->stream;
    const int64_t total = n_tok * m->cfg.n_embd;
    trx_k_pf_combine<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(d_sel_w, d_place, d_back, (int)n_tok,
                                                                     (int)m->cfg.n_used, (int)m->cfg.n_embd, d_x, d_ffn_out);
    return ck(cudaGetLastError(), "ep combine launch") ? 0 : -1;
}

// ---------------------------------------------------------------------------------------------
// expert parallelism over peer memory (ep.cuh): the exchange region, the peers' regions, dispatch / experts / combine

extern "C" int tr_gpu_moe_ep_peer_region(tr_gpu_moe *m, int32_t n_ranks, int32_t rank, int64_t cap, void *ipc_handle_out) {
    g_err.clear();
    if (m == nullptr || n_ranks < 1 || n_ranks > TRX_EP_MAX_RANKS || rank < 0 || rank >= n_ranks || cap < 1 ||
        cap > 256 || ipc_handle_out == nullptr || m->cfg.n_expert % n_ranks != 0 || m->epp_region != nullptr) {
        set_err("bad arguments to tr_gpu_moe_ep_peer_region (or the region exists)");
        return -1;
    }
    if (!ck(cudaSetDevice(m->device), "cudaSetDevice")) return -1;
    size_t ids, rows, back, total;
    trx_ep_layout(n_ranks, (int)cap, (int)m->cfg.n_embd, ids, rows, back, total);
    cudaIpcMemHandle_t h;
    if (!ck(cudaMalloc(&m->epp_region, total), "cudaMalloc(exchange region)") ||
        !ck(cudaMemset(m->epp_region, 0, total), "cudaMemset(exchange region)") ||
        !ck(cudaIpcGetMemHandle(&h, m->epp_region), "cudaIpcGetMemHandle")) {
        if (m->epp_region) cudaFree(m->epp_region);
        m->epp_region = nullptr;
        return -1;
    }
    memcpy(ipc_handle_out, &h, sizeof h);
    m->epp_n = n_ranks;
    m->epp_rank = rank;
    m->epp_cap = cap;
    return 0;
}

extern "C" int tr_gpu_moe_ep_peer_open(tr_gpu_moe *m, const void *ipc_handles) {
    g_err.clear();
    if (m == nullptr || m->epp_region == nullptr || ipc_handles == nullptr || m->epp_dev != nullptr) {
        set_err("bad arguments to tr_gpu_moe_ep_peer_open (no region, or already open)");
        return -1;
    }
    if (!ck(cudaSetDevice(m->device), "cudaSetDevice")) return -1;
    TrxEpPeers P{};
    P.n = m->epp_n;
    P.rank = m->epp_rank;
    P.cap = (int)m->epp_cap;
    P.H = (int)m->cfg.n_embd;
    size_t total;
    trx_ep_layout(P.n, P.cap, P.H, P.off_ids, P.off_rows, P.off_back, total);
    m->epp_opened.assign((size_t)P.n, nullptr);
    for (int r = 0; r < P.n; r++) {
        if (r == P.rank) {
            P.base[r] = m->epp_region;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, (const uint8_t *)ipc_handles + (size_t)r * sizeof h, sizeof h);
        void *p = nullptr;
        if (!ck(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle")) return -1;
        m->epp_opened[(size_t)r] = (uint8_t *)p;
        P.base[r] = (uint8_t *)p;
    }
    if (!ck(cudaMalloc(&m->epp_dev, sizeof P), "cudaMalloc(peer table)") ||
        !ck(cudaMemcpy(m->epp_dev, &P, sizeof P, cudaMemcpyHostToDevice), "copy peer table"))
        return -1;
    return 0;
}

extern "C" int tr_gpu_moe_ep_dispatch(tr_gpu_moe *m, const int64_t *d_sel_id, int64_t n_tok, const float *d_normed,
                                      int32_t *d_place, void *stream) {
    g_err.clear();
    if (m == nullptr || m->epp_dev == nullptr || d_sel_id == nullptr || d_normed == nullptr || d_place == nullptr ||
        n_tok < 1 || n_tok * m->cfg.n_used > m->epp_cap || n_tok * m->cfg.n_used > 256) {
        set_err("bad arguments to tr_gpu_moe_ep_dispatch (no open exchange, or n_tok x n_used above its cap)");
        return -1;
    }
    if (!ck(cudaSetDevice(m->device), "cudaSetDevice")) return -1;
    cudaStream_t st = stream ? (cudaStream_t)stream : m->stream;
    trx_k_ep_dispatch<<<1, 256, 0, st>>>(d_sel_id, (int)n_tok, (int)m->cfg.n_used, (int)(m->cfg.n_expert / m->epp_n),
                                        d_normed, m->epp_dev, d_place);
    return ck(cudaGetLastError(), "ep dispatch launch") ? 0 : -1;
}

extern "C" int tr_gpu_moe_ep_experts(tr_gpu_moe *m, int64_t layer, void *stream) {
    g_err.clear();
    if (m == nullptr || m->epp_dev == nullptr || layer < 0 || layer >= m->cfg.n_layers || !m->layer_set[(size_t)layer]) {
        set_err("bad arguments to tr_gpu_moe_ep_experts (no open exchange, or the layer is not set)");
        return -1;
    }
    if (!ck(cudaSetDevice(m->device), "cudaSetDevice")) return -1;
    cudaStream_t st = stream ? (cudaStream_t)stream : m->stream;
    const tr_gpu_moe_config &c = m->cfg;
    const int64_t n = (int64_t)m->epp_n * m->epp_cap, E = c.n_expert, H = c.n_embd, F = c.n_ff;
    int sg = 0, sd = 0;
    if (!(m->fused_ok && n <= TRX_ROUTE_FUSED_MAX && n <= c.max_tokens && n <= m->grid_fused &&
          fused_stages(m, (int)n, &sg, &sd, 1))) {
        set_err("tr_gpu_moe_ep_experts: n_ranks x cap = %lld rows do not fit the fused kernel (at most %d, and the "
                "context's max_tokens)", (long long)n, TRX_ROUTE_FUSED_MAX);
        return -1;
    }
    size_t ids, rows, back, total;
    trx_ep_layout(m->epp_n, (int)m->epp_cap, (int)H, ids, rows, back, total);
    const TrxLayer &L = m->layers[(size_t)layer];
    const TrxShape S{(int)E, 1, (int)H, (int)F, 0, 0, 1};
    TrxWork w = m->work;
    w.ext_ids = (const int32_t *)(m->epp_region + ids);
    w.ep = m->epp_dev;
    const uint32_t epoch = (++m->epoch & 0x7fffffffu) | 1u;
    return launch_fused(m, L, S, (const float *)(m->epp_region + rows), (int)n, w, nullptr, nullptr, epoch, sg, sd, st,
                        "ep experts launch");
}

extern "C" int tr_gpu_moe_ep_peer_combine(tr_gpu_moe *m, const float *d_sel_w, const int32_t *d_place, int64_t n_tok,
                                          float *d_x, float *d_ffn_out, void *stream) {
    g_err.clear();
    if (m == nullptr || m->epp_dev == nullptr || d_sel_w == nullptr || d_place == nullptr || d_x == nullptr || n_tok < 1) {
        set_err("bad arguments to tr_gpu_moe_ep_peer_combine");
        return -1;
    }
    if (!ck(cudaSetDevice(m->device), "cudaSetDevice")) return -1;
    cudaStream_t st = stream ? (cudaStream_t)stream : m->stream;
    const int64_t total = n_tok * m->cfg.n_embd;
    trx_k_ep_peer_combine<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(d_sel_w, d_place, m->epp_dev, (int)n_tok,
                                                                          (int)m->cfg.n_used, d_x, d_ffn_out, m->work.err);
    return ck(cudaGetLastError(), "ep combine launch") ? 0 : -1;
}

// ---------------------------------------------------------------------------------------------
// decode attention (attention.cuh): Trochilus's GPU attention backend (src/backend/gpu_attn.h) on the B200

struct tr_gpu {
    int device = 0;
    char name[256] = {0};
};

struct tr_gpu_attn {
    tr_gpu *g = nullptr;
    int64_t n_layers = 0, n_head = 0, n_ctx = 0, s_stride = 0;
    float *keys = nullptr, *values = nullptr; // [layer][head][pos][128]
    float *scores = nullptr;                  // [head][s_stride]
    float *io = nullptr;                      // a call's rows: q, k, v of a decode, or a write's chunk; then out
    int32_t *err = nullptr;
    cudaStream_t st = nullptr, warm_st = nullptr;
    uint32_t *h_stop = nullptr, *d_stop = nullptr; // the warm-up kernel's stop word (mapped pinned)
};

namespace {

constexpr int64_t kAttnWriteChunk = 256; // tokens a write moves per copy
constexpr uint64_t kAttnReserve = (uint64_t)512 << 20;
constexpr uint64_t kAttnWarmMaxNs = 200000000;

int64_t attn_s_stride(int64_t n_ctx) { return (n_ctx + TRX_ATTN_CHUNK - 1) / TRX_ATTN_CHUNK * TRX_ATTN_CHUNK; }

// a failed call's stream and error word: whatever was in flight finishes, the word goes back to 0
bool attn_fail(tr_gpu_attn *a, const char *what) {
    cudaStreamSynchronize(a->st);
    cudaMemsetAsync(a->err, 0, 4, a->st);
    cudaStreamSynchronize(a->st);
    set_err("%s", what);
    return false;
}

} // namespace

extern "C" tr_gpu *tr_gpu_open(char *err, size_t err_len) {
    g_err.clear();
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
        cudaGetLastError();
        set_err("no CUDA device (or no driver)");
        put_err(err, err_len);
        return nullptr;
    }
    for (int d = 0; d < n; d++) {
        cudaDeviceProp p;
        if (cudaGetDeviceProperties(&p, d) != cudaSuccess || p.major != 10 || p.minor != 0) continue;
        tr_gpu *g = new tr_gpu;
        g->device = d;
        snprintf(g->name, sizeof g->name, "%s", p.name);
        return g;
    }
    set_err("no device of compute capability 10.0 (the library's kernels are built for sm_100a)");
    put_err(err, err_len);
    return nullptr;
}

extern "C" void tr_gpu_close(tr_gpu *g) { delete g; }

extern "C" const char *tr_gpu_name(const tr_gpu *g) { return g ? g->name : ""; }

extern "C" uint64_t tr_gpu_attn_bytes(int64_t n_layers, int64_t n_head, int64_t head_dim, int64_t n_ctx) {
    if (n_layers < 1 || n_head < 1 || head_dim < 1 || n_ctx < 1) return 0;
    const uint64_t cache = 2ull * (uint64_t)n_layers * (uint64_t)n_head * (uint64_t)n_ctx * (uint64_t)head_dim * 4;
    const uint64_t scores = (uint64_t)n_head * (uint64_t)attn_s_stride(n_ctx) * 4;
    const uint64_t io = (uint64_t)std::max<int64_t>(4, 2 * kAttnWriteChunk) * (uint64_t)(n_head * head_dim) * 4;
    return cache + scores + io + 256;
}

extern "C" void tr_gpu_attn_free(tr_gpu_attn *a) {
    if (a == nullptr) return;
    cudaSetDevice(a->g->device);
    if (a->h_stop) *(volatile uint32_t *)a->h_stop = 1u; // a warm-up still running stops
    if (a->warm_st) cudaStreamSynchronize(a->warm_st);
    if (a->st) cudaStreamSynchronize(a->st);
    cudaFree(a->keys);
    cudaFree(a->values);
    cudaFree(a->scores);
    cudaFree(a->io);
    cudaFree(a->err);
    if (a->h_stop) cudaFreeHost(a->h_stop);
    if (a->st) cudaStreamDestroy(a->st);
    if (a->warm_st) cudaStreamDestroy(a->warm_st);
    delete a;
}

extern "C" tr_gpu_attn *tr_gpu_attn_create(tr_gpu *g, int64_t n_layers, int64_t n_head, int64_t head_dim,
                                           int64_t n_ctx, char *err, size_t err_len) {
    g_err.clear();
    if (head_dim != TRX_ATTN_HD) {
        set_err("head_dim %lld not supported (128)", (long long)head_dim);
        put_err(err, err_len);
        return nullptr;
    }
    if (n_layers < 1 || n_head < 1 || n_head > 65535 || n_ctx < 1 || n_ctx > (1 << 24)) {
        set_err("bad shape (layers %lld, heads %lld, context %lld)", (long long)n_layers, (long long)n_head,
                (long long)n_ctx);
        put_err(err, err_len);
        return nullptr;
    }
    if (g == nullptr) {
        set_err("no device (tr_gpu_open)");
        put_err(err, err_len);
        return nullptr;
    }
    if (!ck(cudaSetDevice(g->device), "cudaSetDevice")) {
        put_err(err, err_len);
        return nullptr;
    }
    size_t free_b = 0, total_b = 0;
    const uint64_t need = tr_gpu_attn_bytes(n_layers, n_head, head_dim, n_ctx);
    if (!ck(cudaMemGetInfo(&free_b, &total_b), "cudaMemGetInfo")) {
        put_err(err, err_len);
        return nullptr;
    }
    if ((uint64_t)free_b < need + kAttnReserve) {
        set_err("the cache needs %llu bytes and %llu must stay free; %llu are", (unsigned long long)need,
                (unsigned long long)kAttnReserve, (unsigned long long)free_b);
        put_err(err, err_len);
        return nullptr;
    }
    tr_gpu_attn *a = new tr_gpu_attn;
    a->g = g;
    a->n_layers = n_layers;
    a->n_head = n_head;
    a->n_ctx = n_ctx;
    a->s_stride = attn_s_stride(n_ctx);
    const size_t cache = (size_t)n_layers * n_head * n_ctx * TRX_ATTN_HD * 4;
    const size_t io = (size_t)std::max<int64_t>(4, 2 * kAttnWriteChunk) * n_head * TRX_ATTN_HD * 4;
    bool ok = ck(cudaMalloc(&a->keys, cache), "cudaMalloc(keys)") &&
              ck(cudaMalloc(&a->values, cache), "cudaMalloc(values)") &&
              ck(cudaMalloc(&a->scores, (size_t)n_head * a->s_stride * 4), "cudaMalloc(scores)") &&
              ck(cudaMalloc(&a->io, io), "cudaMalloc(io)") && ck(cudaMalloc(&a->err, 4), "cudaMalloc(err)") &&
              ck(cudaMemset(a->err, 0, 4), "cudaMemset(err)") &&
              ck(cudaMemset(a->scores, 0, (size_t)n_head * a->s_stride * 4), "cudaMemset(scores)") &&
              ck(cudaStreamCreateWithFlags(&a->st, cudaStreamNonBlocking), "cudaStreamCreate") &&
              ck(cudaStreamCreateWithFlags(&a->warm_st, cudaStreamNonBlocking), "cudaStreamCreate") &&
              ck(cudaHostAlloc((void **)&a->h_stop, 4, cudaHostAllocMapped), "cudaHostAlloc(stop)") &&
              ck(cudaHostGetDevicePointer((void **)&a->d_stop, a->h_stop, 0), "cudaHostGetDevicePointer(stop)") &&
              ck(cudaFuncSetAttribute(trx_attn_values, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      TRX_ATTN_STAGES * TRX_ATTN_STAGE_BYTES),
                 "values kernel shared memory");
    if (!ok) {
        put_err(err, err_len);
        tr_gpu_attn_free(a);
        return nullptr;
    }
    *a->h_stop = 1u;
    return a;
}

extern "C" int tr_gpu_attn_write(tr_gpu_attn *a, int64_t layer, int64_t pos0, int64_t n_tok, const float *k,
                                 const float *v) {
    g_err.clear();
    if (a == nullptr || layer < 0 || layer >= a->n_layers || pos0 < 0 || n_tok < 0 || pos0 + n_tok > a->n_ctx ||
        (n_tok > 0 && (k == nullptr || v == nullptr))) {
        set_err("bad arguments to tr_gpu_attn_write (a range outside the cache)");
        return -1;
    }
    if (!ck(cudaSetDevice(a->g->device), "cudaSetDevice")) return -1;
    const int64_t row = a->n_head * TRX_ATTN_HD, lay = a->n_head * a->n_ctx * TRX_ATTN_HD;
    bool ok = true;
    for (int64_t i = 0; ok && i < n_tok; i += kAttnWriteChunk) {
        const int64_t n = std::min(kAttnWriteChunk, n_tok - i);
        float *sk = a->io, *sv = a->io + kAttnWriteChunk * row;
        const unsigned blocks = (unsigned)((n * a->n_head + 7) / 8);
        ok = ck(cudaMemcpyAsync(sk, k + i * row, (size_t)(n * row) * 4, cudaMemcpyHostToDevice, a->st), "copy k") &&
             ck(cudaMemcpyAsync(sv, v + i * row, (size_t)(n * row) * 4, cudaMemcpyHostToDevice, a->st), "copy v");
        if (ok) {
            trx_attn_store<<<blocks, 256, 0, a->st>>>(sk, (int)n, (int)a->n_head, pos0 + i, a->n_ctx, a->keys + layer * lay);
            trx_attn_store<<<blocks, 256, 0, a->st>>>(sv, (int)n, (int)a->n_head, pos0 + i, a->n_ctx,
                                                      a->values + layer * lay);
            ok = ck(cudaGetLastError(), "store kernel") && stream_wait(a->st); // (the staging is reused)
        }
    }
    return ok ? 0 : -1;
}

extern "C" int tr_gpu_attn_decode(tr_gpu_attn *a, int64_t layer, int64_t pos, const float *q, const float *k,
                                  const float *v, float scale, float *out) {
    g_err.clear();
    if (a == nullptr || layer < 0 || layer >= a->n_layers || pos < 0 || pos >= a->n_ctx || q == nullptr ||
        k == nullptr || v == nullptr || out == nullptr) {
        set_err("bad arguments to tr_gpu_attn_decode (pos outside the cache)");
        return -1;
    }
    *(volatile uint32_t *)a->h_stop = 1u; // a warm-up still running ends
    if (!ck(cudaSetDevice(a->g->device), "cudaSetDevice")) return -1;
    const int64_t row = a->n_head * TRX_ATTN_HD, lay = a->n_head * a->n_ctx * TRX_ATTN_HD, n_pos = pos + 1;
    float *dq = a->io, *dk = a->io + row, *dv = a->io + 2 * row, *dout = a->io + 3 * row;
    float *K = a->keys + layer * lay, *V = a->values + layer * lay;
    bool ok = ck(cudaMemcpyAsync(dq, q, (size_t)row * 4, cudaMemcpyHostToDevice, a->st), "copy q") &&
              ck(cudaMemcpyAsync(dk, k, (size_t)row * 4, cudaMemcpyHostToDevice, a->st), "copy k") &&
              ck(cudaMemcpyAsync(dv, v, (size_t)row * 4, cudaMemcpyHostToDevice, a->st), "copy v");
    if (!ok) return -1;
    const unsigned sb = (unsigned)((a->n_head + 7) / 8);
    trx_attn_store<<<sb, 256, 0, a->st>>>(dk, 1, (int)a->n_head, pos, a->n_ctx, K);
    trx_attn_store<<<sb, 256, 0, a->st>>>(dv, 1, (int)a->n_head, pos, a->n_ctx, V);
    trx_attn_scores<<<dim3((unsigned)((n_pos + 15) / 16), (unsigned)a->n_head), 256, 0, a->st>>>(
        dq, K, V, (int)n_pos, a->n_ctx, scale, a->scores, a->s_stride);
    trx_softmax_rows_k<<<(unsigned)a->n_head, 256, 0, a->st>>>(a->scores, n_pos, a->s_stride);
    trx_attn_values<<<(unsigned)a->n_head, 160, TRX_ATTN_STAGES * TRX_ATTN_STAGE_BYTES, a->st>>>(
        a->scores, a->s_stride, V, (int)n_pos, a->n_ctx, dout, a->err);
    int32_t e = 0;
    ok = ck(cudaGetLastError(), "attention kernels") &&
         ck(cudaMemcpyAsync(out, dout, (size_t)row * 4, cudaMemcpyDeviceToHost, a->st), "copy out") &&
         ck(cudaMemcpyAsync(&e, a->err, 4, cudaMemcpyDeviceToHost, a->st), "copy error word") && stream_wait(a->st);
    if (!ok) return -1;
    if (e != 0) {
        attn_fail(a, "the attention kernel gave up on a bounded wait");
        return -1;
    }
    return 0;
}

extern "C" int tr_gpu_attn_warm(tr_gpu_attn *a, uint64_t ns) {
    g_err.clear();
    if (a == nullptr) {
        set_err("bad arguments to tr_gpu_attn_warm");
        return -1;
    }
    if (!ck(cudaSetDevice(a->g->device), "cudaSetDevice")) return -1;
    // the one before has ended (its stop word was set, or its time ran out), then the stop word is cleared
    *(volatile uint32_t *)a->h_stop = 1u;
    if (!ck(cudaStreamSynchronize(a->warm_st), "warm stream")) return -1;
    *(volatile uint32_t *)a->h_stop = 0u;
    trx_attn_warm<<<1, 1, 0, a->warm_st>>>(a->d_stop, std::min<uint64_t>(ns, kAttnWarmMaxNs));
    return ck(cudaGetLastError(), "warm kernel") ? 0 : -1;
}

// ---------------------------------------------------------------------------------------------
// the kernel level

namespace {

struct KMat {
    uint8_t *dev;
    int64_t bytes;
};

struct KCtx {
    std::mutex mu;
    bool init = false;
    int device = 0;
    cudaStream_t st = nullptr;
    std::unordered_map<std::string, KMat> mats;
    uint8_t *buf = nullptr; // x, prepared x, y
    int64_t buf_bytes = 0;
    uint8_t *tmp = nullptr;
    int64_t tmp_bytes = 0;
};

KCtx &kctx() {
    static KCtx c;
    return c;
}

bool kinit(KCtx &c) {
    if (c.init) return true;
    if (!ck(cudaGetDevice(&c.device), "cudaGetDevice") ||
        !ck(cudaStreamCreateWithFlags(&c.st, cudaStreamNonBlocking), "cudaStreamCreate"))
        return false;
    c.init = true;
    return true;
}

bool kreserve(uint8_t **p, int64_t *have, int64_t need) {
    if (*have >= need) return true;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *have = 0;
    if (!ck(cudaMalloc(p, (size_t)need), "cudaMalloc")) return false;
    *have = need;
    return true;
}

// the device copy of a host matrix, uploaded on first sight
uint8_t *kmat(KCtx &c, const tr_mat &w) {
    char key[96];
    snprintf(key, sizeof key, "%p/%d/%lld/%lld", w.data, (int)w.type, (long long)w.rows, (long long)w.cols);
    auto it = c.mats.find(key);
    if (it != c.mats.end()) return it->second.dev;
    const int64_t bytes = trx_row_bytes(w.type, w.cols) * w.rows;
    uint8_t *d = nullptr;
    if (!ck(cudaMalloc(&d, (size_t)align_up(bytes, 256)), "cudaMalloc(weight)")) return nullptr;
    if (!kreserve(&c.tmp, &c.tmp_bytes, bytes) || !upload_matrix(w.type, w.rows, w.cols, w.data, d, c.tmp, c.st)) {
        cudaFree(d);
        return nullptr;
    }
    c.mats[key] = KMat{d, bytes};
    return d;
}

bool ktype_ok(const tr_mat &w) {
    switch (w.type) {
    case TRX_F32:
    case TRX_F16:
    case TRX_BF16: return w.cols % 16 == 0;
    case TRX_Q8_0:
    case TRX_Q6_K:
    case TRX_Q4_K: return w.cols % 256 == 0;
    default: return false;
    }
}

bool kgrouped(const tr_mat *w, const int64_t *offsets, int64_t n_groups, const float *x, float *y) {
    if (n_groups <= 0 || offsets[n_groups] <= 0 || w[0].rows <= 0) return true;
    const int type = w[0].type;
    const int64_t rows = w[0].rows, cols = w[0].cols, n_in = offsets[n_groups];
    for (int64_t g = 0; g < n_groups; g++)
        if (w[g].type != type || w[g].rows != rows || w[g].cols != cols || !ktype_ok(w[g])) {
            set_err("tr_matmul_grouped: group %lld has type %d %lldx%lld, not supported or not the first's", (long long)g,
                    (int)w[g].type, (long long)w[g].rows, (long long)w[g].cols);
            return false;
        }
    if (n_in > INT32_MAX / 2 || rows > INT32_MAX / 2) {
        set_err("tr_matmul_grouped: too large");
        return false;
    }
    KCtx &c = kctx();
    std::lock_guard<std::mutex> lock(c.mu);
    if (!kinit(c) || !ck(cudaSetDevice(c.device), "cudaSetDevice")) return false;
    std::vector<const uint8_t *> ptrs((size_t)n_groups, nullptr);
    for (int64_t g = 0; g < n_groups; g++)
        if (offsets[g + 1] > offsets[g]) {
            ptrs[(size_t)g] = kmat(c, w[g]);
            if (ptrs[(size_t)g] == nullptr) return false;
        }
    // device buffer: x, prepared x (planes + bf + scale), y, group table, offsets
    const int64_t xb = align_up(n_in * cols * 4, 256), pb = align_up(n_in * cols * 4, 256),
                  bfb = align_up(n_in * (cols / 32) * 8, 256), scb = align_up(n_in * (cols / 256 + 1) * 8, 256),
                  yb = align_up(n_in * rows * 4, 256), gb = align_up(n_groups * 8, 256),
                  ob = align_up((n_groups + 1) * 4, 256);
    if (!kreserve(&c.buf, &c.buf_bytes, xb + pb + bfb + scb + yb + gb + ob)) return false;
    uint8_t *b = c.buf;
    float *dx = (float *)b;
    uint32_t *dq = (uint32_t *)(b + xb);
    double *dbf = (double *)(b + xb + pb);
    double *dsc = (double *)(b + xb + pb + bfb);
    float *dy = (float *)(b + xb + pb + bfb + scb);
    const uint8_t **dg = (const uint8_t **)(b + xb + pb + bfb + scb + yb);
    int32_t *doff = (int32_t *)(b + xb + pb + bfb + scb + yb + gb);
    std::vector<int32_t> off32((size_t)n_groups + 1);
    for (int64_t g = 0; g <= n_groups; g++) off32[(size_t)g] = (int32_t)offsets[g];
    bool ok = ck(cudaMemcpyAsync(dx, x, (size_t)(n_in * cols * 4), cudaMemcpyHostToDevice, c.st), "copy x") &&
              ck(cudaMemcpyAsync(dg, ptrs.data(), (size_t)n_groups * 8, cudaMemcpyHostToDevice, c.st), "copy table") &&
              ck(cudaMemcpyAsync(doff, off32.data(), (size_t)(n_groups + 1) * 4, cudaMemcpyHostToDevice, c.st),
                 "copy offsets");
    if (!ok) return false;
    ok = trx_kapi_grouped(type, rows, cols, dg, doff, (int)n_groups, (int)n_in, dx, dq, dbf, dsc, dy, c.st) &&
         ck(cudaGetLastError(), "grouped kernel") &&
         ck(cudaMemcpyAsync(y, dy, (size_t)(n_in * rows * 4), cudaMemcpyDeviceToHost, c.st), "copy y") &&
         stream_wait(c.st);
    return ok;
}

void kfail(const char *fn) { fprintf(stderr, "trmoe: %s failed: %s\n", fn, g_err.c_str()); }

// Q4_K's prepared road (tr_q4x_road, tr_q4x_prepare, tr_matmul_q4x_prepared(_n), tr_swiglu_prepare). The engine keeps
// a pass's prepared input rows in its own buffer, one slot of tr_q4x_bytes(cols) bytes a row; here a slot holds the
// row's floats at its start, and the GPU prepares the digits inside each matmul from them (the same floats give the
// same digits, so every output is the reference road's).

// the bytes of one slot: Trochilus's tr_q4x_bytes (src/kernels/kernels.c:489-492)
int64_t q4x_slot(int64_t n) {
    const int64_t b = 4 * n + n / 8 + n / 4 + n / 32;
    return (b + 63) / 64 * 64;
}

// the weights the library's Q4_K road takes (its kernels' shape limits); the reference's q4x_road
// (src/kernels/kernels.c:1122-1128) tests w[0] alone too, the other groups being of its type and shape by contract
bool q4x_takes(const tr_mat *w) {
    return w != nullptr && w[0].type == TRX_Q4_K && w[0].rows > 0 && w[0].rows % 16 == 0 && w[0].cols > 0 &&
           w[0].cols % 256 == 0 && w[0].rows <= INT32_MAX / 2 && w[0].cols <= INT32_MAX / 2;
}

std::atomic<uint64_t> g_q4x_fused{0}; // tr_matmul_q4x_prepared_n's calls of more than one weight

// y_m[p rows + r] = row r of ws[m][g(p)] . input row p, for m < n_w (Q4_K weights of one shape, the same groups);
// input row p = the floats at the start of slot map[p] (map NULL: slot p) of xq. The slots the call reads go up in
// one strided copy, the rows are gathered on the GPU, prepared once, and every weight reads them.
bool kprepared(const tr_mat *const *ws, int n_w, const int64_t *offsets, int64_t n_groups, const uint8_t *xq,
               const int64_t *map, float *const *ys) {
    const int64_t rows = ws[0][0].rows, cols = ws[0][0].cols, n_in = offsets[n_groups], slot = q4x_slot(cols);
    for (int m = 0; m < n_w; m++)
        for (int64_t g = 0; g < n_groups; g++)
            if (ws[m][g].type != TRX_Q4_K || ws[m][g].rows != rows || ws[m][g].cols != cols) {
                set_err("weight %d group %lld has type %d %lldx%lld, not Q4_K %lldx%lld", m, (long long)g,
                        (int)ws[m][g].type, (long long)ws[m][g].rows, (long long)ws[m][g].cols, (long long)rows,
                        (long long)cols);
                return false;
            }
    int64_t n_src = n_in;
    if (map) {
        n_src = 0;
        for (int64_t p = 0; p < n_in; p++) {
            if (map[p] < 0 || map[p] >= INT32_MAX / 2) {
                set_err("map[%lld] = %lld is not a prepared row", (long long)p, (long long)map[p]);
                return false;
            }
            n_src = std::max(n_src, map[p] + 1);
        }
    }
    if (n_in > INT32_MAX / 2 || n_groups > 65535) { // (the groups are the grid's second dimension)
        set_err("too large: %lld input rows in %lld groups", (long long)n_in, (long long)n_groups);
        return false;
    }
    KCtx &c = kctx();
    std::lock_guard<std::mutex> lock(c.mu);
    if (!kinit(c) || !ck(cudaSetDevice(c.device), "cudaSetDevice")) return false;
    std::vector<const uint8_t *> ptrs((size_t)(n_w * n_groups), nullptr);
    for (int m = 0; m < n_w; m++)
        for (int64_t g = 0; g < n_groups; g++)
            if (offsets[g + 1] > offsets[g]) {
                ptrs[(size_t)(m * n_groups + g)] = kmat(c, ws[m][g]);
                if (ptrs[(size_t)(m * n_groups + g)] == nullptr) return false;
            }
    // device buffer: the slots' floats, the gathered rows (map given), the prepared rows (planes, sub-block sums,
    // scales), the map, the offsets, then per weight its group table and output
    const int64_t sb = align_up(n_src * cols * 4, 256), xb = map ? align_up(n_in * cols * 4, 256) : 0,
                  pb = align_up(n_in * cols * 4, 256), bfb = align_up(n_in * (cols / 32) * 8, 256),
                  scb = align_up(n_in * (cols / 256 + 1) * 8, 256), mb = map ? align_up(n_in * 4, 256) : 0,
                  ob = align_up((n_groups + 1) * 4, 256), gb = align_up(n_groups * 8, 256),
                  yb = align_up(n_in * rows * 4, 256);
    if (!kreserve(&c.buf, &c.buf_bytes, sb + xb + pb + bfb + scb + mb + ob + n_w * (gb + yb))) return false;
    uint8_t *b = c.buf;
    float *dsrc = (float *)b;
    float *dx = map ? (float *)(b + sb) : dsrc;
    uint32_t *dq = (uint32_t *)(b + sb + xb);
    double *dbf = (double *)(b + sb + xb + pb);
    double *dsc = (double *)(b + sb + xb + pb + bfb);
    int32_t *dmap = (int32_t *)(b + sb + xb + pb + bfb + scb);
    int32_t *doff = (int32_t *)(b + sb + xb + pb + bfb + scb + mb);
    uint8_t *per = b + sb + xb + pb + bfb + scb + mb + ob; // weight m: table at per + m (gb + yb), output after it
    std::vector<int32_t> off32((size_t)n_groups + 1), map32(map ? (size_t)n_in : 0);
    for (int64_t g = 0; g <= n_groups; g++) off32[(size_t)g] = (int32_t)offsets[g];
    for (size_t p = 0; p < map32.size(); p++) map32[p] = (int32_t)map[p];
    bool ok = ck(cudaMemcpy2DAsync(dsrc, (size_t)cols * 4, xq, (size_t)slot, (size_t)cols * 4, (size_t)n_src,
                                   cudaMemcpyHostToDevice, c.st),
                 "copy prepared rows") &&
              ck(cudaMemcpyAsync(doff, off32.data(), off32.size() * 4, cudaMemcpyHostToDevice, c.st), "copy offsets");
    if (ok && map) {
        ok = ck(cudaMemcpyAsync(dmap, map32.data(), map32.size() * 4, cudaMemcpyHostToDevice, c.st), "copy map");
        if (ok) trx_kapi_gather_k<<<(unsigned)n_in, 256, 0, c.st>>>(dsrc, dmap, (int)cols, dx);
    }
    for (int m = 0; ok && m < n_w; m++) {
        const uint8_t **dg = (const uint8_t **)(per + m * (gb + yb));
        float *dy = (float *)(per + m * (gb + yb) + gb);
        ok = ck(cudaMemcpyAsync(dg, ptrs.data() + m * n_groups, (size_t)n_groups * 8, cudaMemcpyHostToDevice, c.st),
                "copy table") &&
             trx_kapi_grouped(TRX_Q4_K, rows, cols, dg, doff, (int)n_groups, (int)n_in, dx, dq, dbf, dsc, dy, c.st,
                              m == 0) &&
             ck(cudaGetLastError(), "grouped kernel") &&
             ck(cudaMemcpyAsync(ys[m], dy, (size_t)(n_in * rows * 4), cudaMemcpyDeviceToHost, c.st), "copy y");
    }
    return ok && stream_wait(c.st);
}

} // namespace

extern "C" void tr_matmul_grouped(tr_pool *pool, const tr_mat *w, const int64_t *offsets, int64_t n_groups,
                                  const float *x, float *y) {
    (void)pool;
    g_err.clear();
    if (!kgrouped(w, offsets, n_groups, x, y)) kfail("tr_matmul_grouped");
}

extern "C" void tr_matmul_grouped_s(tr_pool *pool, const tr_mat *w, const int64_t *offsets, int64_t n_groups,
                                    const float *x, float *y, const void *s) {
    (void)s;
    tr_matmul_grouped(pool, w, offsets, n_groups, x, y);
}

extern "C" void tr_matmul(tr_pool *pool, const tr_mat *w, const float *x, int64_t n_tokens, float *y) {
    const int64_t offsets[2] = {0, n_tokens};
    tr_matmul_grouped(pool, w, offsets, 1, x, y);
}

extern "C" void tr_softmax(float *x, int64_t n) {
    g_err.clear();
    if (n <= 0) return;
    KCtx &c = kctx();
    std::lock_guard<std::mutex> lock(c.mu);
    bool ok = kinit(c) && ck(cudaSetDevice(c.device), "cudaSetDevice") &&
              kreserve(&c.buf, &c.buf_bytes, align_up(n * 4, 256));
    if (ok) {
        float *d = (float *)c.buf;
        ok = ck(cudaMemcpyAsync(d, x, (size_t)n * 4, cudaMemcpyHostToDevice, c.st), "copy") &&
             trx_kapi_softmax(d, n, c.st) && ck(cudaGetLastError(), "softmax kernel") &&
             ck(cudaMemcpyAsync(x, d, (size_t)n * 4, cudaMemcpyDeviceToHost, c.st), "copy back") && stream_wait(c.st);
    }
    if (!ok) kfail("tr_softmax");
}

extern "C" void tr_swiglu(tr_pool *pool, float *x, const float *y, int64_t n) {
    (void)pool;
    g_err.clear();
    if (n <= 0) return;
    KCtx &c = kctx();
    std::lock_guard<std::mutex> lock(c.mu);
    bool ok = kinit(c) && ck(cudaSetDevice(c.device), "cudaSetDevice") &&
              kreserve(&c.buf, &c.buf_bytes, 2 * align_up(n * 4, 256));
    if (ok) {
        float *dx = (float *)c.buf, *dy = (float *)(c.buf + align_up(n * 4, 256));
        ok = ck(cudaMemcpyAsync(dx, x, (size_t)n * 4, cudaMemcpyHostToDevice, c.st), "copy x") &&
             ck(cudaMemcpyAsync(dy, y, (size_t)n * 4, cudaMemcpyHostToDevice, c.st), "copy y") &&
             trx_kapi_swiglu(dx, dy, n, c.st) && ck(cudaGetLastError(), "swiglu kernel") &&
             ck(cudaMemcpyAsync(x, dx, (size_t)n * 4, cudaMemcpyDeviceToHost, c.st), "copy back") && stream_wait(c.st);
    }
    if (!ok) kfail("tr_swiglu");
}

extern "C" void tr_matmul_s(tr_pool *pool, const tr_mat *w, const float *x, int64_t n_tokens, float *y, const void *s) {
    (void)pool;
    (void)s;
    g_err.clear();
    const int64_t offsets[2] = {0, n_tokens};
    if (!kgrouped(w, offsets, 1, x, y)) kfail("tr_matmul_s");
}

extern "C" size_t tr_q4x_bytes(int64_t n) { return (size_t)q4x_slot(n); }

extern "C" int tr_q4x_road(tr_pool *pool, const tr_mat *w, const int64_t *offsets, int64_t n_groups, const void *s) {
    (void)pool;
    (void)offsets;
    (void)n_groups;
    (void)s;
    return q4x_takes(w) ? 1 : 0;
}

extern "C" void tr_q4x_prepare(tr_pool *pool, const float *x, int64_t n, int64_t cols, void *xq) {
    (void)pool;
    if (n <= 0 || cols <= 0) return;
    const int64_t slot = q4x_slot(cols);
    for (int64_t r = 0; r < n; r++) memcpy((uint8_t *)xq + r * slot, x + r * cols, (size_t)cols * 4);
}

extern "C" int tr_matmul_q4x_prepared(tr_pool *pool, const tr_mat *w, const int64_t *offsets, int64_t n_groups,
                                      const void *xq, const int64_t *map, float *y, const void *s) {
    (void)pool;
    (void)s;
    g_err.clear();
    if (n_groups <= 0 || offsets[n_groups] <= 0 || w[0].rows <= 0) return 1;
    if (!q4x_takes(w)) return 0;
    float *const ys[1] = {y};
    if (!kprepared(&w, 1, offsets, n_groups, (const uint8_t *)xq, map, ys)) kfail("tr_matmul_q4x_prepared");
    return 1;
}

extern "C" int tr_matmul_q4x_prepared_n(tr_pool *pool, const tr_mat *const *w, int n_w, const int64_t *offsets,
                                        int64_t n_groups, const void *xq, const int64_t *map, float *const *y,
                                        const void *s) {
    if (n_w < 1 || n_w > TRMOE_Q4X_MATS) return 0;
    if (n_w == 1) return tr_matmul_q4x_prepared(pool, w[0], offsets, n_groups, xq, map, y[0], s);
    g_err.clear();
    if (n_groups <= 0 || offsets[n_groups] <= 0 || w[0][0].rows <= 0) return 1;
    for (int m = 0; m < n_w; m++)
        if (!q4x_takes(w[m]) || w[m][0].rows != w[0][0].rows || w[m][0].cols != w[0][0].cols) return 0;
    g_q4x_fused.fetch_add(1, std::memory_order_relaxed);
    if (!kprepared(w, n_w, offsets, n_groups, (const uint8_t *)xq, map, y)) kfail("tr_matmul_q4x_prepared_n");
    return 1;
}

extern "C" uint64_t tr_q4x_fused_calls(void) { return g_q4x_fused.load(std::memory_order_relaxed); }

extern "C" void tr_swiglu_prepare(tr_pool *pool, float *x, const float *y, int64_t n_rows, int64_t n, void *xq) {
    (void)pool;
    g_err.clear();
    if (n_rows <= 0 || n <= 0) return;
    const int64_t total = n_rows * n, slot = q4x_slot(n);
    KCtx &c = kctx();
    std::lock_guard<std::mutex> lock(c.mu);
    bool ok = kinit(c) && ck(cudaSetDevice(c.device), "cudaSetDevice") &&
              kreserve(&c.buf, &c.buf_bytes, 2 * align_up(total * 4, 256));
    if (ok) {
        float *dx = (float *)c.buf, *dy = (float *)(c.buf + align_up(total * 4, 256));
        ok = ck(cudaMemcpyAsync(dx, x, (size_t)total * 4, cudaMemcpyHostToDevice, c.st), "copy x") &&
             ck(cudaMemcpyAsync(dy, y, (size_t)total * 4, cudaMemcpyHostToDevice, c.st), "copy y") &&
             trx_kapi_swiglu(dx, dy, total, c.st) && ck(cudaGetLastError(), "swiglu kernel") &&
             ck(cudaMemcpyAsync(x, dx, (size_t)total * 4, cudaMemcpyDeviceToHost, c.st), "copy back") &&
             ck(cudaMemcpy2DAsync(xq, (size_t)slot, dx, (size_t)n * 4, (size_t)n * 4, (size_t)n_rows,
                                  cudaMemcpyDeviceToHost, c.st),
                "copy prepared rows") &&
             stream_wait(c.st);
    }
    if (!ok) kfail("tr_swiglu_prepare");
}

extern "C" void trmoe_kernel_cache_clear(void) {
    KCtx &c = kctx();
    std::lock_guard<std::mutex> lock(c.mu);
    for (auto &kv : c.mats) cudaFree(kv.second.dev);
    c.mats.clear();
}

// ---------------------------------------------------------------------------------------------
// tr_matmul_q4k_noalloc: the Q4_K kernel-level product on caller-owned device memory, allocating nothing

// Its scratch, one per GPU that loads the library: bytes 0..7 the group table's one matrix pointer, 8..15 the
// group offsets {0, n_tokens}, then from byte 256 the tokens' prepared rows (planes, sub-block sums, scales).
// Host code never dereferences this name: on the host it only stands for the symbol, whose device address
// cudaGetSymbolAddress gives.
static __device__ __align__(256) uint8_t g_noalloc_scratch[TRMOE_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kNoallocDevices = 64;
std::mutex g_noalloc_mu;
uint8_t *g_noalloc_ptr[kNoallocDevices]; // per device: the scratch's device address, found on its first call

// the scratch's address on the current device `dev`, looked up once with that device current
uint8_t *noalloc_scratch(int dev) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_noalloc_ptr[dev] == nullptr) {
        void *p = nullptr;
        if (!ck(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress")) return nullptr;
        g_noalloc_ptr[dev] = static_cast<uint8_t *>(p);
    }
    return g_noalloc_ptr[dev];
}

// writes the scratch's group table: one group of n_tok rows multiplied by w
__global__ void trx_noalloc_table(uint8_t *scratch, const uint8_t *w, int32_t n_tok) {
    *reinterpret_cast<const uint8_t **>(scratch) = w;
    reinterpret_cast<int32_t *>(scratch + 8)[0] = 0;
    reinterpret_cast<int32_t *>(scratch + 8)[1] = n_tok;
}

} // namespace

extern "C" int tr_matmul_q4k_noalloc(const void *d_w, int64_t rows, int64_t cols, const float *d_x, int64_t n_tokens,
                                     float *d_y, void *stream) {
    g_err.clear();
    if (d_w == nullptr || d_x == nullptr || d_y == nullptr || rows < 1 || rows > (1 << 24) || cols < 256 ||
        cols % 256 != 0 || cols > (1 << 20) || n_tokens < 1 || ((uintptr_t)d_w & 15u) != 0 || ((uintptr_t)d_x & 15u) != 0) {
        set_err("tr_matmul_q4k_noalloc: bad arguments (rows %lld, cols %lld: a multiple of 256, n_tokens %lld, "
                "d_w and d_x 16-byte aligned)",
                (long long)rows, (long long)cols, (long long)n_tokens);
        return -1;
    }
    // the scratch's parts, each rounded up to 256 bytes: table, planes, sub-block sums, scales
    const int64_t pb = align_up(n_tokens * cols * 4, 256), bfb = align_up(n_tokens * (cols / 32) * 8, 256),
                  scb = align_up(n_tokens * (cols / 256) * 8, 256), need = 256 + pb + bfb + scb;
    if (need > (int64_t)TRMOE_NOALLOC_SCRATCH_BYTES) {
        set_err("tr_matmul_q4k_noalloc: %lld tokens of %lld columns need %lld bytes of scratch, more than its %lld",
                (long long)n_tokens, (long long)cols, (long long)need, (long long)TRMOE_NOALLOC_SCRATCH_BYTES);
        return -1;
    }
    int dev = 0;
    if (!ck(cudaGetDevice(&dev), "cudaGetDevice")) return -1;
    if (dev < 0 || dev >= kNoallocDevices) {
        set_err("tr_matmul_q4k_noalloc: device %d is beyond the %d it serves", dev, kNoallocDevices);
        return -1;
    }
    uint8_t *scratch = noalloc_scratch(dev);
    if (scratch == nullptr) return -1;
    cudaStream_t st = (cudaStream_t)stream;
    // nothing in the scratch has to start at zero: this call writes the table and every prepared row it reads
    trx_noalloc_table<<<1, 1, 0, st>>>(scratch, static_cast<const uint8_t *>(d_w), (int32_t)n_tokens);
    uint32_t *dq = reinterpret_cast<uint32_t *>(scratch + 256);
    double *dbf = reinterpret_cast<double *>(scratch + 256 + pb);
    double *dsc = reinterpret_cast<double *>(scratch + 256 + pb + bfb);
    trx_kapi_grouped(TRX_Q4_K, rows, cols, reinterpret_cast<const uint8_t *const *>(scratch),
                     reinterpret_cast<const int32_t *>(scratch + 8), 1, (int)n_tokens, d_x, dq, dbf, dsc, d_y, st);
    return ck(cudaGetLastError(), "tr_matmul_q4k_noalloc launch") ? 0 : -1;
}
