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
#include "decode.cuh"
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
// Polls the stream: busy for the first 2 ms (a decode call's work takes tens of microseconds, and a sleep, however
// short it asks to be, lasts about 60 us on Linux), then with 20 us sleeps between the polls.
// what a kernel's error flag (TrxWork::err) says: the one-token kernel's 16 is a set-up refusal, every other value
// a bounded wait that gave up (the value tells which wait)
const char *err_flag_what(int32_t flag) {
    return flag == 16 ? "the one-token kernel's shared memory was not 128-byte aligned for its tensor copies"
                      : "a kernel gave up on a bounded wait";
}

bool stream_wait(cudaStream_t s, double timeout_s = 60.0) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t e = cudaStreamQuery(s);
        if (e == cudaSuccess) return true;
        if (e != cudaErrorNotReady) return ck(e, "cudaStreamQuery");
        const double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (dt > timeout_s) {
            set_err("the GPU did not finish within %.0f s", timeout_s);
            return false;
        }
        if (dt > 0.002) std::this_thread::sleep_for(std::chrono::microseconds(20));
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
    int64_t off[28];
    int64_t total;
};

// carve the workspace of one context (every piece 256-byte aligned)
// whether a context can take the tensor-core road for long passes: its converters dequantise Q8_0, Q4_K and Q6_K
bool prefill_capable(const tr_gpu_moe_config &c) {
    auto ok = [](int t) { return t == TRX_Q8_0 || t == TRX_Q4_K || t == TRX_Q6_K; };
    return ok(c.gate_type) && ok(c.down_type);
}

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
        TRX_DC_GRID_MAX * E * 8, // 26 the one-token kernel's tagged logits (a row for each CTA)
        TRX_DC_KMAX * F * 8, // 27 and its tagged h values
    };
    WorkLayout w{};
    int64_t o = 0;
    for (int i = 0; i < 28; i++) {
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
    bool dec1_ok = false;  // the one-token decode kernel (decode.cuh) fits and may be launched
    bool dec1_pdl = true;  // and is launched with programmatic dependent launch (off if the driver refuses it)
    // Q4_K: per layer the one-token kernel's tensor maps over the gate, up and (a Q4_K) down matrices
    // (trx_dec1_map)
    std::vector<CUtensorMap> dc_maps;
    int64_t tag_bytes = 0; // its tagged exchange words (work regions 26 and 27), cleared with the counters
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
// the one-token kernel for a router type and a gate/up type (Q4_K: Q4_K_M's road, Q8_0: all Q8_0)
typedef void (*Dec1Fn)(TrxLayer, TrxShape, const float *, TrxWork, TrxSync *, float *, float *, uint32_t, TrxDecPlan,
                       const CUtensorMap, const CUtensorMap, const CUtensorMap);
static Dec1Fn dec1_fn(int router_type, int gate_type, int down_type) {
    const bool bf = router_type == TRX_BF16;
    if (gate_type == TRX_Q8_0)
        return bf ? trx_k_dec1<TRX_BF16, TRX_Q8_0, TRX_Q8_0> : trx_k_dec1<TRX_F32, TRX_Q8_0, TRX_Q8_0>;
    if (down_type == TRX_Q4_K)
        return bf ? trx_k_dec1<TRX_BF16, TRX_Q4_K, TRX_Q4_K> : trx_k_dec1<TRX_F32, TRX_Q4_K, TRX_Q4_K>;
    return bf ? trx_k_dec1<TRX_BF16, TRX_Q4_K, TRX_Q6_K> : trx_k_dec1<TRX_F32, TRX_Q4_K, TRX_Q6_K>;
}

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
    // the one-token kernel: its plan's shared memory, a CTA an SM
    if (m->fused_ok && trx_dec1_takes(c.gate_type, c.down_type, c.router_type, (int)c.n_embd, (int)c.n_ff,
                                      (int)c.n_expert, (int)c.n_used, 1, m->grid_fused, false)) {
        const TrxDecPlan P =
            trx_dec_plan(c.gate_type, c.down_type, (int)c.n_embd, (int)c.n_ff, (int)c.n_used, m->grid_fused);
        bool ok1 = true;
        for (auto fn : {dec1_fn(TRX_F32, c.gate_type, c.down_type), dec1_fn(TRX_BF16, c.gate_type, c.down_type)}) {
            int occ1 = 0;
            cudaFuncAttributes fa1{};
            if (!ck(cudaFuncGetAttributes(&fa1, fn), "cudaFuncGetAttributes") ||
                fa1.sharedSizeBytes + P.total + 1024 > limit ||
                !ck(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)P.total), "smem dec1") ||
                !ck(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ1, fn, TRX_DC_THREADS, P.total), "occupancy"))
                ok1 = false;
            else ok1 = ok1 && occ1 >= 1;
        }
        g_err.clear();
        m->dec1_ok = ok1;
    }
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

extern "C" int trmoe_kernel_arch(void) {
    g_err.clear();
    int dev = 0;
    if (!ck(cudaGetDevice(&dev), "cudaGetDevice")) return -1;
    cudaFuncAttributes a{};
    if (!ck(cudaFuncGetAttributes(&a, trx_k_layer<TRX_Q4_K, TRX_Q6_K>), "cudaFuncGetAttributes")) return -1;
    return a.binaryVersion;
}

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

static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (encode == nullptr) {
        cudaDriverEntryPointQueryResult q{};
        void *fn = nullptr;
        if (!ck(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q), "driver entry point") ||
            q != cudaDriverEntryPointSuccess || fn == nullptr) {
            if (g_err.empty()) set_err("cuTensorMapEncodeTiled is not available");
            return nullptr;
        }
        encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
    }
    return encode;
}

// The one-token kernel's map over a layer's Q4_K gate, up or down matrices: bytes x rows x experts (row bytes, rows,
// expert stride), boxes of one 256-block (144 bytes) of box_rows rows of one expert; rows past the end read as zeros
static bool trx_dec1_map(CUtensorMap *map, const uint8_t *base, int64_t row_bytes, int64_t rows, int64_t experts,
                         int64_t expert_bytes, int box_rows) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (encode == nullptr) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)row_bytes, (cuuint64_t)rows, (cuuint64_t)experts};
    const cuuint64_t strides[2] = {(cuuint64_t)row_bytes, (cuuint64_t)expert_bytes};
    const cuuint32_t box[3] = {144, (cuuint32_t)box_rows, 1}, es[3] = {1, 1, 1};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, (void *)base, dims, strides, box, es,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_err("cuTensorMapEncodeTiled failed (%d)", (int)r);
        return false;
    }
    return true;
}

// a 2-D fp32 tensor map over rows x cols (row-major), boxes of 32 columns x 128 rows, 128-byte swizzle
static bool encode_map(CUtensorMap *map, float *base, int64_t rows, int64_t cols) {
    PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
    if (encode == nullptr) return false;
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

// the tensor-core GEMM for gate/up or down over weights of the given type
typedef void (*PfGemmFn)(const CUtensorMap, const CUtensorMap, TrxPfArgs);
static PfGemmFn pf_gemm_fn(bool gateup, int type) {
    if (gateup)
        return type == TRX_Q4_K ? trx_k_pf_gemm<true, TRX_Q4_K>
               : type == TRX_Q6_K ? trx_k_pf_gemm<true, TRX_Q6_K>
                                  : trx_k_pf_gemm<true, TRX_Q8_0>;
    return type == TRX_Q4_K ? trx_k_pf_gemm<false, TRX_Q4_K>
           : type == TRX_Q6_K ? trx_k_pf_gemm<false, TRX_Q6_K>
                              : trx_k_pf_gemm<false, TRX_Q8_0>;
}

// the tensor-core road: its kernels' shared memory and the A operands' tensor maps (the h planes reuse the h and
// hq regions, which the Q8_0 roads of the other kernels leave free during a prefill call)
static bool plan_prefill(tr_gpu_moe *m) {
    const tr_gpu_moe_config &c = m->cfg;
    const int64_t R = c.max_tokens * c.n_used;
    if (!ck(cudaFuncSetAttribute(pf_gemm_fn(true, c.gate_type), cudaFuncAttributeMaxDynamicSharedMemorySize, TRX_PF_SMEM),
            "smem prefill") ||
        !ck(cudaFuncSetAttribute(pf_gemm_fn(false, c.down_type), cudaFuncAttributeMaxDynamicSharedMemorySize, TRX_PF_SMEM),
            "smem prefill"))
        return false;
    if (!encode_map(&m->pf_map_x[0], m->pf_xhi, R, c.n_embd) || !encode_map(&m->pf_map_x[1], m->pf_xlo, R, c.n_embd) ||
        !encode_map(&m->pf_map_h[0], m->work.h, R, c.n_ff) ||
        !encode_map(&m->pf_map_h[1], reinterpret_cast<float *>(m->work.hq), R, c.n_ff))
        return false;
    m->pf_ok = true;
    // calls this long take the road by default: 256 tokens, or 32 when the down weights are Q4_K, whose exact road
    // (the Q4_K input preparation of every h row) costs about 74 us a token against the road's flat ~1 ms (measured)
    m->pf_min = c.down_type == TRX_Q4_K ? 32 : 256;
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
        m->dc_maps.assign((size_t)(3 * cfg->n_layers), CUtensorMap{});
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
    w.tag_logits = (unsigned long long *)(b + wl.off[26]);
    w.tag_h = (unsigned long long *)(b + wl.off[27]);
    m->tag_bytes = wl.off[27] + align_up(TRX_DC_KMAX * cfg->n_ff * 8, 256) - wl.off[26];
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
    // the one-token kernel's maps over the Q4_K gate and up matrices; without them (no driver entry point) every
    // call takes the fused kernel instead
    if (c.gate_type == TRX_Q4_K && m->dec1_ok &&
        !(trx_dec1_map(&m->dc_maps[(size_t)(3 * layer)], L.gate, trx_row_bytes(c.gate_type, H), F, E, L.gate_mb, 8) &&
          trx_dec1_map(&m->dc_maps[(size_t)(3 * layer + 1)], L.up, trx_row_bytes(c.gate_type, H), F, E, L.up_mb, 8) &&
          (c.down_type != TRX_Q4_K || trx_dec1_map(&m->dc_maps[(size_t)(3 * layer + 2)], L.down,
                                                   trx_row_bytes(c.down_type, F), H, E, L.down_mb, 16)))) {
        m->dec1_ok = false;
        g_err.clear();
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
    // the one-token kernel's tagged words: a word a failed call left could carry the next call's tag
    if (m->tag_bytes > 0) cudaMemsetAsync(m->work.tag_logits, 0, (size_t)m->tag_bytes, st);
    m->epoch = 0;
    stream_wait(st);
}

// whether a plain call of n_tok tokens (no dispatch outputs) runs the one-token kernel once a token
static bool takes_dec1seq(const tr_gpu_moe *m, int64_t n_tok) {
    const tr_gpu_moe_config &c = m->cfg;
    return n_tok > 1 && n_tok <= TRX_DC_SEQ_MAX && m->dec1_ok &&
           trx_dec1_takes(c.gate_type, c.down_type, c.router_type, (int)c.n_embd, (int)c.n_ff, (int)c.n_expert,
                          (int)c.n_used, 1, m->grid_fused, false);
}

extern "C" int tr_gpu_moe_launches(const tr_gpu_moe *m, int64_t n_tok) {
    if (m == nullptr) return 0;
    if (m->pf_ok && m->pf_min > 0 && n_tok >= m->pf_min && !m->prof) return 7; // route 3, gather, 2 GEMMs, combine
    int sg, sd;
    if (m->fused_ok && n_tok <= TRX_ROUTE_FUSED_MAX && m->cfg.n_expert + n_tok <= m->grid_fused && !m->prof &&
        fused_stages(m, (int)n_tok, &sg, &sd))
        return takes_dec1seq(m, n_tok) ? (int)n_tok : 1;
    return (n_tok <= TRX_ROUTE_FUSED_MAX ? 1 : 4) + 2 + (m->cfg.down_type == TRX_Q4_K ? 1 : 0);
}

extern "C" const char *tr_gpu_moe_kernel_name(const tr_gpu_moe *m, int64_t n_tok) {
    if (m == nullptr) return "";
    const int nl = tr_gpu_moe_launches(m, n_tok);
    if (nl == n_tok && n_tok > 1 && takes_dec1seq(m, n_tok)) return "trx_k_dec1";
    if (nl != 1) return "";
    const tr_gpu_moe_config &c = m->cfg;
    if (m->dec1_ok && trx_dec1_takes(c.gate_type, c.down_type, c.router_type, (int)c.n_embd, (int)c.n_ff,
                                     (int)c.n_expert, (int)c.n_used, (int)n_tok, m->grid_fused, false))
        return "trx_k_dec1";
    return "trx_k_layer";
}

extern "C" int tr_gpu_moe_check(tr_gpu_moe *m) {
    g_err.clear();
    if (m == nullptr || !ck(cudaSetDevice(m->device), "cudaSetDevice") || !stream_wait(m->stream)) return -1;
    int32_t flag = 0;
    if (!ck(cudaMemcpy(&flag, m->work.err, 4, cudaMemcpyDeviceToHost), "read error flag")) return -1;
    if (flag != 0) {
        reset_counters(m, m->stream);
        set_err("%s (device error flag %d)", err_flag_what(flag), flag);
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
    pf_gemm_fn(true, L.gate_type)<<<dim3((unsigned)(F / 128), mtiles), TRX_PF_THREADS, TRX_PF_SMEM, st>>>(
        m->pf_map_x[0], m->pf_map_x[1], a);
    a.wa = L.down;
    a.wb = nullptr;
    a.wa_mb = L.down_mb;
    a.wb_mb = 0;
    a.K = F;
    a.N = H;
    a.out_hi = w.h3;
    a.out_lo = nullptr;
    pf_gemm_fn(false, L.down_type)<<<dim3((unsigned)(H / TRX_PF_BN), mtiles), TRX_PF_THREADS, TRX_PF_SMEM, st>>>(
        m->pf_map_h[0], m->pf_map_h[1], a);
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

// the one-token decode kernel (decode.cuh): one cooperative launch, a CTA an SM
static int launch_dec1(tr_gpu_moe *m, int64_t layer, const TrxLayer &L, const TrxShape &S, const float *normed,
                       const TrxWork &w, float *x_io, float *ffn_out, uint32_t epoch, cudaStream_t st) {
    const TrxDecPlan P = trx_dec_plan(L.gate_type, L.down_type, S.H, S.F, S.k, m->grid_fused);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)m->grid_fused);
    cfg.blockDim = dim3(TRX_DC_THREADS);
    cfg.dynamicSmemBytes = P.total;
    cfg.stream = st;
    // cooperative (every CTA resident at once: they wait on one another) and, where the driver takes both,
    // programmatic dependent launch (the kernel's set-up overlaps the previous kernel's tail)
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = m->dec1_pdl ? 2 : 1;
    auto fn = dec1_fn(L.router_type, L.gate_type, L.down_type);
    // (Q4_K: the layer's maps, and the down's for a Q4_K down; Q8_0 takes none, and gets zeroed ones)
    CUtensorMap mg{}, mu{}, md{};
    if (L.gate_type == TRX_Q4_K) {
        mg = m->dc_maps[(size_t)(3 * layer)];
        mu = m->dc_maps[(size_t)(3 * layer + 1)];
        md = m->dc_maps[(size_t)(3 * layer + 2)];
    }
    cudaError_t e = cudaLaunchKernelEx(&cfg, fn, L, S, normed, w, m->sync, x_io, ffn_out, epoch, P, mg, mu, md);
    if (e != cudaSuccess && m->dec1_pdl) { // not taken together: cooperative alone from now on
        (void)cudaGetLastError();
        m->dec1_pdl = false;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, fn, L, S, normed, w, m->sync, x_io, ffn_out, epoch, P, mg, mu, md);
    }
    return ck(e, "decode layer launch") ? 0 : -1;
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
    // (the kernels read the input rows 16 bytes at a time, and x a float at a time)
    if (((uintptr_t)d_normed & 15) != 0 || ((uintptr_t)d_x & 3) != 0) {
        set_err("the input rows must start on a 16-byte boundary and x on a 4-byte one");
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
    // one token on the one-token kernel's shapes: decode.cuh
    const bool dec1 = fused && m->dec1_ok && !S.ext &&
                      trx_dec1_takes(c.gate_type, c.down_type, c.router_type, S.H, S.F, S.E, S.k, T, m->grid_fused, false);
    // a few tokens on those shapes: one launch of it a token. Each token's arithmetic is the one-token call's, so
    // the outputs are the same bits; the fused kernel costs about 40 us a token at T = 8 against its 24. Not when
    // the call's dispatch permutation (offsets, place over every token) is asked for.
    const bool dec1seq = fused && T > 1 && T <= TRX_DC_SEQ_MAX && m->dec1_ok && !S.ext && w.out_offsets == nullptr &&
                         w.out_place == nullptr &&
                         trx_dec1_takes(c.gate_type, c.down_type, c.router_type, S.H, S.F, S.E, S.k, 1, m->grid_fused,
                                        false);
    if (norm_src) {
        // short fused calls normalise inside the kernel when the rows fit the stage area beside the router's staging
        const bool inside = ((dec1 || dec1seq) && ((uintptr_t)norm_src & 15) == 0) ||
                            (fused && T <= TRX_FU_LOCAL_PREP && ((uintptr_t)norm_src & 15) == 0 &&
                             trx_fu_norm_off(T, S.H, E) + (size_t)T * S.H * 4 <=
                                 trx_fused_layout(c.gate_type, c.down_type, S.H, S.F, T, S.k, sg, sd, E, m->grid_fused).bars);
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
        if (dec1 && (!S.norm_in || ((uintptr_t)d_normed & 15) == 0))
            return launch_dec1(m, layer, L, S, d_normed, w, d_x, ffn, epoch, st);
        if (dec1seq && (!S.norm_in || ((uintptr_t)d_normed & 15) == 0)) {
            const int64_t H = S.H;
            for (int t = 0; t < T; t++) {
                TrxWork wt = w;
                wt.host_done = t == T - 1 ? done : nullptr; // the last launch posts the call's epoch
                if (wt.out_logits) wt.out_logits += (int64_t)t * E;
                if (wt.out_sel_id) {
                    wt.out_sel_id += (int64_t)t * S.k;
                    wt.out_sel_w += (int64_t)t * S.k;
                }
                if (wt.out_normed) wt.out_normed += t * H;
                if (launch_dec1(m, layer, L, S, d_normed + t * H, wt, d_x + t * H, ffn ? ffn + t * H : nullptr, epoch,
                                st) != 0)
                    return -1;
            }
            return 0;
        }
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
        set_err("this context has no tensor-core road (its weight types have no converter)");
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
        // the input rows by one copy-engine transfer (with the ffn_norm, of x: the norm reads a device copy of x,
        // which beats every CTA reading all of x over the link). (A variant in which the one-token kernel read a
        // pinned normed itself, each CTA its share over the link, published to the others as tagged words, measured
        // 46 us a call against 39.5: the gather of the whole row in every CTA costs more than the transfer.)
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
        set_err("%s (device error flag %d)", err_flag_what(flag), flag);
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
        set_err("%s (device error flag %d)", err_flag_what(flag), flag);
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

#include "capi_loader.inc"

#include "capi_ep.inc"

#include "capi_attention.inc"

#include "capi_kernel_level.inc"
