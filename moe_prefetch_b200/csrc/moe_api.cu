// moe_api.cu -- the C ABI of libmoeb200.so (include/moeb200.h): context,
// device allocation, weight registration, the hot-path launches, the cache
// step with its copy-stream uploader, and the ExpertCache prototype API.
#include "moeb200.h"
#include "moe_kernels.h"
#include "moe_planner.h"

#include <chrono>
#include <memory>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <list>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

using namespace moe;

namespace {

struct LayerMem {
    uint8_t *slab = nullptr;          // gate | up | down for (ns + 1) slots
    uint8_t *gate = nullptr, *up = nullptr, *down = nullptr;
    const uint8_t *hgate = nullptr, *hup = nullptr, *hdown = nullptr;   // device aliases
    const void *hgate_user = nullptr, *hup_user = nullptr, *hdown_user = nullptr;
    bool registered[3] = {false, false, false};
    int32_t ns = 0;
    uint8_t *shared = nullptr;        // shared expert: gate | up | down (n_shared == 1)
    uint8_t *sgate = nullptr, *sup = nullptr, *sdown = nullptr;
    bool shared_set = false;
};

}  // namespace

struct moe_ctx {
    moe_cfg cfg{};
    std::vector<int32_t> ns;           // per layer
    std::vector<int32_t> slot_off;
    int32_t sum_ns = 0;
    int64_t gate_bytes = 0, down_bytes = 0;
    std::vector<LayerMem> L;
    float *router = nullptr;           // [L][E][H]
    float *router_t = nullptr;         // [L][H][E]
    // slot state (device)
    void *state_mem = nullptr;
    SlotState st{};
    int32_t *d_ns = nullptr, *d_slot_off = nullptr;
    // decode
    LayerDesc *d_layers = nullptr;
    int32_t *d_part = nullptr;         // gu_r0 | gu_r1 | dn_h0 | dn_h1
    int grid = 0;
    DecodeParams dp{};
    float *resid = nullptr, *logits = nullptr, *act = nullptr;
    long long *acc = nullptr;   // decode router accumulators
    unsigned *bar = nullptr;
    unsigned *ready = nullptr;         // decode per-rank activation signals
    int *abort_flag = nullptr, *err = nullptr;
    // scratch for moe_layer_forward / moe_decode_host
    int32_t *s_ids = nullptr;
    float *s_w = nullptr, *s_io = nullptr;
    float *s_act = nullptr;            // per-pair fp32 activations, or the grouped path's Q8_1 scratch
    int s_cap_tok = 0, s_io_cap = 0;
    // grouping of the routed pairs by expert (n_tok > 1) and the unweighted
    // per-pair down rows [P][n_embd]
    int32_t *s_group = nullptr;
    GroupBufs grp{};
    float *s_ypair = nullptr;
    // expert parallelism over peer memory: this rank's mailbox (exported with
    // CUDA IPC), the other ranks' mailboxes opened in this process, the
    // device table of all world bases, the owner's y rows, the epoch
    EpMail ep{};
    uint8_t *ep_mail = nullptr;
    std::vector<uint8_t *> ep_open;    // opened peer mailboxes (closed at destroy)
    uint8_t **ep_peer = nullptr;       // device [world]
    float *ep_y = nullptr;             // [world * cap][n_embd]
    unsigned long long *ep_epoch = nullptr;   // [0] the exchange epoch, [1] the push kernel's CTA count
    bool ep_connected = false;
    // tensor-core GEMM operand tiles (fp16)
    void *s_gemm = nullptr;
    int s_gemm_cap_tok = 0;
    // uploader
    cudaStream_t copy_stream = nullptr;
    cudaEvent_t ev_step = nullptr, ev_copy = nullptr;
    bool copies_pending = false;
    int32_t *h_jobs = nullptr;         // mapped pinned [(host_cap + 1) * 4]
    int jobs_issued = 0;               // early issue: jobs of this step already copying
    // host callbacks (moe_set_predictor / moe_set_observe_hook)
    moe_predict_fn predict = nullptr;
    void *predict_ud = nullptr;
    moe_observe_fn obs_hook = nullptr;
    void *obs_ud = nullptr;
    int32_t *d_pred = nullptr;         // device [64]: the predictor's ids
    // LLAMA_MOE_EVICTOR: the model on the device (moe_set_evictor)
    int32_t *d_ev_index = nullptr;     // [L] in the slot-state block
    float *d_ev_model = nullptr;       // w, bias, prior
    // just-in-time streaming (moe_cfg.stream): the planner and its jobs
    struct StreamJob {
        int layer, expert, slot, plan, word;   // word: index of its pinned table word
        bool cancelled;
    };
    std::unique_ptr<moe_planner> planner;
    std::vector<StreamJob> sjobs;
    int stream_seen = 0;               // entries of the mapped job list examined
    int32_t *h_words = nullptr;        // pinned: the slot value of each streamed job's table word
    int32_t *d_cancel = nullptr;       // device scratch: (layer, expert, slot) to cancel
    float *d_scores = nullptr;         // device [2][E] lookahead scores
    int32_t *d_ahead = nullptr;        // device [2][16] + [2]: the lookahead's picks
    double tau_ns = 103000.0;          // time per layer, running estimate
    uint64_t last_call_ns = 0;
    int last_layer = -1;
    uint64_t free_at_ns = 0;           // when the copy engine runs out of queued bytes
    uint64_t sst[MOE_STREAM_STAT_COUNT] = {};
    int32_t *d_jobs_alias = nullptr;
    uint64_t upload_bytes = 0;
    uint64_t upload_ns = 0;          // time the copy stream spent on step uploads
    cudaEvent_t ev_up0 = nullptr, ev_up1 = nullptr;   // around the last step's uploads
    bool up_timed = false;           // ev_up0/ev_up1 hold an unharvested pair
    std::string err_msg;
};

static int fail(moe_ctx *c, int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    if (c) c->err_msg = buf;
    else fprintf(stderr, "moeb200: %s\n", buf);
    return code;
}

#define CK(call)                                                                               \
    do {                                                                                       \
        cudaError_t e_ = (call);                                                               \
        if (e_ != cudaSuccess)                                                                 \
            return fail(c, MOE_ERR_CUDA, "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                        __FILE__, __LINE__);                                                   \
    } while (0)

static int64_t row_bytes(int type, int n) {
    return (int64_t)(n / MOE_QK) * (type == MOE_QTYPE_Q6_K ? MOE_Q6K_BYTES : MOE_Q4K_BYTES);
}

static size_t al256(size_t v) { return (v + 255) & ~size_t(255); }

// ---------------------------------------------------------------------------
// lifetime
// ---------------------------------------------------------------------------

extern "C" int moe_create(const moe_cfg *cfg, moe_ctx **out) {
    if (!cfg || !out) return fail(nullptr, MOE_ERR_ARG, "moe_create: null argument");
    *out = nullptr;
    moe_ctx *c = new moe_ctx();
    c->cfg = *cfg;
    moe_cfg &g = c->cfg;
    g.slot_profile = nullptr;
    if (g.max_inserts <= 0) g.max_inserts = 2;
    if (g.freeze) g.max_inserts = 0;
    if (g.admit_window <= 0) g.admit_window = 8;
    if (g.admit_half <= 0) g.admit_half = 64;
    auto bad = [&](int code, const char *m) {
        fprintf(stderr, "moeb200: moe_create: %s\n", m);
        delete c;
        return code;
    };
    if (g.n_layers <= 0 || g.n_expert <= 0 || g.n_used <= 0 || g.n_embd <= 0 || g.n_ff <= 0)
        return bad(MOE_ERR_ARG, "non-positive shape");
    if (g.n_expert != 32 && g.n_expert != 64 && g.n_expert != 128 && g.n_expert != 256)
        return bad(MOE_ERR_UNSUPPORTED, "n_expert must be 32, 64, 128 or 256");
    if (g.n_used > 8 || g.n_used > g.n_expert) return bad(MOE_ERR_UNSUPPORTED, "n_used must be <= 8");
    if (g.n_embd != 2048) return bad(MOE_ERR_UNSUPPORTED, "n_embd must be 2048 in this build");
    if (g.n_ff % 256 || g.n_ff > 1024) return bad(MOE_ERR_UNSUPPORTED, "n_ff must be a multiple of 256, <= 1024");
    if (g.down_type != MOE_QTYPE_Q6_K && g.down_type != MOE_QTYPE_Q4_K)
        return bad(MOE_ERR_UNSUPPORTED, "down_type must be Q6_K or Q4_K");
    if (g.predict_top <= 0) g.predict_top = 3;
    if (g.stream && !g.early_issue) return bad(MOE_ERR_ARG, "streaming needs early issue");
    if (g.stream_per_layer <= 0) g.stream_per_layer = 4;
    if (g.stream_per_layer > 16) return bad(MOE_ERR_ARG, "stream_per_layer must be <= 16");
    if (g.stream_reserve < 0) return bad(MOE_ERR_ARG, "stream_reserve must be >= 0");
    if (g.stream_gbps <= 0.0f) g.stream_gbps = 45.7f;
    if (g.stream_topk <= 0) g.stream_topk = 8;
    if (g.stream_topk > 16) return bad(MOE_ERR_ARG, "stream_topk must be <= 16");
    if (g.predict_top > 64) return bad(MOE_ERR_ARG, "predict_top must be <= 64");
    if (g.admit_mode < 0 || g.admit_mode > 2) return bad(MOE_ERR_ARG, "admit_mode");
    if (g.n_shared < 0 || g.n_shared > 1) return bad(MOE_ERR_UNSUPPORTED, "n_shared must be 0 or 1");
    if (g.n_slots <= 0 && !cfg->slot_profile) return bad(MOE_ERR_ARG, "n_slots must be > 0");
    c->ns.resize(g.n_layers);
    c->slot_off.resize(g.n_layers);
    for (int l = 0; l < g.n_layers; ++l) {
        const int ns = cfg->slot_profile && cfg->slot_profile[l] > 0 ? cfg->slot_profile[l] : g.n_slots;
        if (ns <= 0 || ns > 4096) return bad(MOE_ERR_ARG, "slots per layer out of range");
        c->ns[l] = ns;
        c->slot_off[l] = c->sum_ns;
        c->sum_ns += ns;
    }
    *out = c;
    if (cudaSetDevice(g.device) != cudaSuccess) {
        delete c;
        *out = nullptr;
        return fail(nullptr, MOE_ERR_CUDA, "cudaSetDevice(%d) failed", g.device);
    }
    const int L = g.n_layers, E = g.n_expert, H = g.n_embd, I = g.n_ff, K = g.n_used;
    c->gate_bytes = row_bytes(MOE_QTYPE_Q4_K, H) * I;
    c->down_bytes = row_bytes(g.down_type, I) * H;
    c->L.resize(L);
    auto cleanup_fail = [&](int code) {
        moe_destroy(c);
        *out = nullptr;
        return code;
    };
    // slabs
    for (int l = 0; l < L; ++l) {
        LayerMem &m = c->L[l];
        m.ns = c->ns[l];
        const size_t gsz = al256((size_t)(m.ns + 1) * c->gate_bytes);
        const size_t dsz = al256((size_t)(m.ns + 1) * c->down_bytes + 64);
        if (cudaMalloc(&m.slab, 2 * gsz + dsz) != cudaSuccess) {
            fail(c, MOE_ERR_OOM, "slab allocation of layer %d (%zu bytes) failed", l, 2 * gsz + dsz);
            fprintf(stderr, "moeb200: %s\n", c->err_msg.c_str());
            return cleanup_fail(MOE_ERR_OOM);
        }
        m.gate = m.slab;
        m.up = m.slab + gsz;
        m.down = m.slab + 2 * gsz;
        cudaMemsetAsync(m.slab + 2 * gsz + (size_t)m.ns * c->down_bytes, 0,
                        (size_t)c->down_bytes + 64);   // dummy slot + pad
        if (g.n_shared) {
            const size_t sg = al256((size_t)c->gate_bytes), sd = al256((size_t)c->down_bytes + 64);
            if (cudaMalloc(&m.shared, 2 * sg + sd) != cudaSuccess) return cleanup_fail(MOE_ERR_OOM);
            cudaMemsetAsync(m.shared, 0, 2 * sg + sd);
            m.sgate = m.shared;
            m.sup = m.shared + sg;
            m.sdown = m.shared + 2 * sg;
        }
    }
    if (cudaMalloc(&c->router, sizeof(float) * (size_t)L * E * H) != cudaSuccess) return cleanup_fail(MOE_ERR_OOM);
    cudaMemset(c->router, 0, sizeof(float) * (size_t)L * E * H);
    if (cudaMalloc(&c->router_t, sizeof(float) * (size_t)L * E * H) != cudaSuccess) return cleanup_fail(MOE_ERR_OOM);
    cudaMemset(c->router_t, 0, sizeof(float) * (size_t)L * E * H);
    // slot state
    {
        const size_t LE = (size_t)L * E, S = (size_t)c->sum_ns;
        // jobs per layer: with early issue every job holds a slot of the layer's
        // pool, so at most its slot count
        size_t max_ns = 0;
        for (int l = 0; l < L; ++l) max_ns = std::max(max_ns, (size_t)c->ns[l]);
        const size_t MI = g.early_issue ? max_ns : (size_t)(g.max_inserts > 0 ? g.max_inserts : 1);
        std::vector<size_t> sz = {
            LE * 4,            // table
            S * 4,             // slot_expert
            S * 8,             // last_use
            S * 8,             // protect
            S,                 // in_flight
            LE * 4,            // pending
            (size_t)L * 4,     // n_pending
            g.admit_mode == 1 ? LE * 4 : 0,     // heat
            g.admit_mode == 2 ? LE * 8 : 0,     // miss_last
            g.admit_mode == 2 ? LE * 8 : 0,     // miss_prev
            g.use_heat_counts ? LE * 4 : 0,     // use_count
            (size_t)L * 8, (size_t)L * 8,       // n_hit, n_miss
            (size_t)G_COUNT * 8,                // globals
            (size_t)L * MI * 16,                // jobs
            (size_t)L * 4,                      // n_jobs
            (size_t)L * 4, (size_t)L * 4,       // ns, slot_off
            S * 4, (size_t)L * 4,               // free_slots, n_free
            LE * 4,                             // admitted
            (size_t)L * CUR_IDS * 4, (size_t)L * 4,  // cur_ids, n_cur
            (size_t)L * CUR_IDS * 4, (size_t)L * 4,  // prev_ids, n_prev (the evictor's)
            LE * 4, (size_t)L * 4                    // ev_scores, ev_index
        };
        size_t total = 0;
        std::vector<size_t> off;
        for (size_t s : sz) { off.push_back(total); total += al256(s); }
        if (cudaMalloc(&c->state_mem, total) != cudaSuccess) return cleanup_fail(MOE_ERR_OOM);
        cudaMemset(c->state_mem, 0, total);
        uint8_t *b = (uint8_t *)c->state_mem;
        SlotState &st = c->st;
        st.n_layers = L; st.n_expert = E; st.max_inserts = g.max_inserts;
        st.admit_mode = g.admit_mode; st.admit_window = g.admit_window; st.admit_half = g.admit_half;
        st.admit_floor = g.admit_floor; st.cache_prior = g.cache_prior;
        st.spec_probation = g.spec_probation; st.batch_tables = g.batch_tables; st.freeze = g.freeze;
        st.table = (int32_t *)(b + off[0]);
        st.slot_expert = (int32_t *)(b + off[1]);
        st.last_use = (uint64_t *)(b + off[2]);
        st.protect = (uint64_t *)(b + off[3]);
        st.in_flight = (uint8_t *)(b + off[4]);
        st.pending = (int32_t *)(b + off[5]);
        st.n_pending = (int32_t *)(b + off[6]);
        st.heat = g.admit_mode == 1 ? (float *)(b + off[7]) : nullptr;
        st.miss_last = g.admit_mode == 2 ? (uint64_t *)(b + off[8]) : nullptr;
        st.miss_prev = g.admit_mode == 2 ? (uint64_t *)(b + off[9]) : nullptr;
        st.use_count = g.use_heat_counts ? (uint32_t *)(b + off[10]) : nullptr;
        st.n_hit = (uint64_t *)(b + off[11]);
        st.n_miss = (uint64_t *)(b + off[12]);
        st.g = (uint64_t *)(b + off[13]);
        st.jobs = (int32_t *)(b + off[14]);
        st.n_jobs = (int32_t *)(b + off[15]);
        c->d_ns = (int32_t *)(b + off[16]);
        c->d_slot_off = (int32_t *)(b + off[17]);
        st.ns = c->d_ns;
        st.slot_off = c->d_slot_off;
        st.job_cap = (int)MI;
        st.early_issue = g.early_issue;
        st.predict_top = g.predict_top;
        st.have_pred = 0;
        st.stream = g.stream;
        st.stream_reserve = g.stream ? g.stream_reserve : 0;
        // the mapped job list: with streaming, a slot given back and claimed
        // again takes a second entry before the step clears the list
        st.host_cap = L * (int)MI * (g.stream ? 4 : 1);
        st.free_slots = (int32_t *)(b + off[18]);
        st.n_free = (int32_t *)(b + off[19]);
        st.admitted = (int32_t *)(b + off[20]);
        st.cur_ids = (int32_t *)(b + off[21]);
        st.n_cur = (int32_t *)(b + off[22]);
        st.prev_ids = (int32_t *)(b + off[23]);
        st.n_prev = (int32_t *)(b + off[24]);
        st.ev_scores = (float *)(b + off[25]);
        c->d_ev_index = (int32_t *)(b + off[26]);
        st.ev_index = c->d_ev_index;
        st.have_evict = 0;
        st.ev_feat = 0;
        for (int q = 0; q < 4; ++q) st.ev_off[q] = -1;
        st.ev_w = st.ev_bias = st.ev_prior = nullptr;
        {   // every slot free; the lowest on top of each pool
            std::vector<int32_t> fs(S), nf(L);
            for (int l = 0; l < L; ++l) {
                for (int q = 0; q < c->ns[l]; ++q) fs[c->slot_off[l] + q] = c->ns[l] - 1 - q;
                nf[l] = c->ns[l];
            }
            cudaMemcpy(st.free_slots, fs.data(), 4 * S, cudaMemcpyHostToDevice);
            cudaMemcpy(st.n_free, nf.data(), 4 * (size_t)L, cudaMemcpyHostToDevice);
        }
        cudaMemcpy(c->d_ns, c->ns.data(), 4 * L, cudaMemcpyHostToDevice);
        cudaMemcpy(c->d_slot_off, c->slot_off.data(), 4 * L, cudaMemcpyHostToDevice);
        std::vector<int32_t> tbl((size_t)L * E), se(S, -1);
        for (int l = 0; l < L; ++l)
            for (int e = 0; e < E; ++e) tbl[(size_t)l * E + e] = c->ns[l];
        cudaMemcpy(st.table, tbl.data(), 4 * LE, cudaMemcpyHostToDevice);
        cudaMemcpy(st.slot_expert, se.data(), 4 * S, cudaMemcpyHostToDevice);
        if (st.miss_last) {
            cudaMemset(st.miss_last, 0xFF, LE * 8);
            cudaMemset(st.miss_prev, 0xFF, LE * 8);
        }
    }
    // decode partition + buffers
    {
        int dev_sms = 0;
        cudaDeviceGetAttribute(&dev_sms, cudaDevAttrMultiProcessorCount, g.device);
        // one CTA per SM; the partial-logit reduction reads at most 10 CTAs
        // per warp group, so at most 160 CTAs
        const int G = dev_sms > 0 ? std::min(dev_sms, 160) : 1;
        std::vector<int32_t> part(4 * (size_t)G);
        const int64_t R = (int64_t)(K + g.n_shared) * I;
        int gmax = 0, dmax = 0;
        for (int cc = 0; cc < G; ++cc) {
            part[cc] = (int32_t)(cc * R / G);
            part[G + cc] = (int32_t)((cc + 1) * R / G);
            part[2 * G + cc] = (int32_t)((int64_t)cc * H / G);
            part[3 * G + cc] = (int32_t)((int64_t)(cc + 1) * H / G);
            gmax = std::max(gmax, part[G + cc] - part[cc]);
            dmax = std::max(dmax, part[3 * G + cc] - part[2 * G + cc]);
        }
        DecodeParams &p = c->dp;
        p.n_layers = L; p.n_expert = E; p.k = K; p.n_embd = H; p.n_ff = I; p.down_type = g.down_type;
        p.kx = K + g.n_shared;
        p.gate_bytes = c->gate_bytes; p.down_bytes = c->down_bytes;
        p.gu_rows_max = gmax; p.dn_rows_max = dmax;
        decode_smem_layout(p, G);
        c->grid = G;
        if (cudaMalloc(&c->d_part, sizeof(int32_t) * part.size()) != cudaSuccess) return cleanup_fail(MOE_ERR_OOM);
        cudaMemcpy(c->d_part, part.data(), sizeof(int32_t) * part.size(), cudaMemcpyHostToDevice);
        p.gu_r0 = c->d_part; p.gu_r1 = c->d_part + G; p.dn_h0 = c->d_part + 2 * G; p.dn_h1 = c->d_part + 3 * G;
        if (cudaMalloc(&c->d_layers, sizeof(LayerDesc) * L) != cudaSuccess) return cleanup_fail(MOE_ERR_OOM);
        p.layers = c->d_layers;
        if (cudaMalloc(&c->resid, sizeof(float) * H) != cudaSuccess ||
            cudaMalloc(&c->logits, sizeof(float) * 256) != cudaSuccess ||
            cudaMalloc(&c->acc, sizeof(long long) * 2 * (size_t)(E + 1) * moe::ACC_LINE) != cudaSuccess ||
            cudaMalloc(&c->act, sizeof(float) * (size_t)MOE_KMAX * I) != cudaSuccess ||
            cudaMalloc(&c->bar, 64) != cudaSuccess || cudaMalloc(&c->abort_flag, 64) != cudaSuccess ||
            cudaMalloc(&c->ready, sizeof(unsigned) * MOE_KMAX * moe::READY_STRIDE) != cudaSuccess ||
            cudaMalloc(&c->err, 64) != cudaSuccess)
            return cleanup_fail(MOE_ERR_OOM);
        cudaMemset(c->err, 0, 64);
        p.resid = c->resid; p.logits = c->logits; p.act = c->act; p.bar = c->bar; p.ready = c->ready;
        // producers of each rank's activations: the CTAs whose gate/up range
        // [r0, r1) of the flattened (rank, row) space meets that rank
        for (int q = 0; q < MOE_KMAX; ++q) p.n_prod[q] = 0;
        for (int cc = 0; cc < G; ++cc) {
            const int a0 = part[cc], a1 = part[G + cc];
            if (a1 > a0)
                for (int q = a0 / I; q <= (a1 - 1) / I && q < MOE_KMAX; ++q) p.n_prod[q] += 1;
        }
        p.acc = c->acc;
        p.abort_flag = c->abort_flag; p.err = c->err; p.st = c->st;
        p.observe = 1; p.delta = g.cache_prior; p.rms_eps = 1e-6f;
        p.wait_ns = MOE_TIMEOUT_NS; p.starve = 0; p.spec = 1;
    }
    // uploader
    {
        const size_t HC = (size_t)c->st.host_cap;
        const size_t nb = (HC + 1) * 4 * sizeof(int32_t);
        if (cudaHostAlloc((void **)&c->h_jobs, nb, cudaHostAllocMapped) != cudaSuccess) return cleanup_fail(MOE_ERR_OOM);
        memset(c->h_jobs, 0, nb);
        if (cudaHostGetDevicePointer((void **)&c->d_jobs_alias, c->h_jobs, 0) != cudaSuccess) return cleanup_fail(MOE_ERR_CUDA);
        // the device side writes jobs there (at the step, or at observation
        // with early issue); the count follows the host_cap entries
        c->st.host_jobs = c->d_jobs_alias;
        c->st.host_njobs = c->d_jobs_alias + HC * 4;
        c->dp.st = c->st;
        if (cudaMalloc(&c->d_pred, 64 * sizeof(int32_t)) != cudaSuccess) return cleanup_fail(MOE_ERR_OOM);
        if (g.stream) {
            c->planner.reset(new moe_planner(512 * 1024));
            if (cudaHostAlloc((void **)&c->h_words, sizeof(int32_t) * HC, cudaHostAllocDefault) != cudaSuccess ||
                cudaMalloc(&c->d_cancel, sizeof(int32_t) * 3 * HC) != cudaSuccess ||
                cudaMalloc(&c->d_scores, sizeof(float) * 2 * (size_t)E) != cudaSuccess ||
                cudaMalloc(&c->d_ahead, sizeof(int32_t) * 36) != cudaSuccess)
                return cleanup_fail(MOE_ERR_OOM);
        }
        if (cudaStreamCreateWithFlags(&c->copy_stream, cudaStreamNonBlocking) != cudaSuccess ||
            cudaEventCreateWithFlags(&c->ev_step, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&c->ev_copy, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreate(&c->ev_up0) != cudaSuccess || cudaEventCreate(&c->ev_up1) != cudaSuccess)
            return cleanup_fail(MOE_ERR_CUDA);
    }
    if (cudaDeviceSynchronize() != cudaSuccess) return cleanup_fail(MOE_ERR_CUDA);
    return MOE_OK;
}

extern "C" void moe_destroy(moe_ctx *c) {
    if (!c) return;
    cudaSetDevice(c->cfg.device);
    if (c->copy_stream) cudaStreamSynchronize(c->copy_stream);
    cudaDeviceSynchronize();
    for (uint8_t *p : c->ep_open) cudaIpcCloseMemHandle(p);
    cudaFree(c->ep_mail);
    cudaFree(c->ep_peer);
    cudaFree(c->ep_y);
    cudaFree(c->ep_epoch);
    for (auto &m : c->L) {
        if (m.slab) cudaFree(m.slab);
        if (m.shared) cudaFree(m.shared);
        for (int i = 0; i < 3; ++i) {
            const void *p = i == 0 ? m.hgate_user : i == 1 ? m.hup_user : m.hdown_user;
            if (m.registered[i] && p) cudaHostUnregister(const_cast<void *>(p));
        }
    }
    cudaFree(c->router);
    cudaFree(c->router_t);
    cudaFree(c->acc);
    cudaFree(c->state_mem);
    cudaFree(c->d_layers);
    cudaFree(c->d_part);
    cudaFree(c->resid);
    cudaFree(c->logits);
    cudaFree(c->act);
    cudaFree(c->bar);
    cudaFree(c->ready);
    cudaFree(c->abort_flag);
    cudaFree(c->err);
    cudaFree(c->s_ids);
    cudaFree(c->s_w);
    cudaFree(c->s_act);
    cudaFree(c->s_io);
    cudaFree(c->s_group);
    cudaFree(c->s_ypair);
    cudaFree(c->s_gemm);
    if (c->h_jobs) cudaFreeHost(c->h_jobs);
    if (c->ev_step) cudaEventDestroy(c->ev_step);
    if (c->ev_copy) cudaEventDestroy(c->ev_copy);
    if (c->ev_up0) cudaEventDestroy(c->ev_up0);
    cudaFree(c->d_pred);
    if (c->h_words) cudaFreeHost(c->h_words);
    cudaFree(c->d_cancel);
    cudaFree(c->d_ev_model);
    cudaFree(c->d_scores);
    cudaFree(c->d_ahead);
    if (c->ev_up1) cudaEventDestroy(c->ev_up1);
    if (c->copy_stream) cudaStreamDestroy(c->copy_stream);
    delete c;
}

extern "C" const char *moe_last_error(const moe_ctx *c) { return c ? c->err_msg.c_str() : ""; }

extern "C" int moe_get_layer(moe_ctx *c, int layer, moe_layer_info *out) {
    if (!c || !out || layer < 0 || layer >= c->cfg.n_layers) return fail(c, MOE_ERR_ARG, "moe_get_layer: bad layer");
    LayerMem &m = c->L[layer];
    out->gate_c = m.gate;
    out->up_c = m.up;
    out->down_c = m.down;
    out->dev_table = c->st.table + (size_t)layer * c->cfg.n_expert;
    out->gate_bytes = c->gate_bytes;
    out->down_bytes = c->down_bytes;
    out->n_slots = m.ns;
    out->il = layer;
    return MOE_OK;
}

// ---------------------------------------------------------------------------
// weights
// ---------------------------------------------------------------------------

static int refresh_layer_desc(moe_ctx *c, int layer) {
    LayerMem &m = c->L[layer];
    LayerDesc d{};
    d.router_w = c->router + (size_t)layer * c->cfg.n_expert * c->cfg.n_embd;
    d.router_t = c->router_t + (size_t)layer * c->cfg.n_expert * c->cfg.n_embd;
    d.gate = m.gate; d.up = m.up; d.down = m.down;
    d.hgate = m.hgate; d.hup = m.hup; d.hdown = m.hdown;
    d.table = c->st.table + (size_t)layer * c->cfg.n_expert;
    d.sgate = m.sgate; d.sup = m.sup; d.sdown = m.sdown;
    d.ns = m.ns;
    CK(cudaMemcpy(c->d_layers + layer, &d, sizeof(d), cudaMemcpyHostToDevice));
    return MOE_OK;
}

extern "C" int moe_set_shared_expert(moe_ctx *c, int layer, const void *gate, const void *up,
                                     const void *down) {
    if (!c || layer < 0 || layer >= c->cfg.n_layers || !gate || !up || !down)
        return fail(c, MOE_ERR_ARG, "moe_set_shared_expert: bad argument");
    if (!c->cfg.n_shared) return fail(c, MOE_ERR_STATE, "moe_set_shared_expert: the context has n_shared = 0");
    CK(cudaSetDevice(c->cfg.device));
    LayerMem &m = c->L[layer];
    CK(cudaMemcpy(m.sgate, gate, (size_t)c->gate_bytes, cudaMemcpyDefault));
    CK(cudaMemcpy(m.sup, up, (size_t)c->gate_bytes, cudaMemcpyDefault));
    CK(cudaMemcpy(m.sdown, down, (size_t)c->down_bytes, cudaMemcpyDefault));
    m.shared_set = true;
    return refresh_layer_desc(c, layer);
}

extern "C" int moe_set_router(moe_ctx *c, int layer, const float *w) {
    if (!c || !w || layer < 0 || layer >= c->cfg.n_layers) return fail(c, MOE_ERR_ARG, "moe_set_router: bad argument");
    CK(cudaSetDevice(c->cfg.device));
    const size_t n = (size_t)c->cfg.n_expert * c->cfg.n_embd;
    CK(cudaMemcpy(c->router + (size_t)layer * n, w, n * sizeof(float), cudaMemcpyDefault));
    CK(launch_transpose(c->router + (size_t)layer * n, c->router_t + (size_t)layer * n,
                        c->cfg.n_expert, c->cfg.n_embd, 0));
    CK(cudaDeviceSynchronize());
    return refresh_layer_desc(c, layer);
}

static int register_host(moe_ctx *c, const void *p, size_t bytes, const uint8_t **dev, bool *registered) {
    cudaPointerAttributes at{};
    cudaError_t e = cudaPointerGetAttributes(&at, p);
    if (e != cudaSuccess) { (void)cudaGetLastError(); at.type = cudaMemoryTypeUnregistered; }
    if (at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged) {
        *dev = (const uint8_t *)p;   // already device-visible
        *registered = false;
        return MOE_OK;
    }
    if (at.type == cudaMemoryTypeUnregistered) {
        e = cudaHostRegister(const_cast<void *>(p), bytes, cudaHostRegisterPortable | cudaHostRegisterMapped);
        if (e != cudaSuccess) {
            (void)cudaGetLastError();
            return fail(c, MOE_ERR_CUDA, "cudaHostRegister of %zu bytes failed: %s", bytes, cudaGetErrorString(e));
        }
        *registered = true;
    } else {
        *registered = false;
    }
    void *d = nullptr;
    e = cudaHostGetDevicePointer(&d, const_cast<void *>(p), 0);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        return fail(c, MOE_ERR_CUDA, "cudaHostGetDevicePointer failed: %s", cudaGetErrorString(e));
    }
    *dev = (const uint8_t *)d;
    return MOE_OK;
}

extern "C" int moe_set_expert_weights(moe_ctx *c, int layer, const void *gate, const void *up,
                                      const void *down) {
    if (!c || layer < 0 || layer >= c->cfg.n_layers || !gate || !up || !down)
        return fail(c, MOE_ERR_ARG, "moe_set_expert_weights: bad argument");
    if (((uintptr_t)gate | (uintptr_t)up | (uintptr_t)down) & 15)
        return fail(c, MOE_ERR_ARG, "expert weights must be 16-byte aligned");
    CK(cudaSetDevice(c->cfg.device));
    LayerMem &m = c->L[layer];
    const size_t E = (size_t)c->cfg.n_expert;
    const void *src[3] = {gate, up, down};
    const void **user[3] = {&m.hgate_user, &m.hup_user, &m.hdown_user};
    const uint8_t **dev[3] = {&m.hgate, &m.hup, &m.hdown};
    for (int i = 0; i < 3; ++i) {
        if (m.registered[i] && *user[i]) {
            cudaHostUnregister(const_cast<void *>(*user[i]));
            m.registered[i] = false;
        }
        const size_t bytes = E * (size_t)(i == 2 ? c->down_bytes : c->gate_bytes);
        const int r = register_host(c, src[i], bytes, dev[i], &m.registered[i]);
        if (r != MOE_OK) return r;
        *user[i] = src[i];
    }
    return refresh_layer_desc(c, layer);
}

extern "C" int moe_place(moe_ctx *c, int layer, const int32_t *slot_expert, int copy) {
    if (!c || !slot_expert || layer < 0 || layer >= c->cfg.n_layers) return fail(c, MOE_ERR_ARG, "moe_place: bad argument");
    CK(cudaSetDevice(c->cfg.device));
    LayerMem &m = c->L[layer];
    const int E = c->cfg.n_expert, ns = m.ns, so = c->slot_off[layer];
    std::vector<int32_t> cur(ns), tbl(E, ns);
    std::vector<uint8_t> seen(E, 0);
    CK(cudaMemcpy(cur.data(), c->st.slot_expert + so, 4 * ns, cudaMemcpyDeviceToHost));
    for (int s = 0; s < ns; ++s) {
        const int e = slot_expert[s];
        if (e < -1 || e >= E) return fail(c, MOE_ERR_ARG, "moe_place: expert %d out of range", e);
        if (e >= 0) {
            if (seen[e]) return fail(c, MOE_ERR_ARG, "moe_place: expert %d placed twice", e);
            seen[e] = 1;
            tbl[e] = s;
        }
    }
    if (copy) {
        if (!m.hgate) return fail(c, MOE_ERR_STATE, "moe_place: host weights of layer %d not registered", layer);
        for (int s = 0; s < ns; ++s) {
            const int e = slot_expert[s];
            if (e < 0 || cur[s] == e) continue;
            CK(cudaMemcpy(m.gate + (size_t)s * c->gate_bytes, m.hgate_user ? (const uint8_t *)m.hgate_user + (size_t)e * c->gate_bytes : m.hgate + (size_t)e * c->gate_bytes, c->gate_bytes, cudaMemcpyDefault));
            CK(cudaMemcpy(m.up + (size_t)s * c->gate_bytes, (const uint8_t *)m.hup_user + (size_t)e * c->gate_bytes, c->gate_bytes, cudaMemcpyDefault));
            CK(cudaMemcpy(m.down + (size_t)s * c->down_bytes, (const uint8_t *)m.hdown_user + (size_t)e * c->down_bytes, c->down_bytes, cudaMemcpyDefault));
            c->upload_bytes += 2 * c->gate_bytes + c->down_bytes;
        }
    }
    std::vector<uint8_t> zero(ns, 0);
    CK(cudaMemcpy(c->st.slot_expert + so, slot_expert, 4 * ns, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(c->st.table + (size_t)layer * E, tbl.data(), 4 * E, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(c->st.in_flight + so, zero.data(), ns, cudaMemcpyHostToDevice));
    return MOE_OK;
}

// ---------------------------------------------------------------------------
// hot path
// ---------------------------------------------------------------------------

static int ensure_scratch(moe_ctx *c, int n_tok) {
    if (n_tok <= c->s_cap_tok) return MOE_OK;
    cudaFree(c->s_ids); cudaFree(c->s_w); cudaFree(c->s_act);
    cudaFree(c->s_group); cudaFree(c->s_ypair);
    c->s_ids = nullptr; c->s_w = nullptr; c->s_act = nullptr;
    c->s_group = nullptr; c->s_ypair = nullptr;
    const int K = c->cfg.n_used, KX = K + c->cfg.n_shared, E = c->cfg.n_expert + c->cfg.n_shared;
    const size_t P = (size_t)n_tok * KX;   // pairs, the shared expert's included
    // cnt [E] | off [E + 1] | pair_pos [P] | pos_pair [P] | tiles [E + P] | n_tiles [1]
    const size_t gints = (size_t)E + (E + 1) + P + P + (E + P) + 1;
    // s_ids / s_w: [n_tok][K] router outputs, then [n_tok][KX] with the shared pair
    if (cudaMalloc(&c->s_ids, sizeof(int32_t) * (size_t)n_tok * (K + KX)) != cudaSuccess ||
        cudaMalloc(&c->s_w, sizeof(float) * (size_t)n_tok * (K + KX)) != cudaSuccess ||
        cudaMalloc(&c->s_act, std::max(sizeof(float) * P * c->cfg.n_ff,
                                        grouped_scratch_bytes((int)P, c->cfg.n_embd, c->cfg.n_ff))) != cudaSuccess ||
        cudaMalloc(&c->s_group, sizeof(int32_t) * gints) != cudaSuccess ||
        cudaMalloc(&c->s_ypair, sizeof(float) * P * c->cfg.n_embd) != cudaSuccess) {
        c->s_cap_tok = 0;
        return fail(c, MOE_ERR_OOM, "scratch allocation for %d tokens failed", n_tok);
    }
    int32_t *g = c->s_group;
    c->grp.cnt = g; g += E;
    c->grp.off = g; g += E + 1;
    c->grp.pair_pos = g; g += P;
    c->grp.pos_pair = g; g += P;
    c->grp.tiles = g; g += E + P;
    c->grp.n_tiles = g;
    c->s_cap_tok = n_tok;
    return MOE_OK;
}

static ExpertSrc make_src(moe_ctx *c, int layer) {
    LayerMem &m = c->L[layer];
    ExpertSrc s{};
    s.gate = m.gate; s.up = m.up; s.down = m.down;
    s.hgate = m.hgate; s.hup = m.hup; s.hdown = m.hdown;
    s.table = c->st.table + (size_t)layer * c->cfg.n_expert;
    s.sgate = m.sgate; s.sup = m.sup; s.sdown = m.sdown;
    s.gate_bytes = c->gate_bytes; s.down_bytes = c->down_bytes;
    s.ns = m.ns; s.n_expert = c->cfg.n_expert;
    return s;
}

// The pairs the expert kernels see: the routed ids/w, or with a shared
// expert the routed pairs plus (n_expert, 1) per token, built in the second
// half of the id/weight scratch.  Sets *k_out to the pairs per token.
static int expert_pairs(moe_ctx *c, const int32_t *ids, const float *w, int n_tok,
                        cudaStream_t s, const int32_t **ids_e, const float **w_e, int *k_out) {
    const moe_cfg &g = c->cfg;
    *ids_e = ids;
    *w_e = w;
    *k_out = g.n_used;
    if (!g.n_shared) return MOE_OK;
    int32_t *ix = c->s_ids + (size_t)n_tok * g.n_used;
    float *wx = c->s_w + (size_t)n_tok * g.n_used;
    CK(launch_append_shared(ids, w, n_tok, g.n_used, g.n_expert, ix, wx, s));
    *ids_e = ix;
    *w_e = wx;
    *k_out = g.n_used + 1;
    return MOE_OK;
}

static int check_shared(moe_ctx *c, int layer) {
    if (c->cfg.n_shared && !c->L[layer].shared_set)
        return fail(c, MOE_ERR_STATE, "the shared expert of layer %d is not set", layer);
    return MOE_OK;
}

// After a single-token layer was observed (patches/0006:295-400, 0007:
// 271-321): the observe hook with the routed ids; with early issue and a
// predictor, the predictor's ids for the next layer go to k_issue_spec
// (speculative uploads); with early issue the new jobs' copies start now.
// Synchronises the stream only when one of these is on.
static int issue_early_copies(moe_ctx *c, cudaStream_t s);
static volatile int32_t *host_njobs(moe_ctx *c);

// ---- just-in-time streaming (patches/0010:951-1010 and its mover) -----------
// After each single-token layer L of the per-layer entry points, the
// lookahead applies the routers of L + 1 and L + 2 to L's input and claims
// pool slots for their best non-resident experts (k_ahead_claim: jobs of
// spec 2 in the device job lists and the mapped host list).  The host mover
// offers them to the planner with deadlines (now + (target - L) * tau -
// margin, tau the running time per layer) and sends them earliest deadline
// first in 512 KiB chunks on the copy stream, keeping about one layer's worth
// of bytes queued so that a more urgent job never waits behind much; after an
// expert's last chunk the same stream writes its 4-byte table word, so the
// expert's layer finds it resident if the word landed first.  A routed
// expert reads the same bytes from its slot or from host memory, so outputs
// do not depend on when a word lands; the cache prior counts published
// residency only (prior_resident).  Jobs the planner drops (late, or their
// layer read its table first) give their slot back (k_stream_cancel); the
// step publishes the rest with every other job.

static uint64_t now_ns() {
    return (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
               std::chrono::steady_clock::now().time_since_epoch()).count();
}

// Gives back the slot of every streamed job the planner dropped or refused
// (a dropped job's partial copies land in a slot nothing references; later
// copies into that slot are queued behind them on the same stream).
static int stream_cancel_dropped(moe_ctx *c, cudaStream_t s) {
    std::vector<int32_t> q;
    for (auto &j : c->sjobs) {
        if (j.cancelled || (j.plan >= 0 && !c->planner->get(j.plan).dropped)) continue;
        j.cancelled = true;
        q.push_back(j.layer); q.push_back(j.expert); q.push_back(j.slot);
        c->sst[7]++;
    }
    if (q.empty()) return MOE_OK;
    CK(cudaMemcpyAsync(c->d_cancel, q.data(), sizeof(int32_t) * q.size(), cudaMemcpyHostToDevice, s));
    CK(launch_stream_cancel(c->st, c->d_cancel, (int)q.size() / 3, s));
    CK(cudaStreamSynchronize(s));   // q is a host temporary
    return MOE_OK;
}

// Copies bytes [off, off + len) of expert e's (gate | up | down) into slot
// `slot` of layer l, on the copy stream.
static int stream_copy_range(moe_ctx *c, int l, int e, int slot, size_t off, size_t len) {
    LayerMem &m = c->L[l];
    const size_t gb = (size_t)c->gate_bytes, db = (size_t)c->down_bytes;
    const struct { uint8_t *dst; const uint8_t *src; size_t n; } part[3] = {
        {m.gate + (size_t)slot * gb, (const uint8_t *)m.hgate_user + (size_t)e * gb, gb},
        {m.up + (size_t)slot * gb, (const uint8_t *)m.hup_user + (size_t)e * gb, gb},
        {m.down + (size_t)slot * db, (const uint8_t *)m.hdown_user + (size_t)e * db, db}};
    size_t base = 0;
    for (const auto &p : part) {
        const size_t a = std::max(off, base), b = std::min(off + len, base + p.n);
        if (a < b)
            CK(cudaMemcpyAsync(p.dst + (a - base), p.src + (a - base), b - a, cudaMemcpyHostToDevice,
                               c->copy_stream));
        base += p.n;
    }
    return MOE_OK;
}

// Sends chunks while the copy engine holds less than about one layer's
// worth of bytes (tau at the configured rate, at least 1 MiB).
static int stream_drain(moe_ctx *c, cudaStream_t s) {
    const uint64_t t = now_ns();
    const double rate = (double)c->cfg.stream_gbps;   // GB/s = bytes per ns
    uint64_t fa = std::max(t, c->free_at_ns);
    const uint64_t horizon = t + (uint64_t)std::max(c->tau_ns, (double)(1u << 20) / rate);
    std::vector<int> of_plan(c->planner->size(), -1);
    for (int q = 0; q < (int)c->sjobs.size(); ++q)
        if (c->sjobs[q].plan >= 0) of_plan[c->sjobs[q].plan] = q;
    moe_planner::chunk ch;
    bool sent = false;
    while (fa < horizon && c->planner->next(fa, rate, -1, ch)) {
        const moe_ctx::StreamJob sj = c->sjobs[of_plan[ch.job]];
        int r = stream_copy_range(c, sj.layer, sj.expert, sj.slot, ch.offset, ch.len);
        if (r != MOE_OK) return r;
        if (ch.last) {
            CK(cudaMemcpyAsync(c->st.table + (size_t)sj.layer * c->cfg.n_expert + sj.expert,
                               c->h_words + sj.word, sizeof(int32_t), cudaMemcpyHostToDevice, c->copy_stream));
            c->sst[4]++;
        }
        fa += (uint64_t)((double)ch.len / rate);
        c->sst[2]++;
        c->sst[3] += ch.len;
        sent = true;
    }
    c->free_at_ns = fa;
    c->sst[5] = c->planner->n_drop_late;
    if (sent) {
        CK(cudaEventRecord(c->ev_copy, c->copy_stream));
        c->copies_pending = true;
    }
    return stream_cancel_dropped(c, s);
}

// Layer `layer` is about to read its table: its unsent jobs are of no use;
// the others may go on.
static int stream_enter(moe_ctx *c, int layer, cudaStream_t s) {
    const uint64_t t = now_ns();
    // time per layer from consecutive layers of one token (stream_take,
    // patches/0010:1466-1472: a 0.9 / 0.1 average of gaps in (10 us, 1 ms))
    if (c->last_layer >= 0 && layer == c->last_layer + 1 && t > c->last_call_ns) {
        const double dt = (double)(t - c->last_call_ns);
        if (dt > 10000.0 && dt < 1000000.0) c->tau_ns = 0.9 * c->tau_ns + 0.1 * dt;
    }
    c->last_layer = layer;
    c->last_call_ns = t;
    const uint64_t before = c->planner->n_drop_posted;
    c->planner->posted(layer);
    c->sst[6] += c->planner->n_drop_posted - before;
    return stream_drain(c, s);
}

// The lookahead after layer `layer` (x: its input), then the mover's work.
static int stream_after(moe_ctx *c, int layer, const float *x, cudaStream_t s) {
    const moe_cfg &g = c->cfg;
    const int n_targets = std::min(2, g.n_layers - 1 - layer);
    if (n_targets <= 0) return stream_drain(c, s);
    for (int l = layer + 1; l <= layer + n_targets; ++l)
        if (!c->L[l].hgate_user) return stream_drain(c, s);   // nothing to stream from
    CK(launch_ahead(c->st, c->router, x, layer + 1, n_targets, g.n_embd, g.stream_topk, g.stream_per_layer,
                    c->d_scores, c->d_ahead, c->d_ahead + 32, s));
    int32_t ahead[34];
    CK(cudaMemcpyAsync(ahead, c->d_ahead, sizeof(ahead), cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    c->sst[0]++;
    const uint64_t t = now_ns();
    const size_t bytes = 2 * (size_t)c->gate_bytes + (size_t)c->down_bytes;
    auto deadline_of = [&](int tl) {
        const double lead = (double)(tl - layer) * c->tau_ns;
        return t + (uint64_t)(lead > 5000.0 ? lead - 5000.0 : 0.0);   // 5 us margin
    };
    // candidates that already have a job: a nearer layer may tighten its deadline
    for (int tt = 0; tt < n_targets; ++tt) {
        const int nt = std::min(std::max(ahead[32 + tt], 0), 16);
        for (int i = 0; i < nt; ++i)
            for (const auto &j : c->sjobs)
                if (!j.cancelled && j.layer == layer + 1 + tt && j.expert == ahead[16 * tt + i])
                    c->planner->offer(j.layer, j.expert, bytes, deadline_of(j.layer));
    }
    const int nj = *host_njobs(c);
    for (int j = c->stream_seen; j < nj; ++j) {
        const int32_t *e = c->h_jobs + 4 * (size_t)j;
        if (e[3] != 2) continue;
        const int tl = e[0];
        const int plan = c->planner->offer(tl, e[1], bytes, deadline_of(tl));
        c->h_words[j] = e[2];
        c->sjobs.push_back({tl, e[1], e[2], plan, j, false});
        if (plan >= 0) c->sst[1]++;
    }
    c->stream_seen = nj;
    return stream_drain(c, s);
}

static int after_observe(moe_ctx *c, int layer, const int32_t *ids_dev, int n_ids, cudaStream_t s,
                         const float *x = nullptr) {
    const bool pred = c->cfg.early_issue && c->predict && layer + 1 < c->cfg.n_layers;
    if (!c->obs_hook && !pred && !c->cfg.early_issue) return MOE_OK;   // (streaming needs early issue)
    CK(cudaStreamSynchronize(s));
    int32_t cur[64];
    const int n = n_ids < 64 ? n_ids : 64;
    if (c->obs_hook || pred) CK(cudaMemcpy(cur, ids_dev, 4 * (size_t)n, cudaMemcpyDeviceToHost));
    if (c->obs_hook) c->obs_hook(c->obs_ud, layer, cur, 1, n);
    if (pred) {
        int32_t nprev[CUR_IDS];
        int n_nprev = 0;
        CK(cudaMemcpy(&n_nprev, c->st.n_cur + layer + 1, 4, cudaMemcpyDeviceToHost));
        n_nprev = std::min(std::max(n_nprev, 0), CUR_IDS);
        if (n_nprev)
            CK(cudaMemcpy(nprev, c->st.cur_ids + (size_t)(layer + 1) * CUR_IDS, 4 * (size_t)n_nprev,
                          cudaMemcpyDeviceToHost));
        int32_t top[64];
        const int k = c->cfg.predict_top;
        int nt = c->predict(c->predict_ud, layer, cur, n, nprev, n_nprev, top, k);
        nt = std::min(std::max(nt, 0), k);
        if (nt) CK(cudaMemcpy(c->d_pred, top, 4 * (size_t)nt, cudaMemcpyHostToDevice));
        CK(launch_issue_spec(c->st, layer + 1, c->d_pred, nt, s));
    }
    if (c->cfg.early_issue) {
        const int r = issue_early_copies(c, s);   // demand first: it is the most urgent
        if (r != MOE_OK || !c->cfg.stream || !x) return r;
        return stream_after(c, layer, x, s);
    }
    return MOE_OK;
}

extern "C" int moe_layer_forward(moe_ctx *c, int layer, const float *x, float *y, int n_tok,
                                 int32_t *ids, float *w, void *stream) {
    if (!c || !x || !y || n_tok <= 0 || layer < 0 || layer >= c->cfg.n_layers)
        return fail(c, MOE_ERR_ARG, "moe_layer_forward: bad argument");
    int r = check_shared(c, layer);
    if (r != MOE_OK) return r;
    CK(cudaSetDevice(c->cfg.device));
    if ((r = ensure_scratch(c, n_tok)) != MOE_OK) return r;
    cudaStream_t s = (cudaStream_t)stream;
    const moe_cfg &g = c->cfg;
    if (g.stream && n_tok == 1 && (r = stream_enter(c, layer, s)) != MOE_OK) return r;
    int32_t *ids_d = ids ? ids : c->s_ids;
    float *w_d = w ? w : c->s_w;
    const int32_t *table = c->st.table + (size_t)layer * g.n_expert;
    CK(launch_router(c->router + (size_t)layer * g.n_expert * g.n_embd, x, n_tok, g.n_expert, g.n_embd,
                     table, c->L[layer].ns, g.cache_prior, n_tok == 1 && g.cache_prior > 0.0f, g.n_used,
                     ids_d, w_d, nullptr, &c->st, n_tok == 1 ? layer : -1,
                     c->st.slot_expert + c->slot_off[layer], s));
    const int32_t *ids_e;
    const float *w_e;
    int kx;
    if ((r = expert_pairs(c, ids_d, w_d, n_tok, s, &ids_e, &w_e, &kx)) != MOE_OK) return r;
    // group the pairs by expert so that each expert's rows are read once per
    // tile of its tokens (bit-identical to the per-pair kernels); one token
    // takes the same path: its activations are quantised once per tile
    // instead of once per CTA of the per-pair down kernel
    CK(launch_group(ids_e, n_tok * kx, g.n_expert + g.n_shared, GROUP_TILE, c->grp, c->err, s));
    CK(launch_experts_grouped(make_src(c, layer), x, c->grp, n_tok, kx, g.n_embd, g.n_ff,
                              g.down_type, w_e, c->s_act, c->s_ypair, nullptr, y, c->err, s));
    return n_tok == 1 ? after_observe(c, layer, ids_d, g.n_used, s, x) : MOE_OK;
}

static int ensure_gemm_scratch(moe_ctx *c, int n_tok) {
    if (n_tok <= c->s_gemm_cap_tok) return MOE_OK;
    cudaFree(c->s_gemm);
    c->s_gemm = nullptr;
    const moe_cfg &g = c->cfg;
    const size_t halves = gemm_scratch_halves(g.n_expert + g.n_shared, n_tok * (g.n_used + g.n_shared),
                                              g.n_embd, g.n_ff);
    if (cudaMalloc(&c->s_gemm, 2 * halves) != cudaSuccess) {
        c->s_gemm_cap_tok = 0;
        return fail(c, MOE_ERR_OOM, "GEMM scratch allocation for %d tokens failed", n_tok);
    }
    c->s_gemm_cap_tok = n_tok;
    return MOE_OK;
}

extern "C" int moe_layer_forward_path(moe_ctx *c, int layer, const float *x, float *y, int n_tok,
                                      int32_t *ids, float *w, int path, void *stream) {
    if (!c || !x || !y || n_tok <= 0 || layer < 0 || layer >= c->cfg.n_layers)
        return fail(c, MOE_ERR_ARG, "moe_layer_forward_path: bad argument");
    const moe_cfg &g = c->cfg;
    const bool gemm_ok = g.down_type == MOE_QTYPE_Q6_K && g.n_ff % 128 == 0 && g.n_embd % 128 == 0;
    if (path == MOE_PATH_AUTO)
        path = gemm_ok && n_tok * g.n_used >= 4 * g.n_expert ? MOE_PATH_GEMM : MOE_PATH_GEMV;
    if (path == MOE_PATH_GEMV) return moe_layer_forward(c, layer, x, y, n_tok, ids, w, stream);
    if (path != MOE_PATH_GEMM) return fail(c, MOE_ERR_ARG, "moe_layer_forward_path: unknown path %d", path);
    if (!gemm_ok)
        return fail(c, MOE_ERR_UNSUPPORTED, "the GEMM path needs Q6_K down weights and n_ff, n_embd multiples of 128");
    int r = check_shared(c, layer);
    if (r != MOE_OK) return r;
    CK(cudaSetDevice(g.device));
    if ((r = ensure_scratch(c, n_tok)) != MOE_OK) return r;
    if ((r = ensure_gemm_scratch(c, n_tok)) != MOE_OK) return r;
    cudaStream_t s = (cudaStream_t)stream;
    if (g.stream && n_tok == 1 && (r = stream_enter(c, layer, s)) != MOE_OK) return r;
    int32_t *ids_d = ids ? ids : c->s_ids;
    float *w_d = w ? w : c->s_w;
    const int32_t *table = c->st.table + (size_t)layer * g.n_expert;
    CK(launch_router(c->router + (size_t)layer * g.n_expert * g.n_embd, x, n_tok, g.n_expert, g.n_embd,
                     table, c->L[layer].ns, g.cache_prior, n_tok == 1 && g.cache_prior > 0.0f, g.n_used,
                     ids_d, w_d, nullptr, &c->st, n_tok == 1 ? layer : -1,
                     c->st.slot_expert + c->slot_off[layer], s));
    const int32_t *ids_e;
    const float *w_e;
    int kx;
    if ((r = expert_pairs(c, ids_d, w_d, n_tok, s, &ids_e, &w_e, &kx)) != MOE_OK) return r;
    CK(launch_group(ids_e, n_tok * kx, g.n_expert + g.n_shared, GM_NT, c->grp, c->err, s));
    CK(launch_experts_gemm(make_src(c, layer), x, c->grp, n_tok, kx, g.n_embd, g.n_ff,
                           g.down_type, w_e, c->s_gemm, c->s_ypair, nullptr, y, c->err, s));
    return n_tok == 1 ? after_observe(c, layer, ids_d, g.n_used, s, x) : MOE_OK;
}

// ---- expert parallelism -------------------------------------------------------

extern "C" int moe_ep_route_pack(moe_ctx *c, int layer, const float *x, int n_tok, int world,
                                 int capacity, int32_t *ids, float *w, int32_t *send_count,
                                 int32_t *pos, int32_t *send_ids, float *send_x, void *stream) {
    if (!c || !x || !ids || !w || !send_count || !pos || !send_ids || !send_x || n_tok <= 0 ||
        layer < 0 || layer >= c->cfg.n_layers)
        return fail(c, MOE_ERR_ARG, "moe_ep_route_pack: bad argument");
    const moe_cfg &g = c->cfg;
    if (world < 1 || world > 256 || g.n_expert % world)
        return fail(c, MOE_ERR_ARG, "moe_ep_route_pack: world %d does not divide %d experts", world,
                    g.n_expert);
    if (capacity < 0 || (capacity > 0 && capacity < n_tok * g.n_used))
        return fail(c, MOE_ERR_ARG, "moe_ep_route_pack: capacity %d is below the %d pairs of a rank",
                    capacity, n_tok * g.n_used);
    CK(cudaSetDevice(g.device));
    const int r = ensure_scratch(c, n_tok);
    if (r != MOE_OK) return r;
    cudaStream_t s = (cudaStream_t)stream;
    const int32_t *table = c->st.table + (size_t)layer * g.n_expert;
    CK(launch_router(c->router + (size_t)layer * g.n_expert * g.n_embd, x, n_tok, g.n_expert, g.n_embd,
                     table, c->L[layer].ns, 0.0f, 0, g.n_used, ids, w, nullptr, &c->st, -1, nullptr, s));
    GroupBufs gg = c->grp;
    gg.cnt = send_count;
    gg.pair_pos = pos;
    CK(launch_ep_pack(ids, x, n_tok, g.n_used, g.n_expert, g.n_embd, world, capacity, gg, send_ids, send_x,
                      c->err, s));
    return MOE_OK;
}

// moe_experts_rows, with the grouping kernel first waiting on `wait` (the
// expert-parallel owner's rows arrive from peers).
static int experts_rows(moe_ctx *c, int layer, const float *x_rows, const int32_t *ids, int n_rows,
                        float *y_rows, int path, void *stream, const FlagWait *wait) {
    if (!c || n_rows < 0 || layer < 0 || layer >= c->cfg.n_layers || (n_rows && (!x_rows || !ids || !y_rows)))
        return fail(c, MOE_ERR_ARG, "moe_experts_rows: bad argument");
    if (n_rows == 0) return MOE_OK;
    const moe_cfg &g = c->cfg;
    const bool gemm_ok = g.down_type == MOE_QTYPE_Q6_K && g.n_ff % 128 == 0 && g.n_embd % 128 == 0;
    if (path == MOE_PATH_AUTO)
        path = gemm_ok && n_rows >= 4 * c->L[layer].ns ? MOE_PATH_GEMM : MOE_PATH_GEMV;
    if (path != MOE_PATH_GEMV && path != MOE_PATH_GEMM)
        return fail(c, MOE_ERR_ARG, "moe_experts_rows: unknown path %d", path);
    if (path == MOE_PATH_GEMM && !gemm_ok)
        return fail(c, MOE_ERR_UNSUPPORTED, "the GEMM path needs Q6_K down weights and n_ff, n_embd multiples of 128");
    CK(cudaSetDevice(g.device));
    const int n_tok_eq = (n_rows + g.n_used - 1) / g.n_used;   // scratch is sized in tokens of n_used pairs
    int r = ensure_scratch(c, n_tok_eq);
    if (r != MOE_OK) return r;
    cudaStream_t s = (cudaStream_t)stream;
    const int buckets = g.n_expert + g.n_shared;   // id n_expert: the shared expert
    if (path == MOE_PATH_GEMV) {
        CK(launch_group(ids, n_rows, buckets, GROUP_TILE, c->grp, c->err, s, 1, wait));
        CK(launch_experts_grouped(make_src(c, layer), x_rows, c->grp, n_rows, 1, g.n_embd, g.n_ff,
                                  g.down_type, nullptr, c->s_act, c->s_ypair, nullptr, y_rows, c->err, s));
    } else {
        if ((r = ensure_gemm_scratch(c, n_tok_eq)) != MOE_OK) return r;
        CK(launch_group(ids, n_rows, buckets, GM_NT, c->grp, c->err, s, 1, wait));
        CK(launch_experts_gemm(make_src(c, layer), x_rows, c->grp, n_rows, 1, g.n_embd, g.n_ff,
                               g.down_type, nullptr, c->s_gemm, c->s_ypair, nullptr, y_rows, c->err, s));
    }
    return MOE_OK;
}

extern "C" int moe_experts_rows(moe_ctx *c, int layer, const float *x_rows, const int32_t *ids,
                                int n_rows, float *y_rows, int path, void *stream) {
    return experts_rows(c, layer, x_rows, ids, n_rows, y_rows, path, stream, nullptr);
}

extern "C" int moe_ep_combine(moe_ctx *c, const float *y_rows, const int32_t *pos, const float *w,
                              int n_tok, const float *add_rows, float *out, void *stream) {
    if (!c || !pos || !w || !out || n_tok <= 0) return fail(c, MOE_ERR_ARG, "moe_ep_combine: bad argument");
    if (c->cfg.n_shared && !add_rows)
        return fail(c, MOE_ERR_ARG, "moe_ep_combine: the shared expert's rows are missing");
    CK(cudaSetDevice(c->cfg.device));
    CK(launch_combine(y_rows, pos, w, n_tok, c->cfg.n_used, c->cfg.n_embd, add_rows, out,
                      (cudaStream_t)stream));
    return MOE_OK;
}

// ---- expert parallelism over peer memory --------------------------------------

static size_t up256(size_t b) { return (b + 255) & ~(size_t)255; }

extern "C" int moe_ep_mailbox_create(moe_ctx *c, int world, int rank, int max_home_tokens,
                                     void *handle_out) {
    if (!c || !handle_out || world < 2 || world > 256 || rank < 0 || rank >= world || max_home_tokens <= 0)
        return fail(c, MOE_ERR_ARG, "moe_ep_mailbox_create: bad argument");
    if (c->ep_mail) return fail(c, MOE_ERR_ARG, "moe_ep_mailbox_create: the mailbox exists already");
    const moe_cfg &g = c->cfg;
    if (g.n_expert % world)
        return fail(c, MOE_ERR_ARG, "moe_ep_mailbox_create: world %d does not divide %d experts", world,
                    g.n_expert);
    CK(cudaSetDevice(g.device));
    EpMail m{};
    m.world = world;
    m.rank = rank;
    m.cap = max_home_tokens * g.n_used;     // a source may send all its pairs to one owner
    m.n_embd = g.n_embd;
    size_t off = 0;
    m.off_fflag = off; off = up256(off + 8 * (size_t)world);
    m.off_rflag = off; off = up256(off + 8 * (size_t)world);
    m.off_meta = off;  off = up256(off + 8 * (size_t)world);
    m.off_ids = off;   off = up256(off + 4 * (size_t)world * m.cap);
    m.off_x = off;     off = up256(off + 4 * (size_t)world * m.cap * m.n_embd);
    m.off_rety = off;  off = up256(off + 4 * (size_t)m.cap * m.n_embd);
    m.bytes = off;
    if (cudaMalloc(&c->ep_mail, m.bytes) != cudaSuccess ||
        cudaMalloc(&c->ep_peer, sizeof(uint8_t *) * world) != cudaSuccess ||
        cudaMalloc(&c->ep_y, sizeof(float) * (size_t)world * m.cap * m.n_embd) != cudaSuccess ||
        cudaMalloc(&c->ep_epoch, 2 * sizeof(unsigned long long)) != cudaSuccess) {
        cudaFree(c->ep_mail); cudaFree(c->ep_peer); cudaFree(c->ep_y); cudaFree(c->ep_epoch);
        c->ep_mail = nullptr; c->ep_peer = nullptr; c->ep_y = nullptr; c->ep_epoch = nullptr;
        return fail(c, MOE_ERR_OOM, "moe_ep_mailbox_create: %zu bytes of mailbox", m.bytes);
    }
    CK(cudaMemset(c->ep_mail, 0, m.bytes));
    CK(cudaMemset(c->ep_epoch, 0, 2 * sizeof(unsigned long long)));
    cudaIpcMemHandle_t h;
    CK(cudaIpcGetMemHandle(&h, c->ep_mail));
    static_assert(sizeof(cudaIpcMemHandle_t) == MOE_EP_HANDLE_BYTES, "IPC handle size");
    memcpy(handle_out, &h, sizeof(h));
    c->ep = m;
    return MOE_OK;
}

extern "C" int moe_ep_mailbox_connect(moe_ctx *c, const void *handles) {
    if (!c || !handles) return fail(c, MOE_ERR_ARG, "moe_ep_mailbox_connect: bad argument");
    if (!c->ep_mail || c->ep_connected)
        return fail(c, MOE_ERR_ARG, "moe_ep_mailbox_connect: create the mailbox first, once");
    CK(cudaSetDevice(c->cfg.device));
    const EpMail &m = c->ep;
    std::vector<uint8_t *> base(m.world, nullptr);
    for (int r = 0; r < m.world; ++r) {
        if (r == m.rank) {
            base[r] = c->ep_mail;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const uint8_t *>(handles) + (size_t)r * MOE_EP_HANDLE_BYTES, sizeof(h));
        void *p = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess)
            return fail(c, MOE_ERR_CUDA, "moe_ep_mailbox_connect: rank %d's mailbox: %s", r,
                        cudaGetErrorString(e));
        base[r] = static_cast<uint8_t *>(p);
        c->ep_open.push_back(base[r]);
    }
    CK(cudaMemcpy(c->ep_peer, base.data(), sizeof(uint8_t *) * m.world, cudaMemcpyHostToDevice));
    c->ep_connected = true;
    return MOE_OK;
}

// The mailbox layout of one call: blocks of n_tok * n_used slots (every
// rank passes the same n_tok), inside the regions sized for the maximum.
static int ep_call_mail(moe_ctx *c, int n_tok, const char *who, EpMail *m) {
    if (!c->ep_connected) return fail(c, MOE_ERR_ARG, "%s: no connected mailbox", who);
    if (n_tok <= 0 || (int64_t)n_tok * c->cfg.n_used > c->ep.cap)
        return fail(c, MOE_ERR_ARG, "%s: %d home tokens; the mailbox holds 1 to %d", who, n_tok,
                    c->ep.cap / c->cfg.n_used);
    *m = c->ep;
    m->cap = n_tok * c->cfg.n_used;
    return MOE_OK;
}

extern "C" int moe_ep_push(moe_ctx *c, int n_tok, const int32_t *send_count, const int32_t *send_ids,
                           const float *send_x, void *stream) {
    if (!c || !send_count || !send_ids || !send_x)
        return fail(c, MOE_ERR_ARG, "moe_ep_push: bad argument");
    EpMail m;
    const int r = ep_call_mail(c, n_tok, "moe_ep_push", &m);
    if (r != MOE_OK) return r;
    CK(cudaSetDevice(c->cfg.device));
    CK(launch_ep_push(m, c->ep_peer, send_count, send_ids, send_x, c->ep_epoch,
                      reinterpret_cast<unsigned int *>(c->ep_epoch + 1), (cudaStream_t)stream));
    return MOE_OK;
}

extern "C" int moe_ep_serve(moe_ctx *c, int layer, int n_tok, int path, void *stream) {
    if (!c || layer < 0 || layer >= c->cfg.n_layers) return fail(c, MOE_ERR_ARG, "moe_ep_serve: bad argument");
    if (path != MOE_PATH_GEMV && path != MOE_PATH_GEMM)
        return fail(c, MOE_ERR_ARG, "moe_ep_serve: the path must be MOE_PATH_GEMV or MOE_PATH_GEMM");
    EpMail m;
    const int rc = ep_call_mail(c, n_tok, "moe_ep_serve", &m);
    if (rc != MOE_OK) return rc;
    CK(cudaSetDevice(c->cfg.device));
    cudaStream_t s = (cudaStream_t)stream;
    // the grouping kernel waits until every source's rows are in
    const FlagWait fw{reinterpret_cast<const unsigned long long *>(c->ep_mail + m.off_fflag), m.world, c->ep_epoch,
                      c->dp.wait_ns};
    const int r = experts_rows(c, layer, reinterpret_cast<const float *>(c->ep_mail + m.off_x),
                               reinterpret_cast<const int32_t *>(c->ep_mail + m.off_ids), m.world * m.cap, c->ep_y,
                               path, stream, &fw);
    if (r != MOE_OK) return r;
    CK(launch_ep_push(m, c->ep_peer, nullptr, nullptr, c->ep_y, c->ep_epoch,
                      reinterpret_cast<unsigned int *>(c->ep_epoch + 1), s));
    return MOE_OK;
}

extern "C" int moe_ep_collect(moe_ctx *c, const int32_t *pos, const float *w, int n_tok,
                              const float *add_rows, float *out, void *stream) {
    if (!c || !pos || !w || !out) return fail(c, MOE_ERR_ARG, "moe_ep_collect: bad argument");
    if (c->cfg.n_shared && !add_rows)
        return fail(c, MOE_ERR_ARG, "moe_ep_collect: the shared expert's rows are missing");
    EpMail m;
    const int rc = ep_call_mail(c, n_tok, "moe_ep_collect", &m);
    if (rc != MOE_OK) return rc;
    CK(cudaSetDevice(c->cfg.device));
    cudaStream_t s = (cudaStream_t)stream;
    // every CTA of the combine waits until every owner's rows are back
    const FlagWait fw{reinterpret_cast<const unsigned long long *>(c->ep_mail + m.off_rflag), m.world, c->ep_epoch,
                      c->dp.wait_ns};
    CK(launch_combine(reinterpret_cast<const float *>(c->ep_mail + m.off_rety), pos, w, n_tok,
                      c->cfg.n_used, c->cfg.n_embd, add_rows, out, s, &fw, c->err));
    return MOE_OK;
}

// ---- moe_layer_forward_noalloc ----------------------------------------------
// Some callers cannot allocate device memory while they run: their device
// memory is committed up front, and a cudaFree on growth would also wait for
// the whole device.  This variant therefore keeps the router ids/weights and
// the gate/up activations in a static array that is part of the library
// image.  Each device has its own copy of the array.  Every context on that
// device shares it, so calls that overlap in time race on it.

static __device__ __align__(256) uint8_t g_noalloc_scratch[MOE_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kNoallocMaxDevices = 64;
std::mutex g_noalloc_mu;
uint8_t *g_noalloc_ptr[kNoallocMaxDevices] = {};   // device ordinal -> scratch address

constexpr size_t round256(size_t b) { return (b + 255) & ~(size_t)255; }

// Bytes of scratch one call needs: ids and weights, each rounded to 256
// bytes, then the [n_tok][n_used][n_ff] fp32 activations.
size_t noalloc_need(size_t n_tok, size_t k, size_t n_ff) {
    return 2 * round256(4 * n_tok * k) + 4 * n_tok * k * n_ff;
}
}  // namespace

// The first call on a device (with that device current) looks the array's
// address up; later calls reuse it.  The lookup may make the runtime load the
// library's device image, so the first call must come before any stream
// capture.
static int noalloc_scratch(moe_ctx *c, uint8_t **out) {
    const int dev = c->cfg.device;
    if (dev < 0 || dev >= kNoallocMaxDevices)
        return fail(c, MOE_ERR_UNSUPPORTED, "moe_layer_forward_noalloc: device %d is out of range", dev);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return fail(c, MOE_ERR_CUDA, "moe_layer_forward_noalloc: cudaGetSymbolAddress: %s",
                        cudaGetErrorString(e));
        g_noalloc_ptr[dev] = static_cast<uint8_t *>(p);
    }
    *out = g_noalloc_ptr[dev];
    return MOE_OK;
}

extern "C" int moe_layer_forward_noalloc(moe_ctx *c, int layer, const float *x, float *y,
                                         int n_tok, int32_t *ids, float *w, void *stream) {
    if (!c || !x || !y || n_tok <= 0 || layer < 0 || layer >= c->cfg.n_layers)
        return fail(c, MOE_ERR_ARG, "moe_layer_forward_noalloc: bad argument");
    const moe_cfg &g = c->cfg;
    if (g.n_shared)
        return fail(c, MOE_ERR_UNSUPPORTED, "moe_layer_forward_noalloc: contexts with a shared expert are not supported");
    const size_t K = (size_t)g.n_used, I = (size_t)g.n_ff;
    if (noalloc_need((size_t)n_tok, K, I) > MOE_NOALLOC_SCRATCH_BYTES) {
        size_t max_tok = MOE_NOALLOC_SCRATCH_BYTES / (4 * K * I);
        while (max_tok > 0 && noalloc_need(max_tok, K, I) > MOE_NOALLOC_SCRATCH_BYTES) --max_tok;
        return fail(c, MOE_ERR_ARG,
                    "moe_layer_forward_noalloc: %d tokens need %zu bytes of scratch; the static "
                    "scratch holds %u bytes, enough for at most %zu tokens with n_used %d, n_ff %d",
                    n_tok, noalloc_need((size_t)n_tok, K, I), MOE_NOALLOC_SCRATCH_BYTES, max_tok,
                    g.n_used, g.n_ff);
    }
    CK(cudaSetDevice(g.device));
    uint8_t *scr = nullptr;
    const int r = noalloc_scratch(c, &scr);
    if (r != MOE_OK) return r;
    const size_t sel = round256(4 * (size_t)n_tok * K);
    int32_t *ids_d = ids ? ids : reinterpret_cast<int32_t *>(scr);
    float *w_d = w ? w : reinterpret_cast<float *>(scr + sel);
    float *act = reinterpret_cast<float *>(scr + 2 * sel);
    cudaStream_t s = (cudaStream_t)stream;
    const int32_t *table = c->st.table + (size_t)layer * g.n_expert;
    CK(launch_router(c->router + (size_t)layer * g.n_expert * g.n_embd, x, n_tok, g.n_expert, g.n_embd,
                     table, c->L[layer].ns, g.cache_prior, n_tok == 1 && g.cache_prior > 0.0f, g.n_used,
                     ids_d, w_d, nullptr, &c->st, n_tok == 1 ? layer : -1,
                     c->st.slot_expert + c->slot_off[layer], s));
    CK(launch_experts(make_src(c, layer), x, ids_d, w_d, n_tok, g.n_used, g.n_embd, g.n_ff,
                      g.down_type, act, nullptr, y, c->err, s));
    return MOE_OK;
}

extern "C" int moe_decode(moe_ctx *c, const float *h, float *out, int n_tok,
                          const moe_decode_dbg *dbg, void *stream) {
    if (!c || !h || !out || n_tok <= 0) return fail(c, MOE_ERR_ARG, "moe_decode: bad argument");
    for (int l = 0; l < c->cfg.n_layers; ++l) {
        const int r = check_shared(c, l);
        if (r != MOE_OK) return r;
    }
    CK(cudaSetDevice(c->cfg.device));
    if (c->dp.smem_bytes > 227 * 1024)
        return fail(c, MOE_ERR_UNSUPPORTED, "decode needs %d bytes of shared memory", c->dp.smem_bytes);
    cudaStream_t s = (cudaStream_t)stream;
    DecodeParams p = c->dp;
    p.h_in = h;
    p.out = out;
    p.n_tok = n_tok;
    p.dbg_x = dbg ? dbg->x : nullptr;
    p.dbg_ids = dbg ? dbg->ids : nullptr;
    p.dbg_w = dbg ? dbg->w : nullptr;
    p.dbg_y = dbg ? dbg->y : nullptr;
    p.prof = dbg ? dbg->prof : nullptr;
    p.starve = dbg ? dbg->starve : 0;
    if (p.starve < 0 || p.starve > p.kx) return fail(c, MOE_ERR_ARG, "moe_decode: dbg starve out of range");
    const int spec_mode = dbg ? dbg->spec : 0;
    if (spec_mode < 0 || spec_mode > 2) return fail(c, MOE_ERR_ARG, "moe_decode: dbg spec out of range");
    p.spec = spec_mode == 1 ? 0 : spec_mode == 2 ? 2 : 1;
    if (p.dbg_ids && !p.dbg_w) return fail(c, MOE_ERR_ARG, "moe_decode: dbg ids without w");
    CK(cudaMemsetAsync(c->bar, 0, 64, s));
    CK(cudaMemsetAsync(c->abort_flag, 0, 64, s));
    CK(cudaMemsetAsync(c->ready, 0, sizeof(unsigned) * MOE_KMAX * moe::READY_STRIDE, s));
    CK(cudaMemsetAsync(c->acc, 0, sizeof(long long) * 2 * (size_t)(c->cfg.n_expert + 1) * moe::ACC_LINE, s));
    CK(launch_decode(p, c->grid, s));
    return MOE_OK;
}

extern "C" int moe_decode_host(moe_ctx *c, const float *h_host, float *out_host, int n_tok,
                               void *stream) {
    if (!c || !h_host || !out_host || n_tok <= 0) return fail(c, MOE_ERR_ARG, "moe_decode_host: bad argument");
    CK(cudaSetDevice(c->cfg.device));
    const size_t n = (size_t)n_tok * c->cfg.n_embd;
    if ((int)(2 * n) > c->s_io_cap) {
        cudaFree(c->s_io);
        c->s_io = nullptr;
        if (cudaMalloc(&c->s_io, sizeof(float) * 2 * n) != cudaSuccess) {
            c->s_io_cap = 0;
            return fail(c, MOE_ERR_OOM, "io scratch allocation failed");
        }
        c->s_io_cap = (int)(2 * n);
    }
    cudaStream_t s = (cudaStream_t)stream;
    CK(cudaMemcpyAsync(c->s_io, h_host, sizeof(float) * n, cudaMemcpyHostToDevice, s));
    int r = moe_decode(c, c->s_io, c->s_io + n, n_tok, nullptr, stream);
    if (r != MOE_OK) return r;
    CK(cudaMemcpyAsync(out_host, c->s_io + n, sizeof(float) * n, cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    int e = 0;
    CK(cudaMemcpy(&e, c->err, sizeof(int), cudaMemcpyDeviceToHost));
    if (e) {
        // reported once: the next call starts from a clean error word
        CK(cudaMemset(c->err, 0, sizeof(int)));
        if (e & MOE_DEV_ERR_TIMEOUT) return fail(c, MOE_ERR_TIMEOUT, "a device-side wait timed out");
        return fail(c, MOE_ERR_DEVICE, "a kernel saw an out-of-range index");
    }
    return MOE_OK;
}

extern "C" int moe_set_wait_limit(moe_ctx *c, uint64_t ns) {
    if (!c) return MOE_ERR_ARG;
    c->dp.wait_ns = ns ? ns : MOE_TIMEOUT_NS;
    return MOE_OK;
}

extern "C" int moe_sync(moe_ctx *c, void *stream) {
    if (!c) return MOE_ERR_ARG;
    CK(cudaSetDevice(c->cfg.device));
    CK(cudaStreamSynchronize((cudaStream_t)stream));
    int e = 0;
    CK(cudaMemcpy(&e, c->err, sizeof(int), cudaMemcpyDeviceToHost));
    if (e) {
        cudaMemset(c->err, 0, sizeof(int));
        if (e & MOE_DEV_ERR_TIMEOUT) return fail(c, MOE_ERR_TIMEOUT, "a device-side wait timed out");
        return fail(c, MOE_ERR_DEVICE, "a kernel saw an out-of-range index");
    }
    return MOE_OK;
}

// ---------------------------------------------------------------------------
// slot cache step
// ---------------------------------------------------------------------------

extern "C" int moe_observe(moe_ctx *c, int layer, const int32_t *ids, int n_tok, int n_ids,
                           void *stream) {
    if (!c || !ids || layer < 0 || layer >= c->cfg.n_layers || n_ids <= 0 || n_ids > 64)
        return fail(c, MOE_ERR_ARG, "moe_observe: bad argument");
    if (n_tok != 1) return MOE_OK;   // the reference's callback returns early for batches
    CK(cudaSetDevice(c->cfg.device));
    CK(launch_observe(c->st, layer, ids, n_ids, (cudaStream_t)stream));
    return after_observe(c, layer, ids, n_ids, (cudaStream_t)stream);
}

extern "C" int moe_set_predictor(moe_ctx *c, moe_predict_fn fn, void *ud) {
    if (!c) return MOE_ERR_ARG;
    c->predict = fn;
    c->predict_ud = ud;
    c->st.have_pred = fn != nullptr;   // the free pool's target grows by predict_top
    c->dp.st.have_pred = c->st.have_pred;
    return MOE_OK;
}

extern "C" int moe_set_evictor(moe_ctx *c, int n_model, const int32_t *layer_of, int feat_dim,
                               const int32_t *off, const float *w, const float *bias,
                               const float *prior) {
    if (!c) return MOE_ERR_ARG;
    const int E = c->cfg.n_expert, L = c->cfg.n_layers;
    if (n_model == 0) {   // remove: LRU again
        CK(cudaSetDevice(c->cfg.device));
        CK(cudaDeviceSynchronize());
        c->st.have_evict = 0;
        c->dp.st.have_evict = 0;
        return MOE_OK;
    }
    if (n_model < 0 || !layer_of || feat_dim <= 0 || !off || !w || !bias || !prior)
        return fail(c, MOE_ERR_ARG, "moe_set_evictor: bad argument");
    for (int q = 0; q < 4; ++q)
        if (off[q] >= 0 && off[q] + E > feat_dim)
            return fail(c, MOE_ERR_ARG, "moe_set_evictor: block %d at row %d does not fit %d rows", q, off[q], feat_dim);
    std::vector<int32_t> idx(L, -1);
    for (int m = 0; m < n_model; ++m)
        if (layer_of[m] >= 0 && layer_of[m] < L) idx[layer_of[m]] = m;
    CK(cudaSetDevice(c->cfg.device));
    CK(cudaDeviceSynchronize());
    const size_t nw = (size_t)n_model * feat_dim * E, nb = (size_t)n_model * E;
    cudaFree(c->d_ev_model);
    c->d_ev_model = nullptr;
    if (cudaMalloc(&c->d_ev_model, sizeof(float) * (nw + nb + n_model)) != cudaSuccess)
        return fail(c, MOE_ERR_OOM, "moe_set_evictor: %zu bytes", sizeof(float) * (nw + nb + n_model));
    CK(cudaMemcpy(c->d_ev_model, w, sizeof(float) * nw, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(c->d_ev_model + nw, bias, sizeof(float) * nb, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(c->d_ev_model + nw + nb, prior, sizeof(float) * n_model, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(c->d_ev_index, idx.data(), sizeof(int32_t) * L, cudaMemcpyHostToDevice));
    SlotState &st = c->st;
    st.ev_w = c->d_ev_model;
    st.ev_bias = c->d_ev_model + nw;
    st.ev_prior = c->d_ev_model + nw + nb;
    st.ev_feat = feat_dim;
    for (int q = 0; q < 4; ++q) st.ev_off[q] = off[q];
    st.have_evict = 1;
    c->dp.st = st;
    return MOE_OK;
}

extern "C" int moe_set_observe_hook(moe_ctx *c, moe_observe_fn fn, void *ud) {
    if (!c) return MOE_ERR_ARG;
    c->obs_hook = fn;
    c->obs_ud = ud;
    return MOE_OK;
}

// Adds the duration of the last timed upload batch to upload_ns once both
// events have completed.
static void harvest_upload_time(moe_ctx *c) {
    if (!c->up_timed || cudaEventQuery(c->ev_up1) != cudaSuccess) return;
    float ms = 0.0f;
    if (cudaEventElapsedTime(&ms, c->ev_up0, c->ev_up1) == cudaSuccess)
        c->upload_ns += (uint64_t)((double)ms * 1e6);
    c->up_timed = false;
}

// Copies for the jobs in the mapped list from index `from` on, on the copy
// stream; ev_copy follows them.  The caller has synchronised with the
// device work that wrote the list.
static int issue_job_copies(moe_ctx *c, int from, int nj) {
    if (nj > from && !c->up_timed) {
        CK(cudaEventRecord(c->ev_up0, c->copy_stream));
    }
    for (int j = from; j < nj; ++j) {
        const int l = c->h_jobs[4 * j], e = c->h_jobs[4 * j + 1], slot = c->h_jobs[4 * j + 2];
        if (l < 0 || l >= c->cfg.n_layers || e < 0 || e >= c->cfg.n_expert || slot < 0 || slot >= c->L[l].ns)
            return fail(c, MOE_ERR_DEVICE, "moe_step: bad job (%d, %d, %d)", l, e, slot);
        if (c->h_jobs[4 * j + 3] == 2) continue;   // streamed: the mover copies it in chunks
        LayerMem &m = c->L[l];
        if (!m.hgate_user) return fail(c, MOE_ERR_STATE, "moe_step: layer %d has no host weights to upload from", l);
        const uint8_t *hg = (const uint8_t *)m.hgate_user, *hu = (const uint8_t *)m.hup_user,
                      *hd = (const uint8_t *)m.hdown_user;
        CK(cudaMemcpyAsync(m.gate + (size_t)slot * c->gate_bytes, hg + (size_t)e * c->gate_bytes,
                           c->gate_bytes, cudaMemcpyHostToDevice, c->copy_stream));
        CK(cudaMemcpyAsync(m.up + (size_t)slot * c->gate_bytes, hu + (size_t)e * c->gate_bytes,
                           c->gate_bytes, cudaMemcpyHostToDevice, c->copy_stream));
        CK(cudaMemcpyAsync(m.down + (size_t)slot * c->down_bytes, hd + (size_t)e * c->down_bytes,
                           c->down_bytes, cudaMemcpyHostToDevice, c->copy_stream));
        c->upload_bytes += 2 * c->gate_bytes + c->down_bytes;
    }
    if (nj > from) {
        CK(cudaEventRecord(c->ev_up1, c->copy_stream));   // the end of this step's copies so far
        c->up_timed = true;
        CK(cudaEventRecord(c->ev_copy, c->copy_stream));
        c->copies_pending = true;
    }
    return MOE_OK;
}

static volatile int32_t *host_njobs(moe_ctx *c) {
    return c->h_jobs + (size_t)c->st.host_cap * 4;
}

// Early issue: copies for the jobs the device issued since the last call
// (after the device work of `stream` that may have issued them).
static int issue_early_copies(moe_ctx *c, cudaStream_t s) {
    CK(cudaStreamSynchronize(s));
    const int nj = *host_njobs(c);
    const int r = issue_job_copies(c, c->jobs_issued, nj);
    c->jobs_issued = nj;
    return r;
}

extern "C" int moe_step(moe_ctx *c, void *stream) {
    if (!c) return MOE_ERR_ARG;
    CK(cudaSetDevice(c->cfg.device));
    cudaStream_t s = (cudaStream_t)stream;
    if (c->cfg.early_issue) {
        // the jobs of this step were issued when the layers were observed:
        // copy what is not copying yet, publish once every copy is done
        // (deterministic publication), then top the free pools up
        int r = issue_early_copies(c, s);
        if (r != MOE_OK) return r;
        if (c->cfg.stream) {
            // streamed jobs still unsent (their layers did not run) are
            // given back rather than published half copied
            for (int l = 0; l < c->cfg.n_layers; ++l) c->planner->posted(l);
            if ((r = stream_cancel_dropped(c, s)) != MOE_OK) return r;
        }
        if (c->copies_pending) CK(cudaStreamWaitEvent(s, c->ev_copy, 0));
        CK(launch_step(c->st, c->st.host_jobs, c->st.host_njobs, s));
        CK(cudaEventRecord(c->ev_step, s));
        CK(cudaEventSynchronize(c->ev_step));
        c->copies_pending = false;
        c->jobs_issued = 0;
        if (c->cfg.stream) {
            c->planner->reset();
            c->sjobs.clear();
            c->stream_seen = 0;
            c->last_layer = -1;
        }
        harvest_upload_time(c);
        return MOE_OK;
    }
    if (c->copies_pending) CK(cudaStreamWaitEvent(s, c->ev_copy, 0));
    CK(launch_step(c->st, c->st.host_jobs, c->st.host_njobs, s));
    CK(cudaEventRecord(c->ev_step, s));
    CK(cudaEventSynchronize(c->ev_step));
    const int nj = *host_njobs(c);
    c->copies_pending = false;
    harvest_upload_time(c);   // the previous batch is done: the step kernel waited for it
    return issue_job_copies(c, 0, nj);
}

extern "C" int moe_requires_sync(const moe_ctx *c) { return c ? 1 : 0; }

extern "C" int moe_stream_stats(moe_ctx *c, uint64_t *out, int n) {
    if (!c || !out || n < 0) return fail(c, MOE_ERR_ARG, "moe_stream_stats: bad argument");
    CK(cudaSetDevice(c->cfg.device));
    uint64_t g[G_COUNT];
    CK(cudaMemcpy(g, c->st.g, sizeof(g), cudaMemcpyDeviceToHost));
    uint64_t all[MOE_STREAM_STAT_COUNT];
    for (int i = 0; i < 8; ++i) all[i] = c->sst[i];
    all[8] = g[G_STREAM_IN_TIME];
    all[9] = g[G_STREAM_LATE];
    for (int i = 0; i < n && i < MOE_STREAM_STAT_COUNT; ++i) out[i] = all[i];
    return MOE_OK;
}

extern "C" int moe_get_tables(moe_ctx *c, int layer, int32_t *expert_slot, int32_t *slot_expert,
                              uint64_t *last_use, uint8_t *in_flight, uint64_t *protect) {
    if (!c || layer < 0 || layer >= c->cfg.n_layers) return fail(c, MOE_ERR_ARG, "moe_get_tables: bad layer");
    CK(cudaSetDevice(c->cfg.device));
    CK(cudaDeviceSynchronize());
    const int E = c->cfg.n_expert, ns = c->L[layer].ns, so = c->slot_off[layer];
    if (expert_slot) {
        CK(cudaMemcpy(expert_slot, c->st.table + (size_t)layer * E, 4 * E, cudaMemcpyDeviceToHost));
        for (int e = 0; e < E; ++e) if (expert_slot[e] == ns) expert_slot[e] = -1;
    }
    if (slot_expert) CK(cudaMemcpy(slot_expert, c->st.slot_expert + so, 4 * ns, cudaMemcpyDeviceToHost));
    if (last_use) CK(cudaMemcpy(last_use, c->st.last_use + so, 8 * ns, cudaMemcpyDeviceToHost));
    if (in_flight) CK(cudaMemcpy(in_flight, c->st.in_flight + so, ns, cudaMemcpyDeviceToHost));
    if (protect) CK(cudaMemcpy(protect, c->st.protect + so, 8 * ns, cudaMemcpyDeviceToHost));
    return MOE_OK;
}

extern "C" int moe_get_gate_state(moe_ctx *c, int layer, float *heat, uint64_t *miss_last,
                                  uint64_t *miss_prev, uint32_t *use_count) {
    if (!c || layer < 0 || layer >= c->cfg.n_layers) return fail(c, MOE_ERR_ARG, "moe_get_gate_state: bad layer");
    CK(cudaSetDevice(c->cfg.device));
    CK(cudaDeviceSynchronize());
    const size_t E = (size_t)c->cfg.n_expert, o = (size_t)layer * E;
    if (heat && c->st.heat) CK(cudaMemcpy(heat, c->st.heat + o, 4 * E, cudaMemcpyDeviceToHost));
    if (miss_last && c->st.miss_last) CK(cudaMemcpy(miss_last, c->st.miss_last + o, 8 * E, cudaMemcpyDeviceToHost));
    if (miss_prev && c->st.miss_prev) CK(cudaMemcpy(miss_prev, c->st.miss_prev + o, 8 * E, cudaMemcpyDeviceToHost));
    if (use_count && c->st.use_count) CK(cudaMemcpy(use_count, c->st.use_count + o, 4 * E, cudaMemcpyDeviceToHost));
    return MOE_OK;
}

extern "C" int moe_get_stats(moe_ctx *c, uint64_t *out, int n) {
    if (!c || !out || n <= 0) return fail(c, MOE_ERR_ARG, "moe_get_stats: bad argument");
    CK(cudaSetDevice(c->cfg.device));
    CK(cudaDeviceSynchronize());
    uint64_t g[G_COUNT];
    CK(cudaMemcpy(g, c->st.g, sizeof(g), cudaMemcpyDeviceToHost));
    const int L = c->cfg.n_layers;
    std::vector<uint64_t> hit(L), miss(L);
    CK(cudaMemcpy(hit.data(), c->st.n_hit, 8 * L, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(miss.data(), c->st.n_miss, 8 * L, cudaMemcpyDeviceToHost));
    uint64_t h = 0, m = 0;
    for (int l = 0; l < L; ++l) { h += hit[l]; m += miss[l]; }
    harvest_upload_time(c);
    uint64_t all[MOE_STAT_COUNT] = {g[G_STEPS], g[G_CLOCK], h, m, g[G_UPLOADS], g[G_SCHEDULED],
                                    g[G_COPIED], g[G_PUBLISHED], g[G_ADMIT_OK], g[G_ADMIT_DENIED],
                                    g[G_FLUSHES], c->upload_bytes, c->upload_ns};
    for (int i = 0; i < n && i < MOE_STAT_COUNT; ++i) out[i] = all[i];
    return MOE_OK;
}

extern "C" int moe_warm_start(moe_ctx *c, const uint32_t *use_count) {
    if (!c || !use_count) return fail(c, MOE_ERR_ARG, "moe_warm_start: bad argument");
    CK(cudaSetDevice(c->cfg.device));
    const int L = c->cfg.n_layers, E = c->cfg.n_expert;
    if (c->st.use_count) CK(cudaMemcpy(c->st.use_count, use_count, 4 * (size_t)L * E, cudaMemcpyHostToDevice));
    uint64_t clock = 0;
    CK(cudaMemcpy(&clock, c->st.g + G_CLOCK, 8, cudaMemcpyDeviceToHost));
    int placed = 0;
    for (int l = 0; l < L; ++l) {
        const uint32_t *uc = use_count + (size_t)l * E;
        std::vector<int32_t> order(E);
        for (int e = 0; e < E; ++e) order[e] = e;
        std::stable_sort(order.begin(), order.end(), [&](int32_t a, int32_t b) { return uc[a] > uc[b]; });
        const int ns = c->L[l].ns;
        // with early issue the free pool keeps its target free (0007:577-579)
        const int reserve = c->cfg.early_issue
            ? pool_target_of(c->st) : 0;
        const int fill = std::max(0, ns - reserve);
        std::vector<int32_t> se(ns, -1);
        std::vector<uint64_t> lu(ns, 0);
        int slot = 0;
        for (int k = 0; k < E && slot < fill; ++k) {
            const int e = order[k];
            if (uc[e] == 0) break;
            se[slot] = e;
            lu[slot] = (uint64_t)(fill - slot);
            ++slot;
            ++placed;
        }
        clock = std::max<uint64_t>(clock, (uint64_t)fill);
        const int r = moe_place(c, l, se.data(), 1);
        if (r != MOE_OK) return r;
        CK(cudaMemcpy(c->st.last_use + c->slot_off[l], lu.data(), 8 * (size_t)ns, cudaMemcpyHostToDevice));
        // the free pool: every slot past the placed ones, the lowest on top
        std::vector<int32_t> fs;
        for (int f = ns - 1; f >= slot; --f) fs.push_back(f);
        const int nf = (int)fs.size();
        if (nf) CK(cudaMemcpy(c->st.free_slots + c->slot_off[l], fs.data(), 4 * (size_t)nf, cudaMemcpyHostToDevice));
        CK(cudaMemcpy(c->st.n_free + l, &nf, 4, cudaMemcpyHostToDevice));
    }
    CK(cudaMemcpy(c->st.g + G_CLOCK, &clock, 8, cudaMemcpyHostToDevice));
    return placed;
}

// ---------------------------------------------------------------------------
// stateless kernels
// ---------------------------------------------------------------------------

extern "C" int moe_router_run(const float *W, const float *x, int n_tok, int n_expert, int n_embd,
                              const int32_t *table, int n_slots, float delta, int k, int32_t *ids,
                              float *w, float *logits, void *stream) {
    if (!W || !x || !ids || !w || n_tok <= 0 || n_expert % 32 || n_expert > 256 || n_embd % 128 ||
        k <= 0 || k > MOE_KMAX || k > n_expert)
        return fail(nullptr, MOE_ERR_ARG, "moe_router_run: bad argument");
    moe_ctx *c = nullptr;
    CK(launch_router(W, x, n_tok, n_expert, n_embd, table, n_slots, delta,
                     table != nullptr && delta > 0.0f && n_tok == 1, k, ids, w, logits, nullptr, -1,
                     nullptr, (cudaStream_t)stream));
    return MOE_OK;
}

extern "C" int moe_quantize(const float *x, void *y, int64_t n, int qtype, void *stream) {
    if (!x || !y || n % MOE_QK || (qtype != MOE_QTYPE_Q4_K && qtype != MOE_QTYPE_Q6_K))
        return fail(nullptr, MOE_ERR_ARG, "moe_quantize: bad argument");
    moe_ctx *c = nullptr;
    CK(launch_quantize(x, y, n, qtype, (cudaStream_t)stream));
    return MOE_OK;
}

extern "C" int moe_synth_weights(void *y, int64_t n_blocks, int qtype, uint64_t seed, float sigma,
                                 void *stream) {
    if (!y || n_blocks < 0 || (qtype != MOE_QTYPE_Q4_K && qtype != MOE_QTYPE_Q6_K))
        return fail(nullptr, MOE_ERR_ARG, "moe_synth_weights: bad argument");
    moe_ctx *c = nullptr;
    CK(launch_synth_weights(y, n_blocks, qtype, seed, sigma, (cudaStream_t)stream));
    return MOE_OK;
}

extern "C" int moe_synth_f32(float *y, int64_t n, uint64_t seed, float sigma, void *stream) {
    if (!y || n < 0) return fail(nullptr, MOE_ERR_ARG, "moe_synth_f32: bad argument");
    moe_ctx *c = nullptr;
    CK(launch_synth_f32(y, n, seed, sigma, (cudaStream_t)stream));
    return MOE_OK;
}

extern "C" int moe_decode_info(const moe_ctx *c, int32_t *out, int n) {
    if (!c || !out) return MOE_ERR_ARG;
    const int32_t v[] = {c->grid, c->dp.smem_bytes, c->dp.gu_rows_max, c->dp.dn_rows_max, 512};
    for (int i = 0; i < n && i < 5; ++i) out[i] = v[i];
    return MOE_OK;
}

// ---------------------------------------------------------------------------
// ExpertCache (src/prefetch_engine.py)
// ---------------------------------------------------------------------------

struct moe_xc {
    int n_layers = 0, n_experts = 0, capacity = 0, device = 0;
    int64_t bytes = 0;
    const uint8_t *staging = nullptr;
    bool registered = false;
    std::vector<uint8_t *> slabs;
    // per layer: LRU list of experts (front = least recently used) + map
    std::vector<std::list<int32_t>> lru;
    std::vector<std::unordered_map<int32_t, std::pair<int32_t, std::list<int32_t>::iterator>>> map;
    std::vector<std::vector<int32_t>> free_slots;
    std::unordered_map<int64_t, cudaEvent_t> pending;   // (layer, expert) -> event
    std::vector<cudaEvent_t> event_pool;
    cudaStream_t copy_stream = nullptr;
    uint64_t hits = 0, misses = 0, late = 0, fetches = 0, nbytes = 0, evictions = 0;
};

static int64_t xc_key(int layer, int e) { return (int64_t)layer << 32 | (uint32_t)e; }

extern "C" int moe_xc_create(int n_layers, int n_experts, int capacity, int64_t bytes_per_expert,
                             const void *host_staging, int device, moe_xc **out) {
    if (!out || n_layers <= 0 || n_experts <= 0 || capacity <= 0 || bytes_per_expert <= 0 || !host_staging)
        return fail(nullptr, MOE_ERR_ARG, "moe_xc_create: bad argument");
    moe_ctx *c = nullptr;
    CK(cudaSetDevice(device));
    moe_xc *x = new moe_xc();
    x->n_layers = n_layers; x->n_experts = n_experts; x->capacity = capacity; x->device = device;
    x->bytes = bytes_per_expert;
    x->staging = (const uint8_t *)host_staging;
    cudaPointerAttributes at{};
    if (cudaPointerGetAttributes(&at, host_staging) != cudaSuccess) { (void)cudaGetLastError(); at.type = cudaMemoryTypeUnregistered; }
    if (at.type == cudaMemoryTypeUnregistered) {
        if (cudaHostRegister(const_cast<void *>(host_staging), (size_t)n_experts * bytes_per_expert,
                             cudaHostRegisterPortable) != cudaSuccess) {
            (void)cudaGetLastError();
            delete x;
            return fail(nullptr, MOE_ERR_CUDA, "moe_xc_create: cudaHostRegister failed");
        }
        x->registered = true;
    }
    x->slabs.resize(n_layers, nullptr);
    for (int l = 0; l < n_layers; ++l) {
        if (cudaMalloc(&x->slabs[l], (size_t)capacity * bytes_per_expert) != cudaSuccess) {
            moe_xc_destroy(x);
            return fail(nullptr, MOE_ERR_OOM, "moe_xc_create: slab allocation failed");
        }
    }
    x->lru.resize(n_layers);
    x->map.resize(n_layers);
    x->free_slots.resize(n_layers);
    for (int l = 0; l < n_layers; ++l)
        for (int s = 0; s < capacity; ++s) x->free_slots[l].push_back(s);   // pop() takes the last
    if (cudaStreamCreateWithFlags(&x->copy_stream, cudaStreamNonBlocking) != cudaSuccess) {
        moe_xc_destroy(x);
        return fail(nullptr, MOE_ERR_CUDA, "moe_xc_create: stream creation failed");
    }
    *out = x;
    return MOE_OK;
}

extern "C" void moe_xc_destroy(moe_xc *x) {
    if (!x) return;
    cudaSetDevice(x->device);
    if (x->copy_stream) cudaStreamSynchronize(x->copy_stream);
    for (auto &kv : x->pending) cudaEventDestroy(kv.second);
    for (auto ev : x->event_pool) cudaEventDestroy(ev);
    for (auto p : x->slabs) if (p) cudaFree(p);
    if (x->registered) cudaHostUnregister(const_cast<uint8_t *>(x->staging));
    if (x->copy_stream) cudaStreamDestroy(x->copy_stream);
    delete x;
}

static void xc_drop_pending(moe_xc *x, int layer, int e) {
    auto it = x->pending.find(xc_key(layer, e));
    if (it != x->pending.end()) {
        x->event_pool.push_back(it->second);
        x->pending.erase(it);
    }
}

// _slot_for (src/prefetch_engine.py:73-86)
static int32_t xc_slot_for(moe_xc *x, int layer, int e) {
    auto &m = x->map[layer];
    auto &lru = x->lru[layer];
    auto it = m.find(e);
    if (it != m.end()) {
        lru.splice(lru.end(), lru, it->second.second);
        return it->second.first;
    }
    int32_t slot;
    if (!x->free_slots[layer].empty()) {
        slot = x->free_slots[layer].back();
        x->free_slots[layer].pop_back();
    } else {
        const int32_t old = lru.front();
        lru.pop_front();
        slot = m[old].first;
        m.erase(old);
        xc_drop_pending(x, layer, old);
        x->evictions++;
    }
    lru.push_back(e);
    m[e] = {slot, std::prev(lru.end())};
    return slot;
}

static int xc_fetch(moe_xc *x, int layer, const int32_t *ids, int n, bool count_started) {
    moe_ctx *c = nullptr;
    int started = 0;
    for (int i = 0; i < n; ++i) {
        const int e = ids[i];
        if (e < 0 || e >= x->n_experts) return fail(nullptr, MOE_ERR_ARG, "expert id %d out of range", e);
        auto it = x->map[layer].find(e);
        if (it != x->map[layer].end()) {
            x->lru[layer].splice(x->lru[layer].end(), x->lru[layer], it->second.second);
            continue;
        }
        const int32_t slot = xc_slot_for(x, layer, e);
        CK(cudaMemcpyAsync(x->slabs[layer] + (size_t)slot * x->bytes, x->staging + (size_t)e * x->bytes,
                           (size_t)x->bytes, cudaMemcpyHostToDevice, x->copy_stream));
        cudaEvent_t ev;
        if (!x->event_pool.empty()) { ev = x->event_pool.back(); x->event_pool.pop_back(); }
        else CK(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
        CK(cudaEventRecord(ev, x->copy_stream));
        xc_drop_pending(x, layer, e);
        x->pending[xc_key(layer, e)] = ev;
        started++;
        x->fetches++;
        x->nbytes += (uint64_t)x->bytes;
    }
    (void)count_started;
    return started;
}

extern "C" int moe_xc_prefetch(moe_xc *x, int layer, const int32_t *ids, int n) {
    if (!x || layer < 0 || layer >= x->n_layers || (n > 0 && !ids)) return MOE_ERR_ARG;
    cudaSetDevice(x->device);
    return xc_fetch(x, layer, ids, n, true);
}

extern "C" int moe_xc_admit(moe_xc *x, int layer, const int32_t *ids, int n) {
    if (!x || layer < 0 || layer >= x->n_layers || (n > 0 && !ids)) return MOE_ERR_ARG;
    cudaSetDevice(x->device);
    const int r = xc_fetch(x, layer, ids, n, false);
    return r < 0 ? r : MOE_OK;
}

extern "C" int moe_xc_query(moe_xc *x, int layer, const int32_t *ids, int n, int32_t *status) {
    if (!x || layer < 0 || layer >= x->n_layers || (n > 0 && (!ids || !status))) return MOE_ERR_ARG;
    cudaSetDevice(x->device);
    for (int i = 0; i < n; ++i) {
        const int e = ids[i];
        auto it = x->map[layer].find(e);
        if (it == x->map[layer].end()) {
            status[i] = 2;
            x->misses++;
            continue;
        }
        auto pit = x->pending.find(xc_key(layer, e));
        if (pit != x->pending.end()) {
            const cudaError_t q = cudaEventQuery(pit->second);
            if (q == cudaErrorNotReady) {
                (void)cudaGetLastError();
                status[i] = 1;
                x->late++;
                continue;
            }
            xc_drop_pending(x, layer, e);
        }
        x->lru[layer].splice(x->lru[layer].end(), x->lru[layer], it->second.second);
        status[i] = 0;
        x->hits++;
    }
    return MOE_OK;
}

extern "C" int moe_xc_sync(moe_xc *x) {
    if (!x) return MOE_ERR_ARG;
    cudaSetDevice(x->device);
    moe_ctx *c = nullptr;
    CK(cudaStreamSynchronize(x->copy_stream));
    return MOE_OK;
}

extern "C" int64_t moe_xc_vram_bytes(const moe_xc *x) {
    return x ? (int64_t)x->n_layers * x->capacity * x->bytes : 0;
}

extern "C" int moe_xc_stats(const moe_xc *x, uint64_t *out6) {
    if (!x || !out6) return MOE_ERR_ARG;
    out6[0] = x->hits; out6[1] = x->misses; out6[2] = x->late;
    out6[3] = x->fetches; out6[4] = x->nbytes; out6[5] = x->evictions;
    return MOE_OK;
}

extern "C" void *moe_xc_slab(moe_xc *x, int layer) {
    return x && layer >= 0 && layer < x->n_layers ? x->slabs[layer] : nullptr;
}

extern "C" int moe_xc_slot_of(const moe_xc *x, int layer, int expert) {
    if (!x || layer < 0 || layer >= x->n_layers) return -1;
    auto it = x->map[layer].find(expert);
    return it == x->map[layer].end() ? -1 : it->second.first;
}
