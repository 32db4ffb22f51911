// Host side of the context-parallel prefill (g4a_cp_prefill, g4a_cp_wait,
// g4a_nccl_*): one long global attention layer over the W ranks of the
// caller's NCCL communicator.
//
// The reference has no multi-device code: its prompt loop runs one position
// at a time (crates/llm-gemma4/src/impl_/generate.rs:37-41), each position
// attending to every earlier key on global layers (model.rs:326-366 over
// eng/mod.rs:33-35). Both schedules here compute exactly that attention for
// every position, split over ranks in 2W zigzag chunks (rank r: chunks r and
// 2W-1-r, equal causal work), with partial results over disjoint key sets
// merged by log-sum-exp.
//
// NCCL is not linked: its functions are resolved at run time from the
// libnccl.so.2 already loaded in the process (the one that created the
// caller's communicator, e.g. torch's), or loaded here when there is none.
// nccl.h supplies the types and enum values only.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/g4attn.h"
#include "host_internal.h"
#include "internal.h"

using namespace g4a;

namespace {

struct NcclApi {
    bool tried = false, ok = false;
    std::string why;
    decltype(&ncclAllGather) AllGather = nullptr;
    decltype(&ncclAllReduce) AllReduce = nullptr;
    decltype(&ncclReduceScatter) ReduceScatter = nullptr;
    decltype(&ncclSend) Send = nullptr;
    decltype(&ncclRecv) Recv = nullptr;
    decltype(&ncclGroupStart) GroupStart = nullptr;
    decltype(&ncclGroupEnd) GroupEnd = nullptr;
    decltype(&ncclCommCount) CommCount = nullptr;
    decltype(&ncclCommUserRank) CommUserRank = nullptr;
    decltype(&ncclCommGetAsyncError) CommGetAsyncError = nullptr;
    decltype(&ncclCommAbort) CommAbort = nullptr;
    decltype(&ncclGetErrorString) GetErrorString = nullptr;
    decltype(&ncclGetUniqueId) GetUniqueId = nullptr;
    decltype(&ncclCommInitRank) CommInitRank = nullptr;
    decltype(&ncclCommDestroy) CommDestroy = nullptr;
};

NcclApi &nccl() {
    static NcclApi api;
    static std::mutex mu;
    std::lock_guard<std::mutex> lock(mu);
    if (api.tried) return api;
    api.tried = true;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
        const char *e = dlerror();
        api.why = e ? e : "libnccl.so.2 not found";
        return api;
    }
#define G4A_NCCL_SYM(field, name)                                              \
    api.field = reinterpret_cast<decltype(api.field)>(dlsym(h, name));         \
    if (!api.field) {                                                          \
        api.why = "libnccl.so.2 has no " name;                                 \
        return api;                                                            \
    }
    G4A_NCCL_SYM(AllGather, "ncclAllGather")
    G4A_NCCL_SYM(AllReduce, "ncclAllReduce")
    G4A_NCCL_SYM(ReduceScatter, "ncclReduceScatter")
    G4A_NCCL_SYM(Send, "ncclSend")
    G4A_NCCL_SYM(Recv, "ncclRecv")
    G4A_NCCL_SYM(GroupStart, "ncclGroupStart")
    G4A_NCCL_SYM(GroupEnd, "ncclGroupEnd")
    G4A_NCCL_SYM(CommCount, "ncclCommCount")
    G4A_NCCL_SYM(CommUserRank, "ncclCommUserRank")
    G4A_NCCL_SYM(CommGetAsyncError, "ncclCommGetAsyncError")
    G4A_NCCL_SYM(CommAbort, "ncclCommAbort")
    G4A_NCCL_SYM(GetErrorString, "ncclGetErrorString")
    G4A_NCCL_SYM(GetUniqueId, "ncclGetUniqueId")
    G4A_NCCL_SYM(CommInitRank, "ncclCommInitRank")
    G4A_NCCL_SYM(CommDestroy, "ncclCommDestroy")
#undef G4A_NCCL_SYM
    api.ok = true;
    return api;
}

// A call on a non-blocking communicator may return ncclInProgress: wait
// (bounded) until it is issued. Any other failure is G4A_NCCL.
int nccl_check(g4a_ctx *ctx, NcclApi &api, ncclComm_t comm, ncclResult_t r, const char *what) {
    if (r == ncclSuccess) return G4A_OK;
    if (r == ncclInProgress) {
        const auto t0 = std::chrono::steady_clock::now();
        while (std::chrono::steady_clock::now() - t0 < std::chrono::seconds(10)) {
            ncclResult_t a = ncclInProgress;
            api.CommGetAsyncError(comm, &a);
            if (a == ncclSuccess) return G4A_OK;
            if (a != ncclInProgress) {
                r = a;
                break;
            }
            std::this_thread::sleep_for(std::chrono::microseconds(20));
        }
        if (r == ncclInProgress) return fail(ctx, G4A_TIMEOUT, "nccl: %s was not issued within 10 s", what);
    }
    return fail(ctx, G4A_NCCL, "nccl: %s: %s", what, api.GetErrorString(r));
}

#define G4A_NCCL_TRY(ctx, api, comm, call)                                          \
    do {                                                                            \
        const int rc_ = nccl_check(ctx, api, comm, (call), #call);                  \
        if (rc_ != G4A_OK) return rc_;                                              \
    } while (0)

// Collects the first failure of the calls inside an ncclGroupStart/End pair
// so that the group is always closed before an error is returned.
struct Group {
    NcclApi &api;
    ncclResult_t first = ncclSuccess;
    const char *what = nullptr;
    explicit Group(NcclApi &a) : api(a) {}
    void operator()(ncclResult_t r, const char *w) {
        if (first == ncclSuccess && r != ncclSuccess && r != ncclInProgress) {
            first = r;
            what = w;
        }
    }
    int close(g4a_ctx *ctx, ncclComm_t comm) {
        const ncclResult_t e = api.GroupEnd();
        if (first != ncclSuccess) return fail(ctx, G4A_NCCL, "nccl: %s: %s", what, api.GetErrorString(first));
        return nccl_check(ctx, api, comm, e, "ncclGroupEnd");
    }
};
#define G4A_GROUP_CALL(g, call) (g)((call), #call)

struct CpState {
    int device = -1;
    cudaStream_t side = nullptr;
    cudaEvent_t ev_start = nullptr, ev_gathered = nullptr;
    uint16_t *gathered = nullptr;  // bf16: all queries [T][8][hd], or keys then values [T][hd] each
    size_t gathered_cap = 0;       // elements
    float *part = nullptr;     // partial outputs and their lse
    size_t part_cap = 0;       // floats
    float *rowmax = nullptr;
    size_t rowmax_cap = 0;
    float *packed = nullptr;
    size_t packed_cap = 0;
    float *recv = nullptr;
    size_t recv_cap = 0;
};

void cp_state_free(void *p) {
    auto *s = static_cast<CpState *>(p);
    if (!s) return;
    if (s->side) cudaStreamSynchronize(s->side);
    cudaFree(s->gathered);
    cudaFree(s->part);
    cudaFree(s->rowmax);
    cudaFree(s->packed);
    cudaFree(s->recv);
    if (s->ev_start) cudaEventDestroy(s->ev_start);
    if (s->ev_gathered) cudaEventDestroy(s->ev_gathered);
    if (s->side) cudaStreamDestroy(s->side);
    delete s;
}

int cp_state(g4a_ctx *ctx, CpState **out) {
    auto *s = static_cast<CpState *>(ctx->cp);
    if (!s) {
        s = new CpState();
        s->device = ctx->device;
        ctx->cp = s;
        ctx->cp_free = cp_state_free;
        G4A_CUDA_TRY(ctx, cudaStreamCreateWithFlags(&s->side, cudaStreamNonBlocking));
        G4A_CUDA_TRY(ctx, cudaEventCreateWithFlags(&s->ev_start, cudaEventDisableTiming));
        G4A_CUDA_TRY(ctx, cudaEventCreateWithFlags(&s->ev_gathered, cudaEventDisableTiming));
    }
    *out = s;
    return G4A_OK;
}

// Grows a buffer of the state; queued work of the previous call may still
// read the old one, so both streams drain first.
template <typename T>
int grow_cp(g4a_ctx *ctx, CpState *s, T **p, size_t *cap, size_t need) {
    if (need <= *cap) return G4A_OK;
    cudaStreamSynchronize(ctx->stream);
    cudaStreamSynchronize(s->side);
    cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    G4A_CUDA_TRY(ctx, cudaMalloc(reinterpret_cast<void **>(p), need * sizeof(T)));
    *cap = need;
    return G4A_OK;
}

cudaEvent_t take_event(g4a_ctx *ctx) {
    cudaEvent_t e = nullptr;
    if (!ctx->spare.empty()) {
        e = ctx->spare.back();
        ctx->spare.pop_back();
    } else {
        cudaEventCreate(&e);
    }
    return e;
}

// A region of queued work on stream `st` timed under profile id `kernel`
// when the context is profiling.
struct Region {
    g4a_ctx *ctx;
    int kernel;
    cudaStream_t st;
    cudaEvent_t a = nullptr;
    Region(g4a_ctx *c, int k, cudaStream_t s) : ctx(c), kernel(k), st(s) {
        if (ctx->profiling) {
            a = take_event(ctx);
            cudaEventRecord(a, st);
        }
    }
    void end() {
        if (!a) return;
        cudaEvent_t b = take_event(ctx);
        cudaEventRecord(b, st);
        ctx->recs.push_back({kernel, a, b});
        a = nullptr;
    }
};

// SMs the local attention leaves to the exchange running beside it: NCCL's
// kernels need SMs of their own, and a persistent prefill holding all of them
// would delay the exchange until it ends (G4A_CP_RESERVE_SMS overrides, for
// measurement).
int exchange_sms() {
    static const int n = [] {
        const char *e = getenv("G4A_CP_RESERVE_SMS");
        return e ? std::max(0, atoi(e)) : 8;
    }();
    return n;
}

int run_prefill(g4a_ctx *ctx, const std::vector<g4a_prefill_problem> &probs, int reserve_sms = 0) {
    if (probs.empty()) return G4A_OK;
    const char *msg = "";
    const int rc = prefill_run(ctx->prefill, ctx->d_err, (int32_t)probs.size(), probs.data(), ctx->stream, &msg,
                               false, reserve_sms);
    if (rc != G4A_OK) return fail(ctx, rc, "compute: %s", msg);
    return G4A_OK;
}

g4a_prefill_problem problem(int32_t hd, const void *q, int32_t n_q, int32_t q_pos0, const void *k, const void *v,
                            int32_t n_kv, int32_t kv_pos0, float *out, float *lse) {
    g4a_prefill_problem p{};
    p.head_dim = hd;
    p.window = 0;
    p.n_q = n_q;
    p.q_pos0 = q_pos0;
    p.n_kv = n_kv;
    p.kv_pos0 = kv_pos0;
    p.q_dev = q;
    p.k_dev = k;
    p.v_dev = v;
    p.out_dev = out;
    p.lse_dev = lse;
    return p;
}

const uint16_t *bf16_at(const void *base, size_t elems) { return static_cast<const uint16_t *>(base) + elems; }

// Key/value chunks gathered, diagonal blocks meanwhile, then each query chunk
// against all earlier keys, then a two-part log-sum-exp merge per chunk.
int schedule_gather_kv(g4a_ctx *ctx, NcclApi &api, ncclComm_t comm, CpState *s, int W, int r,
                       const g4a_cp_problem &p) {
    const int32_t hd = p.head_dim, T = p.seq_len, c = T / (2 * W);
    const size_t qrow = (size_t)kHeads * hd, krow = (size_t)hd;
    const int32_t a0 = r * c, b0 = (2 * W - 1 - r) * c;
    int rc;
    // keys then values, [T][hd] bf16 each (rows [0, b0) are read)
    if ((rc = grow_cp(ctx, s, &s->gathered, &s->gathered_cap, 2 * (size_t)T * krow))) return rc;
    uint16_t *keys = s->gathered, *values = keys + (size_t)T * krow;
    // partials: diag A, diag B, off A, off B -> out [c][8][hd] + lse [c][8] each
    const size_t po = (size_t)c * qrow, pl = (size_t)c * kHeads;
    if ((rc = grow_cp(ctx, s, &s->part, &s->part_cap, 4 * (po + pl)))) return rc;
    float *o[4], *l[4];
    for (int i = 0; i < 4; i++) {
        o[i] = s->part + i * po;
        l[i] = s->part + 4 * po + i * pl;
    }
    const void *qA = p.q_dev, *qB = bf16_at(p.q_dev, (size_t)c * qrow);
    const void *kA = p.k_dev, *kB = bf16_at(p.k_dev, (size_t)c * krow);
    const void *vA = p.v_dev, *vB = bf16_at(p.v_dev, (size_t)c * krow);
    float *outA = p.out_dev, *outB = p.out_dev + (size_t)c * qrow;

    // exchange on the side stream, after the caller's prior work on its stream
    G4A_CUDA_TRY(ctx, cudaEventRecord(s->ev_start, ctx->stream));
    G4A_CUDA_TRY(ctx, cudaStreamWaitEvent(s->side, s->ev_start, 0));
    {
        Region reg(ctx, G4A_K_CP_EXCHANGE, s->side);
        // chunks 0..W-1 are the ranks' first chunks: an all-gather puts them in place
        G4A_NCCL_TRY(ctx, api, comm, api.GroupStart());
        Group g(api);
        G4A_GROUP_CALL(g, api.AllGather(kA, keys, (size_t)c * krow, ncclBfloat16, comm, s->side));
        G4A_GROUP_CALL(g, api.AllGather(vA, values, (size_t)c * krow, ncclBfloat16, comm, s->side));
        if ((rc = g.close(ctx, comm))) return rc;
        // chunk 2W-1-j of rank j is needed only by ranks below j
        if (W > 1) {
            G4A_NCCL_TRY(ctx, api, comm, api.GroupStart());
            Group g2(api);
            for (int j = 0; j < W; j++) {
                if (j > r) {
                    const size_t at = (size_t)(2 * W - 1 - j) * c * krow;
                    G4A_GROUP_CALL(g2, api.Recv(keys + at, (size_t)c * krow, ncclBfloat16, j, comm, s->side));
                    G4A_GROUP_CALL(g2, api.Recv(values + at, (size_t)c * krow, ncclBfloat16, j, comm, s->side));
                } else if (j < r) {
                    G4A_GROUP_CALL(g2, api.Send(kB, (size_t)c * krow, ncclBfloat16, j, comm, s->side));
                    G4A_GROUP_CALL(g2, api.Send(vB, (size_t)c * krow, ncclBfloat16, j, comm, s->side));
                }
            }
            if ((rc = g2.close(ctx, comm))) return rc;
        }
        reg.end();
    }
    G4A_CUDA_TRY(ctx, cudaEventRecord(s->ev_gathered, s->side));
    {
        Region reg(ctx, G4A_K_CP_ATTEND_LOCAL, ctx->stream);
        if ((rc = run_prefill(ctx,
                              {problem(hd, qA, c, a0, kA, vA, c, a0, o[0], l[0]),
                               problem(hd, qB, c, b0, kB, vB, c, b0, o[1], l[1])},
                              W > 1 ? exchange_sms() : 0)))
            return rc;
        reg.end();
    }
    G4A_CUDA_TRY(ctx, cudaStreamWaitEvent(ctx->stream, s->ev_gathered, 0));
    {
        Region reg(ctx, G4A_K_CP_ATTEND_REMOTE, ctx->stream);
        std::vector<g4a_prefill_problem> off;
        if (a0 > 0) off.push_back(problem(hd, qA, c, a0, keys, values, a0, 0, o[2], l[2]));
        off.push_back(problem(hd, qB, c, b0, keys, values, b0, 0, o[3], l[3]));
        if ((rc = run_prefill(ctx, off))) return rc;
        reg.end();
    }
    {
        Region reg(ctx, G4A_K_CP_MERGE, ctx->stream);
        const float *pa_o[2] = {o[0], o[2]}, *pa_l[2] = {l[0], l[2]};
        const float *pb_o[2] = {o[1], o[3]}, *pb_l[2] = {l[1], l[3]};
        G4A_CUDA_TRY(ctx, launch_lse_merge(a0 > 0 ? 2 : 1, pa_o, pa_l, c, kHeads, hd, outA, nullptr, ctx->stream));
        G4A_CUDA_TRY(ctx, launch_lse_merge(2, pb_o, pb_l, c, kHeads, hd, outB, nullptr, ctx->stream));
        reg.end();
    }
    return G4A_OK;
}

// Queries gathered; each rank attends every row that sees its own key chunks
// (its own rows first, while the gather runs); the ranks' partial results
// merged by an all-reduce (MAX) of the row maxima and a reduce-scatter (SUM)
// of the weighted outputs and weights.
int schedule_kv_shards(g4a_ctx *ctx, NcclApi &api, ncclComm_t comm, CpState *s, int W, int r,
                       const g4a_cp_problem &p) {
    const int32_t hd = p.head_dim, T = p.seq_len, c = T / (2 * W);
    const size_t qrow = (size_t)kHeads * hd, krow = (size_t)hd;
    const int32_t a0 = r * c, a1 = a0 + c, b0 = (2 * W - 1 - r) * c, b1 = b0 + c;
    const size_t stride = qrow + kHeads;  // packed row: weighted outputs, then weights
    int rc;
    if ((rc = grow_cp(ctx, s, &s->gathered, &s->gathered_cap, (size_t)T * qrow))) return rc;
    uint16_t *q_all = s->gathered;
    const void *qA = p.q_dev, *qB = bf16_at(p.q_dev, (size_t)c * qrow);
    const void *kA = p.k_dev, *kB = bf16_at(p.k_dev, (size_t)c * krow);
    const void *vA = p.v_dev, *vB = bf16_at(p.v_dev, (size_t)c * krow);
    // partial segments: rows [t0, t1) against key chunk A (kv_pos0 a0) or B (b0)
    struct Seg {
        int32_t t0, t1;
        bool chunk_b, own;
    };
    std::vector<Seg> segs = {{a0, a1, false, true}, {b0, b1, false, true}, {b0, b1, true, true}};
    if (b0 > a1) segs.push_back({a1, b0, false, false});
    if (T > b1) {
        segs.push_back({b1, T, false, false});
        segs.push_back({b1, T, true, false});
    }
    size_t rows = 0;
    for (const auto &g : segs) rows += (size_t)(g.t1 - g.t0);
    if ((rc = grow_cp(ctx, s, &s->part, &s->part_cap, rows * (qrow + kHeads)))) return rc;
    if ((rc = grow_cp(ctx, s, &s->rowmax, &s->rowmax_cap, (size_t)T * kHeads))) return rc;
    if ((rc = grow_cp(ctx, s, &s->packed, &s->packed_cap, (size_t)T * stride))) return rc;
    if ((rc = grow_cp(ctx, s, &s->recv, &s->recv_cap, 2 * (size_t)c * stride))) return rc;
    CpSegs dsegs{};
    std::vector<g4a_prefill_problem> local, remote;
    size_t at_o = 0, at_l = rows * qrow;
    for (const auto &g : segs) {
        const int32_t n = g.t1 - g.t0;
        float *o = s->part + at_o, *l = s->part + at_l;
        at_o += (size_t)n * qrow;
        at_l += (size_t)n * kHeads;
        const void *q = g.own ? (g.t0 == a0 ? qA : qB) : static_cast<const void *>(q_all + (size_t)g.t0 * qrow);
        const g4a_prefill_problem pr = g.chunk_b ? problem(hd, q, n, g.t0, kB, vB, c, b0, o, l)
                                                 : problem(hd, q, n, g.t0, kA, vA, c, a0, o, l);
        (g.own ? local : remote).push_back(pr);
        dsegs.s[dsegs.n++] = CpSeg{g.t0, g.t1, o, l};
    }

    G4A_CUDA_TRY(ctx, cudaEventRecord(s->ev_start, ctx->stream));
    G4A_CUDA_TRY(ctx, cudaStreamWaitEvent(s->side, s->ev_start, 0));
    {
        Region reg(ctx, G4A_K_CP_EXCHANGE, s->side);
        G4A_NCCL_TRY(ctx, api, comm, api.AllGather(qA, q_all, (size_t)c * qrow, ncclBfloat16, comm, s->side));
        if (W > 1) {
            G4A_NCCL_TRY(ctx, api, comm, api.GroupStart());
            Group g(api);
            for (int j = 0; j < W; j++) {
                if (j == r) continue;
                G4A_GROUP_CALL(g, api.Send(qB, (size_t)c * qrow, ncclBfloat16, j, comm, s->side));
                G4A_GROUP_CALL(g, api.Recv(q_all + (size_t)(2 * W - 1 - j) * c * qrow, (size_t)c * qrow,
                                           ncclBfloat16, j, comm, s->side));
            }
            if ((rc = g.close(ctx, comm))) return rc;
        }
        reg.end();
    }
    G4A_CUDA_TRY(ctx, cudaEventRecord(s->ev_gathered, s->side));
    {
        Region reg(ctx, G4A_K_CP_ATTEND_LOCAL, ctx->stream);
        if ((rc = run_prefill(ctx, local, W > 1 ? exchange_sms() : 0))) return rc;
        reg.end();
    }
    G4A_CUDA_TRY(ctx, cudaStreamWaitEvent(ctx->stream, s->ev_gathered, 0));
    {
        Region reg(ctx, G4A_K_CP_ATTEND_REMOTE, ctx->stream);
        if ((rc = run_prefill(ctx, remote))) return rc;
        reg.end();
    }
    {
        Region reg(ctx, G4A_K_CP_MERGE, ctx->stream);
        G4A_CUDA_TRY(ctx, launch_cp_rowmax(dsegs, T, s->rowmax, ctx->stream));
        reg.end();
    }
    {
        Region reg(ctx, G4A_K_CP_EXCHANGE, ctx->stream);
        G4A_NCCL_TRY(ctx, api, comm,
                     api.AllReduce(s->rowmax, s->rowmax, (size_t)T * kHeads, ncclFloat32, ncclMax, comm, ctx->stream));
        reg.end();
    }
    {
        Region reg(ctx, G4A_K_CP_MERGE, ctx->stream);
        G4A_CUDA_TRY(ctx, launch_cp_pack(dsegs, s->rowmax, W, c, hd, s->packed, ctx->stream));
        reg.end();
    }
    {
        Region reg(ctx, G4A_K_CP_EXCHANGE, ctx->stream);
        G4A_NCCL_TRY(ctx, api, comm,
                     api.ReduceScatter(s->packed, s->recv, 2 * (size_t)c * stride, ncclFloat32, ncclSum, comm,
                                       ctx->stream));
        reg.end();
    }
    {
        Region reg(ctx, G4A_K_CP_MERGE, ctx->stream);
        G4A_CUDA_TRY(ctx, launch_cp_finish(s->recv, 2 * c, hd, p.out_dev, ctx->stream));
        reg.end();
    }
    return G4A_OK;
}

}  // namespace

extern "C" int g4a_cp_prefill(g4a_ctx *ctx, void *nccl_comm, int32_t schedule, const g4a_cp_problem *p) {
    if (!ctx) return G4A_COMPUTE;
    cudaSetDevice(ctx->device);
    if (!nccl_comm || !p) return fail(ctx, G4A_COMPUTE, "compute: null communicator or problem");
    if (schedule != G4A_CP_KV_SHARDS && schedule != G4A_CP_GATHER_KV)
        return fail(ctx, G4A_COMPUTE, "compute: unknown context-parallel schedule %d", schedule);
    if (ctx->hp.n_heads != kHeads || ctx->hp.n_kv_heads != 1)
        return fail(ctx, G4A_COMPUTE, "compute: prefill serves %d query heads over 1 KV head", kHeads);
    if (p->head_dim != 256 && p->head_dim != 512)
        return fail(ctx, G4A_COMPUTE, "compute: prefill head width must be 256 or 512");
    NcclApi &api = nccl();
    if (!api.ok) return fail(ctx, G4A_NCCL, "nccl: %s", api.why.c_str());
    ncclComm_t comm = static_cast<ncclComm_t>(nccl_comm);
    int W = 0, r = -1;
    G4A_NCCL_TRY(ctx, api, comm, api.CommCount(comm, &W));
    G4A_NCCL_TRY(ctx, api, comm, api.CommUserRank(comm, &r));
    if (W <= 0 || r < 0 || r >= W) return fail(ctx, G4A_NCCL, "nccl: communicator of %d ranks, rank %d", W, r);
    if (p->seq_len <= 0 || p->seq_len % (2 * W) != 0 || (int64_t)p->seq_len * kHeads > INT32_MAX)
        return fail(ctx, G4A_COMPUTE, "compute: sequence length %d is not a positive multiple of 2 x %d ranks",
                    p->seq_len, W);
    if (!p->q_dev || !p->k_dev || !p->v_dev || !p->out_dev)
        return fail(ctx, G4A_COMPUTE, "compute: null context-parallel buffers");
    if (((uintptr_t)p->q_dev | (uintptr_t)p->k_dev | (uintptr_t)p->v_dev | (uintptr_t)p->out_dev) & 15u)
        return fail(ctx, G4A_COMPUTE, "compute: context-parallel buffers must be 16-byte aligned");
    CpState *s = nullptr;
    int rc = cp_state(ctx, &s);
    if (rc) return rc;
    return schedule == G4A_CP_KV_SHARDS ? schedule_kv_shards(ctx, api, comm, s, W, r, *p)
                                        : schedule_gather_kv(ctx, api, comm, s, W, r, *p);
}

extern "C" int g4a_cp_wait(g4a_ctx *ctx, void *nccl_comm, int32_t timeout_ms) {
    if (!ctx) return G4A_COMPUTE;
    cudaSetDevice(ctx->device);
    if (!nccl_comm || timeout_ms < 0) return fail(ctx, G4A_COMPUTE, "compute: invalid wait arguments");
    NcclApi &api = nccl();
    if (!api.ok) return fail(ctx, G4A_NCCL, "nccl: %s", api.why.c_str());
    ncclComm_t comm = static_cast<ncclComm_t>(nccl_comm);
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t q = cudaStreamQuery(ctx->stream);
        if (q == cudaSuccess) break;
        if (q != cudaErrorNotReady) return cuda_fail(ctx, q, "cudaStreamQuery");
        ncclResult_t a = ncclSuccess;
        const ncclResult_t qr = api.CommGetAsyncError(comm, &a);
        if (qr != ncclSuccess || (a != ncclSuccess && a != ncclInProgress)) {
            const ncclResult_t bad = qr != ncclSuccess ? qr : a;
            api.CommAbort(comm);
            return fail(ctx, G4A_NCCL, "nccl: communicator error (%s); communicator aborted", api.GetErrorString(bad));
        }
        if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) {
            api.CommAbort(comm);
            return fail(ctx, G4A_TIMEOUT, "nccl: the queued work did not finish within %d ms; communicator aborted",
                        timeout_ms);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    return g4a_sync(ctx);
}

extern "C" int g4a_nccl_unique_id(uint8_t *id) {
    if (!id) return G4A_COMPUTE;
    NcclApi &api = nccl();
    if (!api.ok) return G4A_NCCL;
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
    ncclUniqueId u;
    if (api.GetUniqueId(&u) != ncclSuccess) return G4A_NCCL;
    std::memcpy(id, &u, sizeof u);
    return G4A_OK;
}

extern "C" int g4a_nccl_comm_init(int32_t n_ranks, int32_t rank, const uint8_t *id, int device, void **comm_out) {
    if (!id || !comm_out || n_ranks <= 0 || rank < 0 || rank >= n_ranks) return G4A_COMPUTE;
    *comm_out = nullptr;
    NcclApi &api = nccl();
    if (!api.ok) return G4A_NCCL;
    if (cudaSetDevice(device) != cudaSuccess) return G4A_CUDA;
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof u);
    ncclComm_t comm = nullptr;
    if (api.CommInitRank(&comm, n_ranks, u, rank) != ncclSuccess) return G4A_NCCL;
    *comm_out = comm;
    return G4A_OK;
}

extern "C" void g4a_nccl_comm_destroy(void *comm) {
    if (!comm) return;
    NcclApi &api = nccl();
    if (api.ok) api.CommDestroy(static_cast<ncclComm_t>(comm));
}
