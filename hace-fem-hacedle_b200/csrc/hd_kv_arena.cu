// hd_kv_arena.cu -- the device KV-cache manager: a fixed pool of KV slots in
// HBM, sessions and souls bound to slots, positions, and snapshots for
// branching (copies of a session's cached positions into a free slot).
//
// Replaces the runtime/kv_cache.rs skeleton: KvArena (:8-34), SessionKv
// (:37-56), SoulKv / SoulMemoryRegistry (:58-118) and the KvCacheManager
// trait (:121-127) with its KvError cases (:129-135).  The reference plans
// the arena but allocates nothing (null key/value pointers) and its
// snapshot/restore/swap are empty; here the pool is real device memory:
//   K and V, each [layers][slots][max_ctx][n_kv][head_dim] f32,
// the layout of the decoder's cache, so one layer's block is
// [slots][max_ctx][n_kv][head_dim] and the append / attention kernels index
// it by slot (hd_kv_append_slots, hd_attention_decode_slots).  f32, not the
// arena plan's 2 bytes per element, because the fp32 path's greedy tokens
// must be the oracle's.  Bookkeeping (names, positions, free slots) is host
// state; device work is one copy kernel per snapshot or restore.  KvError
// maps to: SessionNotFound / SoulNotFound -> HD_E_ARG, ContextFull ->
// HD_E_SHAPE, AllocationFailed -> HD_E_OOM, each with its name in the
// context's message.
#include <map>
#include <set>
#include <string>
#include <vector>

#include "hd_internal.cuh"

struct hd_kv_arena {
    hd_ctx *ctx = nullptr;
    int layers = 0, n_kv = 0, head_dim = 0, max_ctx = 0, slots = 0;
    float *k = nullptr, *v = nullptr;
    struct Session {
        int slot = -1, pos = 0;
        std::string soul;
    };
    struct Snap {
        int slot = -1, pos = 0;
        std::string session, soul;
    };
    std::map<std::string, Session> sessions;
    std::map<std::string, std::set<std::string>> souls;
    std::map<uint64_t, Snap> snaps;
    std::vector<int> free_slots;
    uint64_t next_snap = 1, clock = 0;
    int64_t slot_floats() const { return (int64_t)max_ctx * n_kv * head_dim; }
    int64_t layer_floats() const { return slot_floats() * slots; }
};

namespace {

// Copies positions [0, pos) of slot `src` to slot `dst` in every layer, K and
// V (grid.y = 2 * layers).
__global__ void k_kv_copy(float *k, float *v, int64_t layer_floats, int64_t slot_floats, int src, int dst,
                          int64_t count) {
    pdl_wait();
    pdl_trigger();
    const int l = blockIdx.y >> 1;
    float *base = (blockIdx.y & 1) ? v : k;
    const float4 *s = (const float4 *)(base + l * layer_floats + (int64_t)src * slot_floats);
    float4 *d = (float4 *)(base + l * layer_floats + (int64_t)dst * slot_floats);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count / 4; i += (int64_t)gridDim.x * blockDim.x)
        d[i] = s[i];
}

// Row r's k and v [n_kv * head_dim] appended to slot slots[r] at position pos[r].
__global__ void k_kv_append_slots(const float *__restrict__ k, const float *__restrict__ v, float *kc, float *vc,
                                  const int32_t *__restrict__ slots, const int32_t *__restrict__ pos, int rows,
                                  int width, int max_ctx) {
    pdl_wait();
    pdl_trigger();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)rows * width) return;
    const int r = (int)(i / width), e = (int)(i % width);
    const int p = pos[r];
    if (p < 0 || p >= max_ctx) return;  // KvCache::append ignores pos >= max_seq_len
    const int64_t dst = ((int64_t)slots[r] * max_ctx + p) * width + e;
    kc[dst] = k[i];
    vc[dst] = v[i];
}

int copy_slot(hd_kv_arena *a, int src, int dst, int pos) {
    if (pos <= 0 || src == dst) return HD_OK;
    const int64_t count = (int64_t)pos * a->n_kv * a->head_dim;  // head_dim % 4 == 0 (checked at create)
    const int64_t c4 = count / 4;
    const unsigned gx = (unsigned)(c4 + 255) / 256 < 64 ? (unsigned)((c4 + 255) / 256) : 64;
    HD_CUDA_TRY(a->ctx, hd_launch(a->ctx, k_kv_copy, dim3(gx > 0 ? gx : 1, (unsigned)(2 * a->layers)), dim3(256), 0,
                                  a->k, a->v, a->layer_floats(), a->slot_floats(), src, dst, count));
    return HD_OK;
}

int take_slot(hd_kv_arena *a, int *slot) {
    if (a->free_slots.empty()) return hd_fail(a->ctx, HD_E_OOM, "AllocationFailed: all %d KV slots are in use", a->slots);
    *slot = a->free_slots.back();
    a->free_slots.pop_back();
    return HD_OK;
}

hd_kv_arena::Session *find(hd_kv_arena *a, const char *sid) {
    auto it = a->sessions.find(sid);
    return it == a->sessions.end() ? nullptr : &it->second;
}

}  // namespace

extern "C" {

int hd_kv_arena_create(hd_ctx *ctx, int layers, int n_kv, int head_dim, int max_ctx, int slots, hd_kv_arena **out) {
    if (!ctx || !out) return hd_fail(ctx, HD_E_ARG, "hd_kv_arena_create: null argument");
    *out = nullptr;
    HD_REQUIRE(ctx, layers > 0 && n_kv > 0 && head_dim > 0 && head_dim % 4 == 0 && max_ctx > 0 && slots > 0,
               HD_E_SHAPE, "hd_kv_arena_create: bad shape (layers %d, n_kv %d, head_dim %d, max_ctx %d, slots %d)",
               layers, n_kv, head_dim, max_ctx, slots);
    hd_kv_arena *a = new hd_kv_arena;
    a->ctx = ctx;
    a->layers = layers;
    a->n_kv = n_kv;
    a->head_dim = head_dim;
    a->max_ctx = max_ctx;
    a->slots = slots;
    const size_t bytes = (size_t)a->layer_floats() * layers * sizeof(float);
    if (cudaMalloc(&a->k, bytes) != cudaSuccess || cudaMalloc(&a->v, bytes) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(a->k);
        delete a;
        return hd_fail(ctx, HD_E_OOM, "AllocationFailed: KV arena of 2 x %zu bytes", bytes);
    }
    for (int s = slots - 1; s >= 0; s--) a->free_slots.push_back(s);
    *out = a;
    return HD_OK;
}

int hd_kv_arena_free(hd_kv_arena *a) {
    if (!a) return HD_E_ARG;
    cudaStreamSynchronize(a->ctx->stream);
    cudaFree(a->k);
    cudaFree(a->v);
    delete a;
    return HD_OK;
}

int hd_kv_layer(hd_kv_arena *a, int layer, float **k_dev, float **v_dev) {
    if (!a || !k_dev || !v_dev) return hd_fail(a ? a->ctx : nullptr, HD_E_ARG, "hd_kv_layer: null argument");
    HD_REQUIRE(a->ctx, layer >= 0 && layer < a->layers, HD_E_ARG, "hd_kv_layer: layer %d of %d", layer, a->layers);
    *k_dev = a->k + layer * a->layer_floats();
    *v_dev = a->v + layer * a->layer_floats();
    return HD_OK;
}

int hd_kv_allocate(hd_kv_arena *a, const char *session_id, const char *soul_id, int *slot) {
    if (!a || !session_id || !soul_id) return hd_fail(a ? a->ctx : nullptr, HD_E_ARG, "hd_kv_allocate: null argument");
    if (hd_kv_arena::Session *s = find(a, session_id)) {  // get_or_create_session: existing sessions are kept
        if (slot) *slot = s->slot;
        return HD_OK;
    }
    int sl = -1;
    const int rc = take_slot(a, &sl);
    if (rc) return rc;
    a->sessions[session_id] = {sl, 0, soul_id};
    a->souls[soul_id].insert(session_id);
    if (slot) *slot = sl;
    return HD_OK;
}

int hd_kv_release(hd_kv_arena *a, const char *session_id) {
    if (!a || !session_id) return hd_fail(a ? a->ctx : nullptr, HD_E_ARG, "hd_kv_release: null argument");
    hd_kv_arena::Session *s = find(a, session_id);
    if (!s) return hd_fail(a->ctx, HD_E_ARG, "SessionNotFound: '%s'", session_id);
    a->free_slots.push_back(s->slot);
    auto so = a->souls.find(s->soul);
    so->second.erase(session_id);
    if (so->second.empty()) a->souls.erase(so);
    a->sessions.erase(session_id);
    return HD_OK;
}

int hd_kv_session(hd_kv_arena *a, const char *session_id, int *slot, int *position) {
    if (!a || !session_id) return hd_fail(a ? a->ctx : nullptr, HD_E_ARG, "hd_kv_session: null argument");
    hd_kv_arena::Session *s = find(a, session_id);
    if (!s) return hd_fail(a->ctx, HD_E_ARG, "SessionNotFound: '%s'", session_id);
    if (slot) *slot = s->slot;
    if (position) *position = s->pos;
    return HD_OK;
}

int hd_kv_advance(hd_kv_arena *a, const char *session_id, int count) {
    if (!a || !session_id || count < 0) return hd_fail(a ? a->ctx : nullptr, HD_E_ARG, "hd_kv_advance: bad argument");
    hd_kv_arena::Session *s = find(a, session_id);
    if (!s) return hd_fail(a->ctx, HD_E_ARG, "SessionNotFound: '%s'", session_id);
    if ((int64_t)s->pos + count > a->max_ctx)
        return hd_fail(a->ctx, HD_E_SHAPE, "ContextFull: '%s' at %d + %d > %d", session_id, s->pos, count, a->max_ctx);
    s->pos += count;
    return HD_OK;
}

int hd_kv_soul_sessions(hd_kv_arena *a, const char *soul_id, int *count) {
    if (!a || !soul_id || !count) return hd_fail(a ? a->ctx : nullptr, HD_E_ARG, "hd_kv_soul_sessions: null argument");
    auto so = a->souls.find(soul_id);
    if (so == a->souls.end()) return hd_fail(a->ctx, HD_E_ARG, "SoulNotFound: '%s'", soul_id);
    *count = (int)so->second.size();
    return HD_OK;
}

int hd_kv_snapshot(hd_kv_arena *a, const char *session_id, hd_kv_snapshot_t *out) {
    if (!a || !session_id || !out) return hd_fail(a ? a->ctx : nullptr, HD_E_ARG, "hd_kv_snapshot: null argument");
    hd_kv_arena::Session *s = find(a, session_id);
    if (!s) return hd_fail(a->ctx, HD_E_ARG, "SessionNotFound: '%s'", session_id);
    int sl = -1;
    int rc = take_slot(a, &sl);
    if (rc) return rc;
    rc = copy_slot(a, s->slot, sl, s->pos);
    if (rc) {
        a->free_slots.push_back(sl);
        return rc;
    }
    const uint64_t id = a->next_snap++;
    a->snaps[id] = {sl, s->pos, session_id, s->soul};
    out->snapshot_id = id;
    out->token_position = s->pos;
    out->slot = sl;
    out->kv_offset = (uint64_t)sl * (uint64_t)a->slot_floats() * sizeof(float);
    out->timestamp = ++a->clock;
    return HD_OK;
}

int hd_kv_restore(hd_kv_arena *a, const hd_kv_snapshot_t *snap, const char *session_id) {
    if (!a || !snap || !session_id) return hd_fail(a ? a->ctx : nullptr, HD_E_ARG, "hd_kv_restore: null argument");
    auto it = a->snaps.find(snap->snapshot_id);
    if (it == a->snaps.end()) return hd_fail(a->ctx, HD_E_ARG, "hd_kv_restore: unknown snapshot %llu",
                                             (unsigned long long)snap->snapshot_id);
    // the target session: existing, or a new one under the snapshot's soul (a branch)
    int rc = hd_kv_allocate(a, session_id, it->second.soul.c_str(), nullptr);
    if (rc) return rc;
    hd_kv_arena::Session *s = find(a, session_id);
    rc = copy_slot(a, it->second.slot, s->slot, it->second.pos);
    if (rc) return rc;
    s->pos = it->second.pos;
    return HD_OK;
}

int hd_kv_snapshot_free(hd_kv_arena *a, const hd_kv_snapshot_t *snap) {
    if (!a || !snap) return hd_fail(a ? a->ctx : nullptr, HD_E_ARG, "hd_kv_snapshot_free: null argument");
    auto it = a->snaps.find(snap->snapshot_id);
    if (it == a->snaps.end()) return hd_fail(a->ctx, HD_E_ARG, "hd_kv_snapshot_free: unknown snapshot %llu",
                                             (unsigned long long)snap->snapshot_id);
    a->free_slots.push_back(it->second.slot);
    a->snaps.erase(it);
    return HD_OK;
}

int hd_kv_append_slots(hd_ctx *ctx, const float *k, const float *v, float *kc, float *vc, const int32_t *slots_dev,
                       const int32_t *pos_dev, int rows, int n_kv, int head_dim, int max_ctx) {
    if (!ctx || !k || !v || !kc || !vc || !slots_dev || !pos_dev)
        return hd_fail(ctx, HD_E_ARG, "hd_kv_append_slots: null argument");
    HD_REQUIRE(ctx, rows >= 0 && n_kv > 0 && head_dim > 0 && max_ctx > 0, HD_E_SHAPE, "hd_kv_append_slots: bad shape");
    const int64_t total = (int64_t)rows * n_kv * head_dim;
    if (total == 0) return HD_OK;
    HD_CUDA_TRY(ctx, hd_launch(ctx, k_kv_append_slots, dim3((unsigned)((total + 255) / 256)), dim3(256), 0, k, v, kc, vc,
                               slots_dev, pos_dev, rows, n_kv * head_dim, max_ctx));
    return HD_OK;
}

int hd_attention_decode_slots(hd_ctx *ctx, const float *q, const float *kc, const float *vc, const int32_t *slots_dev,
                              const int32_t *len_dev, int rows, int n_heads, int n_kv, int head_dim, int max_ctx,
                              float *out) {
    if (!len_dev || !slots_dev) return hd_fail(ctx, HD_E_ARG, "hd_attention_decode_slots: null lengths or slots");
    return hd_attention_run(ctx, q, 0, kc, vc, len_dev, rows, 0, 1, n_heads, n_kv, head_dim, max_ctx, max_ctx, out,
                            "hd_attention_decode_slots", slots_dev);
}

}  // extern "C"
