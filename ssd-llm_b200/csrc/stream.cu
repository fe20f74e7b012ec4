// stream.cu — SSD -> HBM streaming tier: decode a model whose layer matrices live in a GGUF
// file and pass through a budgeted set of HBM layer slots.
//
// The reference streams layers from disk for models larger than memory: SsdStreamer
// (src/ssd/streamer.rs:34-80) loads a layer's tensors from the mmap'd file on a cache miss,
// LayerCache (src/model/cache.rs) keeps loaded layers under a byte budget with LRU eviction,
// pinning and hit / miss / eviction / prefetch-hit counters, and Prefetcher
// (src/ssd/prefetch.rs:24-67) looks `LookAhead(n)` layers ahead (madvise WILLNEED) before
// each layer runs (transformer.rs:151-163). Here the cache is HBM: n_slots = budget / slot
// bytes device slots, each sized for the largest layer in the library's weight layout.
//  * A miss reads the layer's seven matrices from the file (pread, up to 8 threads per tensor,
//    into one of two pinned host buffers), copies them to the device on a copy stream and repacks them into the slot
//    (the same repack as ssd_weight_upload); the layer's kernels are enqueued once the
//    slot's `ready` event has completed.
//  * After a layer's kernels are enqueued, the next `lookahead` layers are loaded the same way
//    (wrapping past the last layer to the next token's first ones), so the host's file reads
//    and the copies overlap the GPU's work on the layers before them.
//  * A slot is reused only after the compute stream has passed its `released` event (recorded
//    after the last kernels that read it): the copy stream waits on it, the host never does
//    except to reuse a pinned buffer whose copy is still queued.
//  * Victims: a free slot, else the least recently used one whose layer is neither pinned nor
//    inside the current prefetch window.
// Norms, token_embd, output_norm and output are loaded once into the model (resident).
// Differences from the reference, each a B200 choice: the cache holds quantized weights in
// HBM, not f32 copies in RAM; the prefetch loads into HBM instead of hinting the page cache;
// the lookahead wraps to the next token. tp_size 1 only.
#include <fcntl.h>
#include <unistd.h>

#include <algorithm>
#include <array>
#include <string>
#include <thread>
#include <vector>

#include "model.cuh"

namespace {

constexpr int kMats = 7;
const char* const kMatNames[kMats] = {"attn_q", "attn_k",   "attn_v",  "attn_output",
                                      "ffn_gate", "ffn_up", "ffn_down"};

struct Mat {
    int type = 0, rows = 0, cols = 0;
    uint64_t file_off = 0;  // absolute offset in the file
    size_t raw = 0;         // the reference's bytes
    size_t off = 0;         // offset in the slot
    ssd::WeightLayout lay;
};

struct Slot {
    uint8_t* base = nullptr;
    int layer = -1;
    ssd_weight w[kMats];
    ssd_weight* wp[kMats] = {};
    cudaEvent_t ready = nullptr, released = nullptr;
    uint64_t used = 0;  // LRU tick
};

}  // namespace

struct ssd_stream {
    ssd_model* m = nullptr;
    ssd_ctx* ctx = nullptr;
    int fd = -1;
    int n_layers = 0, lookahead = 0, cur = 0;
    std::vector<std::array<Mat, kMats>> mats;
    size_t slot_bytes = 0, raw_max = 0;
    std::vector<Slot> slots;
    std::vector<int> slot_of;
    std::vector<char> pinned, prefetched;
    void* raw_dev = nullptr;  // device staging of one tensor's raw bytes (repacked types)
    void* host[2] = {nullptr, nullptr};
    cudaEvent_t host_free[2] = {nullptr, nullptr};
    int next_host = 0;
    cudaStream_t copy = nullptr;
    uint64_t tick = 0;
    ssd_stream_stats st = {};
};

using namespace ssd;

namespace {

int read_at(int fd, void* dst, size_t n, uint64_t off) {
    uint8_t* p = (uint8_t*)dst;
    while (n) {
        const ssize_t r = pread(fd, p, n, (off_t)off);
        SSD_REQ(r > 0, SSD_ERR_ARG, "short read of the model file at offset %llu",
                (unsigned long long)off);
        p += r;
        n -= (size_t)r;
        off += (uint64_t)r;
    }
    return SSD_OK;
}

// The same from up to 8 host threads for large tensors (page-cache copies and NVMe queues
// both scale with readers).
int read_parallel(int fd, void* dst, size_t n, uint64_t off) {
    constexpr size_t kChunk = (size_t)4 << 20;
    const int k = (int)std::min<size_t>(8, n / kChunk);
    if (k < 2) return read_at(fd, dst, n, off);
    std::vector<std::thread> th;
    std::vector<int> st(k, SSD_OK);
    const size_t per = (n + k - 1) / k;
    for (int i = 0; i < k; i++) {
        const size_t a = (size_t)i * per, len = std::min(per, n - a);
        th.emplace_back([&, i, a, len] { st[i] = read_at(fd, (uint8_t*)dst + a, len, off + a); });
    }
    for (auto& t : th) t.join();
    for (int i = 0; i < k; i++)  // errors are recorded per thread: restate it on this one
        SSD_REQ(st[i] == SSD_OK, st[i], "short read of the model file at offset %llu",
                (unsigned long long)(off + (size_t)i * per));
    return SSD_OK;
}

// Layer l's matrices into slot `si` (after its previous layer's kernels are done).
int load_layer(ssd_stream* S, int l, int si) {
    Slot& sl = S->slots[si];
    if (sl.layer >= 0) {
        S->slot_of[sl.layer] = -1;
        S->prefetched[sl.layer] = 0;
        S->st.evictions++;
    }
    sl.layer = -1;
    SSD_CK(cudaStreamWaitEvent(S->copy, sl.released, 0));
    size_t bytes = 0;
    for (int j = 0; j < kMats; j++) {
        const Mat& t = S->mats[l][j];
        carve_weight(S->ctx, t.type, t.rows, t.cols, t.lay, sl.base + t.off, &sl.w[j]);
        if (t.lay.fix)
            SSD_CK(cudaMemsetAsync(sl.w[j].fix_counter, 0, t.lay.counter_bytes, S->copy));
        const int b = S->next_host;
        S->next_host ^= 1;
        SSD_CK(cudaEventSynchronize(S->host_free[b]));  // its last copy has left the buffer
        SSD_TRY(read_parallel(S->fd, S->host[b], t.raw, t.file_off));
        const bool as_is = type_block(t.type) == 1 || is_lowbit(t.type);
        SSD_CK(cudaMemcpyAsync(as_is ? (void*)sl.w[j].qs : S->raw_dev, S->host[b], t.raw,
                               cudaMemcpyHostToDevice, S->copy));
        SSD_CK(cudaEventRecord(S->host_free[b], S->copy));
        if (!as_is) SSD_TRY(upload_raw(&sl.w[j], S->raw_dev, S->copy));
        bytes += t.raw;
    }
    SSD_CK(cudaEventRecord(sl.ready, S->copy));
    sl.layer = l;
    S->slot_of[l] = si;
    S->st.loads++;
    S->st.bytes_read += bytes;
    return SSD_OK;
}

// Is layer x inside the window of layers [from, from + n) (mod n_layers)?
bool in_window(const ssd_stream* S, int x, int from, int n) {
    const int d = ((x - from) % S->n_layers + S->n_layers) % S->n_layers;
    return d < n;
}

// A slot for a new layer: a free one, else the least recently used one whose layer is not
// pinned and not in the window [from, from + n); -1 if there is none.
int pick_slot(const ssd_stream* S, int from, int n) {
    int best = -1;
    for (int i = 0; i < (int)S->slots.size(); i++) {
        const int L = S->slots[i].layer;
        if (L < 0) return i;
        if (S->pinned[L] || in_window(S, L, from, n)) continue;
        if (best < 0 || S->slots[i].used < S->slots[best].used) best = i;
    }
    return best;
}

int acquire(void* user, int l, cudaStream_t s, ssd_weight* const* (&w)) {
    ssd_stream* S = (ssd_stream*)user;
    S->cur = l;
    int si = S->slot_of[l];
    if (si >= 0) {
        S->st.hits++;
        if (S->prefetched[l]) {
            S->st.prefetch_hits++;
            S->prefetched[l] = 0;
        }
    } else {
        S->st.misses++;
        si = pick_slot(S, l, 1);  // any unpinned layer but this one
        SSD_REQ(si >= 0, SSD_ERR_NOMEM, "every HBM layer slot holds a pinned layer");
        SSD_TRY(load_layer(S, l, si));
    }
    S->slots[si].used = ++S->tick;
    // The host waits for the slot's copies before enqueueing the layer: its first kernel
    // prefetches weights ahead of its programmatic-launch wait, so the matrices must be in
    // place before that kernel exists (the GPU keeps working on the layers before it).
    SSD_CK(cudaEventSynchronize(S->slots[si].ready));
    SSD_CK(cudaStreamWaitEvent(s, S->slots[si].ready, 0));
    w = S->slots[si].wp;
    return SSD_OK;
}

int release(void* user, int l, cudaStream_t s) {
    ssd_stream* S = (ssd_stream*)user;
    SSD_CK(cudaEventRecord(S->slots[S->slot_of[l]].released, s));
    // look ahead (Prefetcher::on_layer_start's LookAhead(n)): layers l+1 .. l+n, wrapping
    for (int i = 1; i <= S->lookahead && i < S->n_layers; i++) {
        const int n = (l + i) % S->n_layers;
        if (S->slot_of[n] >= 0) continue;
        const int si = pick_slot(S, l + 1, S->lookahead);
        if (si < 0) break;
        SSD_TRY(load_layer(S, n, si));
        S->slots[si].used = ++S->tick;
        S->prefetched[n] = 1;
    }
    return SSD_OK;
}

void destroy(ssd_stream* S) {
    if (S->copy) cudaStreamSynchronize(S->copy);
    for (Slot& sl : S->slots) {
        if (sl.ready) cudaEventDestroy(sl.ready);
        if (sl.released) cudaEventDestroy(sl.released);
        if (sl.base) cudaFree(sl.base);
    }
    for (int b = 0; b < 2; b++) {
        if (S->host_free[b]) cudaEventDestroy(S->host_free[b]);
        if (S->host[b]) cudaFreeHost(S->host[b]);
    }
    if (S->raw_dev) cudaFree(S->raw_dev);
    if (S->copy) cudaStreamDestroy(S->copy);
    if (S->fd >= 0) close(S->fd);
    delete S;
}

}  // namespace

extern "C" int ssd_stream_open(ssd_model* m, const char* gguf_path, size_t hbm_budget,
                               int lookahead, ssd_stream** out) {
    SSD_REQ(m && gguf_path && out, SSD_ERR_ARG, "null argument");
    SSD_REQ(lookahead >= 0, SSD_ERR_ARG, "negative lookahead");
    ssd_ctx* ctx = model_ctx(m);
    SSD_TRY(check_ctx(ctx));
    const ssd_model_config& c = model_cfg(m);
    SSD_REQ(c.tp_size <= 1, SSD_ERR_ARG, "the streaming tier runs at tp_size 1");
    // the step binds each layer's slot matrices for its enqueue only and leaves the layer
    // empty: a model with matrices of its own would lose them
    SSD_REQ(!model_has_layer_matrices(m), SSD_ERR_STATE,
            "the model already holds layer matrices; the streaming tier supplies them");
    ssd_gguf* g = nullptr;
    SSD_TRY(ssd_gguf_open(gguf_path, &g));
    ssd_stream* S = new ssd_stream();
    S->m = m;
    S->ctx = ctx;
    S->n_layers = c.n_layers;
    S->lookahead = lookahead;
    uint64_t data_off = 0;
    int st = ssd_gguf_info(g, nullptr, nullptr, nullptr, &data_off);
    auto fail = [&](int code) {
        ssd_gguf_close(g);
        destroy(S);
        return code;
    };
    if (st != SSD_OK) return fail(st);
    // every layer's matrices: type, shape, file range, place in the slot
    S->mats.resize(c.n_layers);
    for (int l = 0; l < c.n_layers && st == SSD_OK; l++) {
        size_t off = 0;
        for (int j = 0; j < kMats && st == SSD_OK; j++) {
            const std::string name = "blk." + std::to_string(l) + "." + kMatNames[j] + ".weight";
            int64_t idx = -1;
            st = ssd_gguf_find(g, name.c_str(), &idx);
            if (st != SSD_OK) break;
            if (idx < 0) {
                set_error("GGUF: tensor %s missing", name.c_str());
                st = SSD_ERR_ARG;
                break;
            }
            uint32_t nd = 0, type = 0;
            uint64_t dims[8] = {0}, toff = 0, tsize = 0;
            st = ssd_gguf_tensor(g, (uint64_t)idx, nullptr, 0, &nd, dims, &type, &toff, &tsize);
            if (st != SSD_OK) break;
            if (nd != 2) {
                set_error("GGUF: %s is not a matrix", name.c_str());
                st = SSD_ERR_SHAPE;
                break;
            }
            Mat& t = S->mats[l][j];
            t.type = (int)type;
            t.cols = (int)dims[0];  // ne0: elements per row
            t.rows = (int)dims[1];
            t.file_off = data_off + toff;
            t.raw = (size_t)tsize;
            if (ssd_row_bytes(t.type, t.cols) * (size_t)t.rows != t.raw) {
                set_error("GGUF: %s size does not match its shape", name.c_str());
                st = SSD_ERR_SHAPE;
                break;
            }
            st = weight_layout(t.type, t.rows, t.cols, &t.lay);
            t.off = off;
            off += t.lay.total;
            if (t.raw > S->raw_max) S->raw_max = t.raw;
        }
        if (off > S->slot_bytes) S->slot_bytes = off;
    }
    // resident tensors: the norms of every layer and the global ones, through the model
    std::vector<uint8_t> buf;
    auto load_resident = [&](const std::string& file_name, const char* model_name, int layer) {
        int64_t idx = -1;
        SSD_TRY(ssd_gguf_find(g, file_name.c_str(), &idx));
        SSD_REQ(idx >= 0, SSD_ERR_ARG, "GGUF: tensor %s missing", file_name.c_str());
        uint32_t type = 0;
        uint64_t tsize = 0;
        SSD_TRY(ssd_gguf_tensor(g, (uint64_t)idx, nullptr, 0, nullptr, nullptr, &type, nullptr,
                                &tsize));
        buf.resize((size_t)tsize);
        SSD_TRY(ssd_gguf_read(g, (uint64_t)idx, buf.data(), buf.size()));
        return ssd_model_set_tensor_typed(m, model_name, layer, buf.data(), buf.size(), (int)type);
    };
    for (int l = 0; l < c.n_layers && st == SSD_OK; l++) {
        st = load_resident("blk." + std::to_string(l) + ".attn_norm.weight", "attn_norm", l);
        if (st == SSD_OK)
            st = load_resident("blk." + std::to_string(l) + ".ffn_norm.weight", "ffn_norm", l);
    }
    if (st == SSD_OK) st = load_resident("token_embd.weight", "token_embd", -1);
    if (st == SSD_OK) st = load_resident("output_norm.weight", "output_norm", -1);
    if (st == SSD_OK) {
        int64_t oi = -1;
        st = ssd_gguf_find(g, "output.weight", &oi);
        if (st == SSD_OK)
            st = load_resident(oi >= 0 ? "output.weight" : "token_embd.weight", "output", -1);
    }
    ssd_gguf_close(g);
    g = nullptr;
    auto fail2 = [&](int code) {
        destroy(S);
        return code;
    };
    if (st != SSD_OK) return fail2(st);
    // the slots the budget pays for (at least one, at most one per layer)
    S->slot_bytes = (S->slot_bytes + 255) & ~(size_t)255;
    size_t n_slots = hbm_budget / S->slot_bytes;
    if (n_slots > (size_t)c.n_layers) n_slots = (size_t)c.n_layers;
    if (n_slots < 1) {
        set_error("HBM budget of %zu bytes is below one layer (%zu bytes)", hbm_budget,
                  S->slot_bytes);
        return fail2(SSD_ERR_NOMEM);
    }
    cudaSetDevice(ctx->device);
    S->slots.resize(n_slots);
    for (Slot& sl : S->slots) {
        if (cudaMalloc(&sl.base, S->slot_bytes) != cudaSuccess ||
            cudaEventCreateWithFlags(&sl.ready, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&sl.released, cudaEventDisableTiming) != cudaSuccess) {
            cudaGetLastError();
            set_error("HBM layer slot allocation failed");
            return fail2(SSD_ERR_NOMEM);
        }
        for (int j = 0; j < kMats; j++) sl.wp[j] = &sl.w[j];
    }
    if (cudaStreamCreateWithFlags(&S->copy, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&S->raw_dev, S->raw_max) != cudaSuccess) {
        cudaGetLastError();
        set_error("copy stream / staging allocation failed");
        return fail2(SSD_ERR_NOMEM);
    }
    for (int b = 0; b < 2; b++)
        if (cudaMallocHost(&S->host[b], S->raw_max) != cudaSuccess ||
            cudaEventCreateWithFlags(&S->host_free[b], cudaEventDisableTiming) != cudaSuccess) {
            cudaGetLastError();
            set_error("pinned staging allocation failed");
            return fail2(SSD_ERR_NOMEM);
        }
    S->fd = open(gguf_path, O_RDONLY);
    if (S->fd < 0) {
        set_error("cannot open %s", gguf_path);
        return fail2(SSD_ERR_ARG);
    }
    posix_fadvise(S->fd, 0, 0, POSIX_FADV_SEQUENTIAL);  // the loader's MADV_SEQUENTIAL
    S->slot_of.assign(c.n_layers, -1);
    S->pinned.assign(c.n_layers, 0);
    S->prefetched.assign(c.n_layers, 0);
    S->st.n_slots = (int)n_slots;
    S->st.slot_bytes = S->slot_bytes;
    *out = S;
    return SSD_OK;
}

extern "C" int ssd_stream_pin(ssd_stream* S, int layer) {
    SSD_REQ(S && layer >= 0 && layer < S->n_layers, SSD_ERR_ARG, "bad layer");
    if (S->pinned[layer]) return SSD_OK;
    int pinned = 0;
    for (char p : S->pinned) pinned += p;
    SSD_REQ(pinned + 1 < (int)S->slots.size() || (int)S->slots.size() == S->n_layers,
            SSD_ERR_NOMEM, "pinning layer %d would leave no slot for the others", layer);
    if (S->slot_of[layer] < 0) {  // load it now, so that it stays resident from here on
        const int si = pick_slot(S, layer, 1);
        SSD_REQ(si >= 0, SSD_ERR_NOMEM, "no slot for layer %d", layer);
        SSD_TRY(load_layer(S, layer, si));
        S->slots[si].used = ++S->tick;
    }
    S->pinned[layer] = 1;
    return SSD_OK;
}

extern "C" int ssd_stream_decode_token(ssd_stream* S, int32_t token_in, int32_t* token_out) {
    SSD_REQ(S && token_out, SSD_ERR_ARG, "null argument");
    LayerHooks hk{acquire, release, S};
    return model_decode_token_hooked(S->m, token_in, token_out, hk);
}

extern "C" int ssd_stream_stats_get(const ssd_stream* S, ssd_stream_stats* out) {
    SSD_REQ(S && out, SSD_ERR_ARG, "null argument");
    *out = S->st;
    return SSD_OK;
}

extern "C" int ssd_stream_close(ssd_stream* S) {
    if (!S) return SSD_OK;
    cudaSetDevice(S->ctx->device);
    cudaStreamSynchronize(S->ctx->stream);
    destroy(S);
    return SSD_OK;
}
