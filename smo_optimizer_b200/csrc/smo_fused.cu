// smo_fused.cu -- host side of the fused single-pass step (smo_fused.cuh):
// which tensors it takes, the launch plan (window-shape groups, strip
// lengths), the workspace layout, and one launch per group through the
// instance of the group's storage type.
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "smo_fused.cuh"

namespace smo {

// Poll limit of the inter-CTA waits (smo_set_wait_limit; negative = default)
static std::atomic<int64_t> g_wait_limit{-1};
// Diagnostic: waits look for a flag value that no strip publishes
// (smo_inject_wait_timeout), so each runs out its poll limit
static std::atomic<unsigned int> g_wait_skew{0};

int64_t wait_limit() {
    const int64_t v = g_wait_limit.load(std::memory_order_relaxed);
    return v < 0 ? kDefaultWaitIters : v;
}

int64_t set_wait_limit(int64_t polls) { return g_wait_limit.exchange(polls < 0 ? -1 : polls); }

int inject_wait_timeout(int on) { return (int)g_wait_skew.exchange(on ? 1u : 0u); }

unsigned int wait_skew() { return g_wait_skew.load(std::memory_order_relaxed); }

// ---------------------------------------------------------------- host side

static bool supported_window(int64_t k) { return k == 2 || k == 4 || k == 8; }

static int64_t gcd64(int64_t a, int64_t b) {
    while (b) {
        int64_t t = a % b;
        a = b;
        b = t;
    }
    return a;
}

static FastDiv make_fast_div(uint32_t d) {
    FastDiv f;
    f.d = d;
    uint32_t l = 0;
    while (l < 32 && (1ull << l) < d) l++;
    f.l = l;
    f.m = (uint32_t)(((((uint64_t)1 << l) - d) << 32) / d + 1);
    return f;
}

// Compact rows per strip for a target length: a multiple of the rows after
// which int8 blocks realign with row starts, at most the tensor's rows.
static int64_t strip_rows(const smo_tensor &t, int64_t target) {
    int64_t align = 1;
    if (t.kind == SMO_KIND_POOLED8) align = t.q_block / gcd64(t.comp_cols, t.q_block);
    int64_t L = (target + align - 1) / align * align;
    return L < t.comp_rows ? L : t.comp_rows;
}

bool fused_takes(const smo_tensor &t) {
    if (t.kind != SMO_KIND_POOLED8 && t.kind != SMO_KIND_POOLED32) return false;
    if (t.flags & SMO_FLAG_GENERAL_PATH) return false;
    if (t.dtype != SMO_DTYPE_F32 && t.dtype != SMO_DTYPE_BF16 && t.dtype != SMO_DTYPE_F16) return false;
    if (t.row_perm || t.col_perm || t.row_perm_inv || t.col_perm_inv) return false;  // permute_basis
    if (t.rows <= 0 || t.cols <= 0 || t.comp_rows <= 0 || t.comp_cols <= 0) return false;
    if (t.rows % t.comp_rows != 0 || t.cols % t.comp_cols != 0) return false;
    const int64_t kh = t.rows / t.comp_rows, kw = t.cols / t.comp_cols;
    if (!supported_window(kh) || !supported_window(kw)) return false;
    if (t.cols <= 128) return false;  // torch's small-output interpolation order
    if (t.comp_cols > kMaxFusedCols) return false;
    if (t.comp_rows * t.comp_cols >= ((int64_t)1 << 31)) return false;  // 32-bit cell indices
    if (t.rows >= ((int64_t)1 << 24)) return false;  // exact float row coordinates (compute_rowco)
    if (t.kind == SMO_KIND_POOLED8 && t.q_block > t.comp_cols) return false;
    // one window row is one or two vector accesses of kw elements
    const size_t row_bytes = (size_t)kw * (t.dtype == SMO_DTYPE_F32 ? 4 : 2);
    const size_t a = row_bytes < 16 ? row_bytes : 16;
    if ((uintptr_t)t.param % a || (uintptr_t)t.grad % a) return false;
    if (t.interp_band < 0) return false;
    // the look-ahead reads the next strip's OLD state while that strip writes
    // the new one: in-place state would race, so it needs separate buffers
    if (t.kind == SMO_KIND_POOLED8 &&
        ((const void *)t.m_q_in == (const void *)t.m_q_out || (const void *)t.m_s_in == (const void *)t.m_s_out ||
         (const void *)t.v_q_in == (const void *)t.v_q_out || (const void *)t.v_s_in == (const void *)t.v_s_out))
        return false;
    if (t.kind == SMO_KIND_POOLED32 &&
        ((const void *)t.m_in == (const void *)t.m_out || (const void *)t.v_in == (const void *)t.v_out))
        return false;
    return true;
}

static int64_t num_strips(const smo_tensor &t, int64_t target) {
    const int64_t L = strip_rows(t, target);
    return (t.comp_rows + L - 1) / L;
}

// launch key: storage type and window shape (one kernel instance per key)
static int window_key(const smo_tensor &t) {
    return (int)(t.dtype * 256 + (t.rows / t.comp_rows) * 16 + (t.cols / t.comp_cols));
}

// CTA width of a launch: 192 threads (four CTAs of 80 registers per SM, so
// four independent row pipelines hide each other's load latency), or 256 or
// 128 (six CTAs per SM) when that leaves fewer idle thread-columns over the
// batch's compact rows (a compact row of w cells takes ceil(w / NT) passes of
// NT threads); ties keep 192.  Narrow rows are where 128 wins: the TinyViT and
// char-LM sets (rows of 96-512 cells) step 5-11 % faster with it, while the
// 700M decoder's rows (384-1536 cells, no idle columns at 192) run 5-8 %
// slower with it, whole or in per-rank shares.
// SMO_B200_FUSED_THREADS (128, 192, 256 or 384) forces one width, for
// measurements.
int pick_threads(const FusedBatch &b) {
    static int forced = -1;
    if (forced < 0) {
        const char *e = getenv("SMO_B200_FUSED_THREADS");
        forced = e ? atoi(e) : 0;
    }
    if (forced == 128 || forced == 192 || forced == 256 || forced == 384) return forced;
    int64_t idle128 = 0, idle192 = 0, idle256 = 0;
    for (int i = 0; i < b.n; i++) {
        const int64_t w = b.d[i].w, rows = b.d[i].h;
        idle128 += rows * ((w + 127) / 128 * 128 - w);
        idle192 += rows * ((w + 191) / 192 * 192 - w);
        idle256 += rows * ((w + 255) / 256 * 256 - w);
    }
    if (idle128 < idle192 && idle128 < idle256) return 128;
    return idle256 < idle192 ? 256 : 192;
}

int current_device() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
    return dev;
}

// SM count of the current device, queried once per device
int device_sm_count() {
    static int cached[kMaxDevices];
    const int dev = current_device();
    if (dev < 0) return 148;
    if (cached[dev] > 0) return cached[dev];
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) return 148;
    cached[dev] = sms;
    return sms;
}

static inline size_t align_up(size_t x) { return (x + kScratchAlign - 1) / kScratchAlign * kScratchAlign; }

// Launch plan: tensors the fused kernel takes, grouped by window shape in scan
// order (at most kMaxFused per launch), ordered by row width within a group,
// each with its strip length.
// Short launches get shorter strips so that every CTA slot sees several
// strips (the last strips of a launch otherwise leave SMs idle): the longest
// of 16, 8, 4 rows that gives at least 5 strips per CTA slot of a 4-CTA/SM
// grid.
struct LaunchGroup {
    int key;
    std::vector<int32_t> members;
    std::vector<int64_t> target;  // strip length target of each member
};

static void plan_launches(const smo_tensor *t, int32_t n, std::vector<LaunchGroup> &out) {
    out.clear();
    std::vector<char> done((size_t)n);
    for (int32_t i = 0; i < n; i++) done[i] = !fused_takes(t[i]);
    const int64_t want = 5 * 4 * (int64_t)device_sm_count();
    for (int32_t i = 0; i < n; i++) {
        if (done[i]) continue;
        LaunchGroup g;
        g.key = window_key(t[i]);
        for (int32_t k = i; k < n && (int)g.members.size() < kMaxFused; k++) {
            if (done[k] || window_key(t[k]) != g.key) continue;
            g.members.push_back(k);
            done[k] = 1;
        }
        // widest rows first: the largest strips are taken early and the
        // launch ends on the smallest ones, which shortens its tail
        std::stable_sort(g.members.begin(), g.members.end(),
                         [&](int32_t a, int32_t b) { return t[a].cols > t[b].cols; });
        int64_t rows = kStripRows;
        while (rows > 4) {
            int64_t strips = 0;
            for (int32_t k : g.members) strips += num_strips(t[k], rows);
            if (strips >= want) break;
            rows /= 2;
        }
        g.target.assign(g.members.size(), rows);
        out.push_back(std::move(g));
    }
}

// Workspace after the header: [flags: one word per strip][published rows:
// 2*w floats per strip].  Sized for the largest window-group launch of the
// set; each launch reuses the space.  The flag words sit
// in a region of their own that nothing else writes (the general path's
// scratch starts after it): a flag word may only ever hold a launch epoch,
// or a stale float could read as "strip published".
FusedLayout fused_workspace_layout(const smo_tensor *t, int32_t n) {
    std::vector<LaunchGroup> groups;
    plan_launches(t, n, groups);
    FusedLayout out{0, 0};
    for (const LaunchGroup &g : groups) {
        size_t strips = 0, halo_floats = 0;
        for (size_t m = 0; m < g.members.size(); m++) {
            const int32_t k = g.members[m];
            const int64_t s = num_strips(t[k], g.target[m]);
            strips += (size_t)s;
            halo_floats += (size_t)s * 2 * (size_t)t[k].comp_cols;
        }
        const size_t flags = align_up(strips * sizeof(unsigned int));
        const size_t body = align_up(halo_floats * sizeof(float));
        out.flag_bytes = out.flag_bytes > flags ? out.flag_bytes : flags;
        out.body_bytes = out.body_bytes > body ? out.body_bytes : body;
    }
    return out;
}

static int dispatch(int key, FusedBatch &b, int64_t max_w, size_t halo_floats, char *ws, size_t flag_bytes,
                    cudaStream_t stream) {
    switch (key >> 8) {
        case SMO_DTYPE_F32: return launch_fused_f32(key & 255, b, max_w, halo_floats, ws, flag_bytes, stream);
        case SMO_DTYPE_BF16: return launch_fused_bf16(key & 255, b, max_w, halo_floats, ws, flag_bytes, stream);
        case SMO_DTYPE_F16: return launch_fused_f16(key & 255, b, max_w, halo_floats, ws, flag_bytes, stream);
        default: return SMO_ERR_INVALID;
    }
}

static void fill(FusedDesc &f, const smo_tensor &t, int64_t halo_off, int64_t target_rows) {
    memset(&f, 0, sizeof(f));
    f.p = t.param;
    f.g = t.grad;
    f.mq_in = t.m_q_in; f.ms_in = t.m_s_in; f.vq_in = t.v_q_in; f.vs_in = t.v_s_in;
    f.mq_out = t.m_q_out; f.ms_out = t.m_s_out; f.vq_out = t.v_q_out; f.vs_out = t.v_s_out;
    f.m_in = t.m_in; f.v_in = t.v_in; f.m_out = t.m_out; f.v_out = t.v_out;
    f.H = t.rows; f.W = t.cols; f.band = t.interp_band;
    f.h = (int32_t)t.comp_rows; f.w = (int32_t)t.comp_cols;
    f.B = t.kind == SMO_KIND_POOLED8 ? (int32_t)t.q_block : 1;
    f.L = (int32_t)strip_rows(t, target_rows);
    f.div_B = make_fast_div((uint32_t)f.B);
    f.div_w = make_fast_div((uint32_t)f.w);
    f.halo_off = halo_off;
    f.kind = t.kind;
    f.hp = t.hp;
}

int fused_step(const smo_tensor *t, int32_t n, char *ws, size_t flag_bytes, cudaStream_t stream) {
    static thread_local FusedBatch batch;
    static thread_local std::vector<LaunchGroup> groups;
    plan_launches(t, n, groups);
    // one launch per group (window shape, at most kMaxFused tensors); the
    // groups run one after another and reuse the workspace
    for (const LaunchGroup &g : groups) {
        batch.n = 0;
        batch.strip_start[0] = 0;
        int64_t halo_off = 0, max_w = 0;
        for (size_t m = 0; m < g.members.size(); m++) {
            const int32_t k = g.members[m];
            FusedDesc &f = batch.d[batch.n];
            fill(f, t[k], halo_off, g.target[m]);
            const int64_t s = num_strips(t[k], g.target[m]);
            halo_off += s * 2 * t[k].comp_cols;
            max_w = max_w > t[k].comp_cols ? max_w : t[k].comp_cols;
            batch.strip_start[batch.n + 1] = batch.strip_start[batch.n] + s;
            batch.n++;
        }
        const int st = dispatch(g.key, batch, max_w, (size_t)halo_off, ws, flag_bytes, stream);
        if (st != SMO_OK) return st;
    }
    return SMO_OK;
}

}  // namespace smo
