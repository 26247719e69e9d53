// session.cpp - host-side KV bookkeeping of a streaming session, the part of
// Qwen3VL::ask_session that decides which cache rows survive a turn
// (src/models/qwen3vl/qwen3vl_model.cpp:1066-1202):
//
//   * window rule (qwen3vl_model.cpp:1110-1124, same as MageVL::session_evict,
//     mage_model.cpp:1827-1841): while more than max_frames frames are retained
//     and more than one completed turn exists, drop the oldest turn (its frames,
//     text and answer); then trim single frames from the front;
//   * instead of the reference's full re-prefill of the shortened window
//     (generate(..., resume=false) -> kv.clear(), :972-976), the evicted rows
//     are removed in place by sv_kv_compact (the moss_vl kv_shift_rows
//     mechanism, moss_vl_model.cpp:264-291) and the new turn is appended after
//     the surviving rows, which keep their original positions (the caller's
//     rope positions are unchanged, as moss_vl's sess_rdelta does);
//   * the splice predicate (qwen3vl_model.cpp:1165-1171);
//   * the row-budget eviction of MossVL's streaming session (session_compact_self,
//     moss_vl_model.cpp:273-292): before n new rows are written into a full cache, the oldest rows
//     after the pinned sink prefix leave in 128-row quanta, never reaching into the newest 256
//     rows, the survivors move down in place (sv_kv_compact) and the eviction count accumulates
//     into the rope-position shift (the reference's sess_rdelta), so every surviving row keeps
//     its original position.
#include <algorithm>
#include <cstdio>
#include <vector>

#include "internal.hpp"

struct sv_session {
    struct Turn {
        int start = 0;        // first cache row of the turn
        int frames = 0;       // frames still held by the turn
        int text_rows = 0;
        int answer_rows = 0;
        int rows(int rpf) const { return frames * rpf + text_rows + answer_rows; }
    };
    sv_kv* kv = nullptr;
    int max_frames = 64;
    int rows_per_frame = 1;
    int sink_rows = 0;
    std::vector<Turn> turns;           // completed turns, oldest first
    std::vector<int64_t> row_ids;      // original id of every live cache row
    int64_t next_id = 0;
    int n_marks = 0;                   // retained frames incl. the open turn's
    bool open = false;
    int open_frames = 0;
    int64_t rope_shift = 0;            // rows evicted by sv_session_make_room since the last reset
};

namespace {

void reset_rows(sv_session* s) {
    s->turns.clear();
    s->row_ids.clear();
    for (int i = 0; i < s->sink_rows; i++) s->row_ids.push_back(i);
    s->next_id = s->sink_rows;
    s->n_marks = 0;
    s->open = false;
    s->open_frames = 0;
    s->rope_shift = 0;
}

// MossVL's session_compact_self constants (moss_vl_model.cpp:278, 281)
constexpr int kRecentFloor = 256;   // the newest rows are never evicted
constexpr int kEvictQuantum = 128;  // evictions are rounded up to whole quanta

}  // namespace

extern "C" {

int sv_can_splice(const int32_t* cached, int64_t kv_len, int64_t n_past, const int32_t* ids, int64_t n_ids,
                  int64_t* skip) {
    if (skip) *skip = 0;
    if (!(kv_len > 0 && n_ids > kv_len && kv_len == n_past)) return 0;
    if (!cached || !ids) return 0;
    if (!std::equal(cached, cached + kv_len, ids)) return 0;
    if (skip) *skip = kv_len;
    return 1;
}

int sv_session_create(sv_kv* kv, int max_frames, int rows_per_frame, int sink_rows, sv_session** out) {
    if (!out || max_frames < 1 || rows_per_frame < 1 || sink_rows < 0 || (kv && sink_rows > kv->n_ctx))
        return SV_ERR_INVALID;
    sv_session* s = new sv_session();
    s->kv = kv;
    s->max_frames = max_frames;
    s->rows_per_frame = rows_per_frame;
    s->sink_rows = sink_rows;
    reset_rows(s);
    *out = s;
    return SV_OK;
}

int sv_session_destroy(sv_session* s) {
    if (!s) return SV_ERR_INVALID;
    delete s;
    return SV_OK;
}

int sv_session_reset(sv_session* s) {
    if (!s) return SV_ERR_INVALID;
    reset_rows(s);
    return SV_OK;
}

int sv_session_begin_turn(sv_session* s, int n_new_frames, int* first_row, int* kept_new_frames, void* stream) {
    if (!s || n_new_frames < 0 || s->open) return SV_ERR_INVALID;
    const int rpf = s->rows_per_frame;
    // the frame count is worked out in a local and written back only once the compaction succeeded,
    // so a failed call leaves the session as it was
    int n_marks = s->n_marks + n_new_frames;
    int new_kept = n_new_frames;

    // ---- the window rule on the turn table
    const int n_before = (int)s->row_ids.size();
    std::vector<sv_segment> segs;
    if (s->sink_rows > 0) segs.push_back({0, s->sink_rows, 1});
    size_t drop_turns = 0;
    while (n_marks > s->max_frames && s->turns.size() - drop_turns > 1) {
        const sv_session::Turn& t = s->turns[drop_turns];
        n_marks -= t.frames;
        segs.push_back({t.start, t.rows(rpf), 0});
        drop_turns++;
    }
    int trim = 0;   // frames trimmed from the (new) front turn
    while (n_marks > s->max_frames) {
        n_marks--;
        if (drop_turns < s->turns.size() && s->turns[drop_turns].frames - trim > 0) trim++;
        else if (new_kept > 0) new_kept--;
    }
    bool changed = drop_turns > 0 || trim > 0;
    if (changed) {
        for (size_t i = drop_turns; i < s->turns.size(); i++) {
            const sv_session::Turn& t = s->turns[i];
            if (i == drop_turns && trim > 0) {
                segs.push_back({t.start, trim * rpf, 0});
                segs.push_back({t.start + trim * rpf, t.rows(rpf) - trim * rpf, 1});
            } else {
                segs.push_back({t.start, t.rows(rpf), 1});
            }
        }
        int new_len = 0;
        for (const sv_segment& g : segs) new_len += g.keep ? g.n_rows : 0;
        if (s->kv) {   // a host-only session (kv == NULL) plans rows without a cache
            const int rc = sv_kv_compact(s->kv, segs.data(), (int)segs.size(), 0, &new_len, stream);
            if (rc != SV_OK) return rc;
        }
        // host bookkeeping follows the same segments
        std::vector<int64_t> ids;
        ids.reserve(new_len);
        for (const sv_segment& g : segs)
            if (g.keep)
                for (int r = 0; r < g.n_rows; r++) ids.push_back(s->row_ids[g.src + r]);
        s->row_ids.swap(ids);
        s->turns.erase(s->turns.begin(), s->turns.begin() + drop_turns);
        if (!s->turns.empty() && trim > 0) s->turns.front().frames -= trim;
        int row = s->sink_rows;
        for (sv_session::Turn& t : s->turns) {
            t.start = row;
            row += t.rows(rpf);
        }
        fprintf(stderr, "session: evicted %d rows (%zu turns, %d frames), %d live\n", n_before - new_len,
                drop_turns, trim, new_len);
    }
    s->n_marks = n_marks;
    s->open = true;
    s->open_frames = new_kept;
    if (first_row) *first_row = (int)s->row_ids.size();
    if (kept_new_frames) *kept_new_frames = new_kept;
    return SV_OK;
}

int sv_session_end_turn(sv_session* s, int frames, int text_rows, int answer_rows) {
    if (!s || !s->open || frames < 0 || text_rows < 0 || answer_rows < 0) return SV_ERR_INVALID;
    sv_session::Turn t;
    t.start = (int)s->row_ids.size();
    t.frames = frames;
    t.text_rows = text_rows;
    t.answer_rows = answer_rows;
    const int rows = t.rows(s->rows_per_frame);
    if (s->kv && t.start + rows > s->kv->n_ctx) return SV_ERR_OVERFLOW;
    // frames the window dropped from the open turn were never written
    s->n_marks -= s->open_frames - std::min(frames, s->open_frames);
    for (int r = 0; r < rows; r++) s->row_ids.push_back(s->next_id++);
    s->turns.push_back(t);
    s->open = false;
    return SV_OK;
}

int sv_session_make_room(sv_session* s, int need, int capacity, int* evicted, int64_t* rope_shift, void* stream) {
    if (evicted) *evicted = 0;
    if (!s || need < 0 || capacity < 0 || s->open || !s->turns.empty()) return SV_ERR_INVALID;
    const int cap = capacity > 0 ? capacity : (s->kv ? s->kv->n_ctx : 0);
    if (cap <= 0 || (s->kv && cap > s->kv->n_ctx)) return SV_ERR_INVALID;
    const int n_past = (int)s->row_ids.size();
    if (rope_shift) *rope_shift = s->rope_shift;
    if (n_past + need <= cap) return SV_OK;
    const int needed_free = n_past + need - cap;
    const int evictable = n_past - s->sink_rows - kRecentFloor;
    if (evictable < needed_free) return SV_ERR_OVERFLOW;
    const int evict = std::min(evictable, (needed_free + kEvictQuantum - 1) / kEvictQuantum * kEvictQuantum);
    const int tail = n_past - s->sink_rows - evict;
    if (s->kv) {
        const sv_segment segs[3] = {{0, s->sink_rows, 1}, {s->sink_rows, evict, 0}, {s->sink_rows + evict, tail, 1}};
        int new_len = 0;
        const int rc = sv_kv_compact(s->kv, segs, 3, 0, &new_len, stream);
        if (rc != SV_OK) return rc;
    }
    s->row_ids.erase(s->row_ids.begin() + s->sink_rows, s->row_ids.begin() + s->sink_rows + evict);
    s->rope_shift += evict;
    if (evicted) *evicted = evict;
    if (rope_shift) *rope_shift = s->rope_shift;
    fprintf(stderr, "session: evicted %d rows (sink %d, live %d)\n", evict, s->sink_rows, n_past - evict);
    return SV_OK;
}

int sv_session_push_rows(sv_session* s, int n) {
    if (!s || n < 0 || s->open || !s->turns.empty()) return SV_ERR_INVALID;
    if (s->kv && (int64_t)s->row_ids.size() + n > s->kv->n_ctx) return SV_ERR_OVERFLOW;
    for (int r = 0; r < n; r++) s->row_ids.push_back(s->next_id++);
    return SV_OK;
}

int sv_session_rows(const sv_session* s, int* n_rows, int64_t* rows_out, int max_rows) {
    if (!s || !n_rows) return SV_ERR_INVALID;
    *n_rows = (int)s->row_ids.size();
    if (rows_out)
        for (int i = 0; i < std::min(max_rows, *n_rows); i++) rows_out[i] = s->row_ids[i];
    return SV_OK;
}

}  // extern "C"
