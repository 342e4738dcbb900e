// moe_planner.h -- which expert copy goes on the copy engine next, for
// just-in-time expert streaming (the reference's moe_planner,
// patches/0010-team-and-streaming.patch:760-900; its interface is kept so
// that the reference's own unit test, cpp/test-moe-planner.cpp, runs against
// this implementation).
//
// A job is one expert (gate, up and down slices, `bytes` in all) that layer
// `target` wants before `deadline_ns`.  Jobs are sent earliest deadline first
// in chunks of at most chunk_bytes, so that an urgent job waits at most one
// chunk behind a less urgent one.  A job that can no longer finish before its
// deadline at the copy engine's rate is dropped instead of sent late; so are
// the unfinished jobs of a layer that has already read its table ("posted").
// Host-side bookkeeping only: no CUDA, no locks, one thread.
#pragma once

#include <cstddef>
#include <cstdint>
#include <vector>

class moe_planner {
public:
    enum drop_reason { DROP_NONE = 0, DROP_LATE, DROP_POSTED };

    struct job {
        int target = 0;
        int32_t expert = 0;
        size_t bytes = 0;
        size_t sent = 0;            // bytes handed out in chunks so far
        uint64_t deadline_ns = 0;
        bool dropped = false;
        drop_reason drop = DROP_NONE;
    };

    struct chunk {
        int job = -1;
        size_t offset = 0;
        size_t len = 0;
        bool last = false;          // the job's final chunk (its table word follows it)
    };

    explicit moe_planner(size_t chunk_bytes) : chunk_(chunk_bytes ? chunk_bytes : 1) {}

    // Token boundary: no jobs, no posted layers.
    void reset() {
        jobs_.clear();
        posted_.clear();
    }

    // A new job's id, or -1: when the target has posted already, or when
    // (target, expert) has a job (then an earlier deadline replaces its own,
    // unless it was dropped).
    int offer(int target, int32_t expert, size_t bytes, uint64_t deadline_ns) {
        if (has_posted(target)) return -1;
        for (job &j : jobs_) {
            if (j.target != target || j.expert != expert) continue;
            if (!j.dropped && deadline_ns < j.deadline_ns) j.deadline_ns = deadline_ns;
            ++n_dup;
            return -1;
        }
        job j;
        j.target = target;
        j.expert = expert;
        j.bytes = bytes;
        j.deadline_ns = deadline_ns;
        jobs_.push_back(j);
        ++n_offered;
        return (int)jobs_.size() - 1;
    }

    // Layer `target` has read its table: what is still unsent for it is dropped.
    void posted(int target) {
        posted_.push_back(target);
        for (job &j : jobs_) {
            if (j.target == target && !j.dropped && j.sent < j.bytes) {
                j.dropped = true;
                j.drop = DROP_POSTED;
                ++n_drop_posted;
            }
        }
    }

    // The next chunk, earliest deadline first, or false when nothing can go
    // now.  free_at_ns: when the copy engine finishes what it already holds;
    // bytes_per_ns: its rate.  Every open job that could no longer land in
    // time from free_at_ns is dropped on the way.  hold_after >= 0 keeps jobs
    // for layers past it waiting (not dropped).
    bool next(uint64_t free_at_ns, double bytes_per_ns, int hold_after, chunk &out) {
        int pick = -1;
        for (int i = 0; i < (int)jobs_.size(); ++i) {
            job &j = jobs_[i];
            if (j.dropped || j.sent >= j.bytes) continue;
            const double rest_ns = (double)(j.bytes - j.sent) / bytes_per_ns;
            if (free_at_ns + (uint64_t)rest_ns > j.deadline_ns) {
                j.dropped = true;
                j.drop = DROP_LATE;
                ++n_drop_late;
                continue;
            }
            if (hold_after >= 0 && j.target > hold_after) continue;
            if (pick < 0 || j.deadline_ns < jobs_[pick].deadline_ns) pick = i;
        }
        if (pick < 0) return false;
        job &j = jobs_[pick];
        const size_t rest = j.bytes - j.sent;
        out.job = pick;
        out.offset = j.sent;
        out.len = rest < chunk_ ? rest : chunk_;
        out.last = out.len == rest;
        j.sent += out.len;
        return true;
    }

    const job &get(int id) const { return jobs_[id]; }
    size_t size() const { return jobs_.size(); }

    uint64_t n_offered = 0, n_dup = 0, n_drop_late = 0, n_drop_posted = 0;

private:
    bool has_posted(int target) const {
        for (int l : posted_)
            if (l == target) return true;
        return false;
    }

    size_t chunk_;
    std::vector<job> jobs_;
    std::vector<int> posted_;
};
