// C shim over the reference's own predictor (cpp/moe-predictor.{h,cpp} in
// everett6/moe-prefetch), compiled from the reference sources where they lie
// into oracle/_ref/.  TEST INFRASTRUCTURE ONLY: used to pin our Python MOEP
// reader/scorer (moe_prefetch_b200/predictor.py) against the reference's C++.
#include "moe-predictor.h"

#include <cstring>
#include <string>

extern "C" {

void *refpred_load(const char *path, char *err, int err_cap) {
    auto *p = new moe_predictor();
    std::string e;
    if (!p->load(path, e)) {
        if (err && err_cap > 0) {
            std::strncpy(err, e.c_str(), (size_t)err_cap - 1);
            err[err_cap - 1] = 0;
        }
        delete p;
        return nullptr;
    }
    return p;
}

void refpred_free(void *h) { delete static_cast<moe_predictor *>(h); }

int refpred_info(void *h, int *out) {
    auto *p = static_cast<moe_predictor *>(h);
    out[0] = (int)p->n_expert;
    out[1] = (int)p->n_layers;
    out[2] = (int)p->feat_dim;
    out[3] = (int)p->top_k;
    out[4] = p->off_prev;
    out[5] = p->off_cur;
    out[6] = p->off_below;
    out[7] = p->off_self_prev;
    out[8] = p->off_pca;
    out[9] = (int)p->layer_of.size();
    return 0;
}

int refpred_has_layer(void *h, int il) { return static_cast<moe_predictor *>(h)->has_layer(il); }

void refpred_score(void *h, int il, const int32_t *prev, int n_prev, const int32_t *cur,
                   int n_cur, const int32_t *below, int n_below, const int32_t *self_prev,
                   int n_self_prev, float *out) {
    moe_predictor::inputs in;
    in.prev = prev; in.n_prev = (size_t)n_prev;
    in.cur = cur; in.n_cur = (size_t)n_cur;
    in.below = below; in.n_below = (size_t)n_below;
    in.self_prev = self_prev; in.n_self_prev = (size_t)n_self_prev;
    static_cast<moe_predictor *>(h)->score(il, in, out);
}

int refpred_top_k(void *h, const float *scores, int k, int32_t *out) {
    return (int)static_cast<moe_predictor *>(h)->top_k_ids(scores, (size_t)k, out);
}

float refpred_update(void *h, int il, const int32_t *prev, int n_prev, const int32_t *cur,
                     int n_cur, const int32_t *below, int n_below, const int32_t *self_prev,
                     int n_self_prev, const int32_t *truth, int n_truth, float lr) {
    moe_predictor::inputs in;
    in.prev = prev; in.n_prev = (size_t)n_prev;
    in.cur = cur; in.n_cur = (size_t)n_cur;
    in.below = below; in.n_below = (size_t)n_below;
    in.self_prev = self_prev; in.n_self_prev = (size_t)n_self_prev;
    return static_cast<moe_predictor *>(h)->update(il, in, truth, (size_t)n_truth, lr);
}

int refpred_save(void *h, const char *path, char *err, int err_cap) {
    std::string e;
    const bool ok = static_cast<moe_predictor *>(h)->save(path, e);
    if (!ok && err && err_cap > 0) {
        std::strncpy(err, e.c_str(), (size_t)err_cap - 1);
        err[err_cap - 1] = 0;
    }
    return ok ? 1 : 0;
}

}  // extern "C"
