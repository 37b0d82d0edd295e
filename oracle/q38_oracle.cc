// CPU restatement of the reference token sampler, with the extensions the
// B200 engine adds.
//
// TEST INFRASTRUCTURE ONLY: the parity checker.  Only tests/, the smoke()
// check in __graft_entry__.py and the cpu_baseline leg of bench.py load it.
// The product (libq38s.so) never links, loads or calls this file.
//
// Parity pin: with tie_mode = 1 ("libstdc++ order") prepare_row() performs
// the same float/double operations in the same order as
// src/sampling.cc:59-146 of the reference and calls the same std::nth_element
// / std::sort with a value-only comparator, so it returns the reference's
// token bit for bit (checked against the compiled reference in
// tests/test_oracle.py and against tests/golden/*.json).  tie_mode = 0
// ("canonical") orders candidates by (value desc, index asc); that is the
// order the GPU engine implements.  The two modes differ only in which of
// several equal-valued candidates sits at a given sorted position.
//
// Extensions (no reference code exists; parity for them is unpinned except
// for the reductions noted):
//   * fp32 logits (dtype 2): identical to the bf16 path after the load.
//   * min_p: after top-k, candidates with weight w_i < min_p are dropped,
//     where w_i = exp((double)(v_i - v_0)) is the reference's own weight
//     (sampling.cc:112-113), i.e. p_i < min_p * p_max.  min_p = 0 keeps every
//     candidate, so it reduces exactly to the reference.
//   * speculative verification (mtp_verify): Leviathan et al. 2023 /
//     Chen et al. 2023 rejection sampling over the reference transform.
//   * vocab shards (shard_topk): local top-K of a contiguous column range,
//     global token ids, canonical order.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <thread>
#include <unordered_map>
#include <utility>
#include <vector>

namespace {

constexpr std::uint64_t kGamma = UINT64_C(0x9e3779b97f4a7c15);
// Domain separator for the acceptance uniform of speculative verification.
constexpr std::uint64_t kAcceptDomain = UINT64_C(0xd6e8feb86659fd93);

// sampling.cc:15-20
float bf16_to_float(std::uint16_t value) {
    const std::uint32_t bits = static_cast<std::uint32_t>(value) << 16u;
    float result;
    std::memcpy(&result, &bits, sizeof(result));
    return result;
}

// sampling.cc:22-27
std::uint64_t splitmix64(std::uint64_t state) {
    auto v = state;
    v = (v ^ (v >> 30u)) * UINT64_C(0xbf58476d1ce4e5b9);
    v = (v ^ (v >> 27u)) * UINT64_C(0x94d049bb133111eb);
    return v ^ (v >> 31u);
}

// sampling.cc:33-36
double uniform01(std::uint64_t state) {
    return static_cast<double>(splitmix64(state) >> 11u) *
           (1.0 / 9007199254740992.0);
}

}  // namespace

extern "C" {

struct q38o_row_params {
    std::uint32_t top_k;
    float top_p;
    float min_p;
    float temperature;
    float repetition_penalty;
    float frequency_penalty;
    float presence_penalty;
    std::uint32_t reserved;
    std::uint64_t rng_state;  // SamplerStateV1::rng_state before the draw
};
static_assert(sizeof(q38o_row_params) == 40, "oracle params layout");

struct q38o_result {
    std::int32_t token;
    std::int32_t status;  // 0 ok, 1 invalid_argument, 2 logic, 3 runtime
    std::uint64_t rng_before;
    std::uint64_t rng_after;
    std::uint32_t n_candidates;  // after top-k and min-p
    std::uint32_t n_retained;    // after top-p
    double total_all;            // sum of weights over the candidates
    double total;                // sum over the retained prefix
    double draw;                 // uniform01(rng_after) * total
    std::uint32_t selected;      // sorted position of the token
    std::uint32_t reserved;
};

}  // extern "C"

namespace {

struct Cand {
    float v;
    std::int32_t t;
};

int validate(std::uint32_t vocab, const q38o_row_params& p) {
    // sampling.cc:43-55 plus the min_p range of the extension.
    if (vocab == 0) return 1;
    if (!(p.temperature > 0.0f) || !std::isfinite(p.temperature) ||
        !(p.top_p > 0.0f) || p.top_p > 1.0f || !std::isfinite(p.top_p) ||
        p.top_k > vocab || p.repetition_penalty < 1.0f ||
        !std::isfinite(p.repetition_penalty) ||
        !std::isfinite(p.frequency_penalty) ||
        !std::isfinite(p.presence_penalty) || !(p.min_p >= 0.0f) ||
        p.min_p > 1.0f)
        return 1;
    return 0;
}

// Stage A of sampling.cc:67-93: penalties and temperature, one candidate per
// token in token order.  `col_begin` shifts token ids for a vocab shard.
int build_candidates(std::uint32_t n, std::uint32_t col_begin,
                     std::uint32_t vocab, const q38o_row_params& p, int dtype,
                     const void* logits, const std::uint32_t* counts,
                     const std::int32_t* extra, std::size_t n_extra,
                     std::vector<Cand>* out) {
    std::unordered_map<std::int32_t, std::uint32_t> additional;
    for (std::size_t i = 0; i < n_extra; ++i) {
        const auto token = extra[i];
        if (token < 0 || static_cast<std::uint32_t>(token) >= vocab) return 1;
        ++additional[token];
    }
    out->clear();
    out->reserve(n);
    for (std::uint32_t j = 0; j < n; ++j) {
        const std::uint32_t token = col_begin + j;
        float logit = dtype == 2
                          ? static_cast<const float*>(logits)[j]
                          : bf16_to_float(static_cast<const std::uint16_t*>(logits)[j]);
        if (!std::isfinite(logit)) logit = -std::numeric_limits<float>::infinity();
        const auto ex = additional.find(static_cast<std::int32_t>(token));
        const std::uint64_t count =
            (counts ? counts[j] : 0u) + (ex == additional.end() ? 0u : ex->second);
        if (count != 0) {
            if (p.repetition_penalty != 1.0f)
                logit = logit > 0.0f ? logit / p.repetition_penalty
                                     : logit * p.repetition_penalty;
            logit -= p.presence_penalty;
            logit -= p.frequency_penalty * static_cast<float>(count);
        }
        out->push_back(Cand{logit / p.temperature, static_cast<std::int32_t>(token)});
    }
    return 0;
}

// Stage B of sampling.cc:94-104 in either tie order.
void select_sort(std::vector<Cand>* c, std::uint32_t top_k, int tie_mode) {
    if (tie_mode == 1) {
        const auto by_value = [](const Cand& a, const Cand& b) { return a.v > b.v; };
        if (top_k != 0 && top_k < c->size()) {
            std::nth_element(c->begin(), c->begin() + top_k, c->end(), by_value);
            c->resize(top_k);
        }
        std::sort(c->begin(), c->end(), by_value);
    } else {
        const auto canon = [](const Cand& a, const Cand& b) {
            return a.v > b.v || (a.v == b.v && a.t < b.t);
        };
        if (top_k != 0 && top_k < c->size()) {
            std::nth_element(c->begin(), c->begin() + top_k, c->end(), canon);
            c->resize(top_k);
        }
        std::sort(c->begin(), c->end(), canon);
    }
}

// Stages C-E of sampling.cc:105-145 (min-p inserted after the weights).
// Fills `res` and returns the status.  `w` receives the weights.
int finish(const std::vector<Cand>& c0, const q38o_row_params& p,
           std::vector<Cand>* kept, std::vector<double>* w, q38o_result* res) {
    res->rng_before = p.rng_state;
    res->rng_after = p.rng_state + kGamma;
    if (c0.empty() || !std::isfinite(c0.front().v)) return 3;
    const float maximum = c0.front().v;
    std::size_t n = c0.size();
    w->assign(n, 0.0);
    for (std::size_t i = 0; i < n; ++i)
        (*w)[i] = std::exp(static_cast<double>(c0[i].v - maximum));
    if (p.min_p > 0.0f) {
        const double floor_w = static_cast<double>(p.min_p);
        std::size_t m = 0;
        while (m < n && (*w)[m] >= floor_w) ++m;
        n = m;
        w->resize(n);
    }
    kept->assign(c0.begin(), c0.begin() + static_cast<std::ptrdiff_t>(n));
    double total = 0.0;
    for (std::size_t i = 0; i < n; ++i) total += (*w)[i];
    res->total_all = total;
    res->n_candidates = static_cast<std::uint32_t>(n);
    if (!(total > 0.0) || !std::isfinite(total)) return 3;
    std::size_t retained = n;
    if (p.top_p < 1.0f) {
        double cumulative = 0.0;
        retained = 0;
        while (retained < n) {
            cumulative += (*w)[retained] / total;
            ++retained;
            if (cumulative >= p.top_p) break;
        }
        total = 0.0;
        for (std::size_t i = 0; i < retained; ++i) total += (*w)[i];
    }
    res->n_retained = static_cast<std::uint32_t>(retained);
    res->total = total;
    const double draw = uniform01(res->rng_after) * total;
    res->draw = draw;
    double cumulative = 0.0;
    std::size_t selected = retained - 1;
    for (std::size_t i = 0; i < retained; ++i) {
        cumulative += (*w)[i];
        if (draw < cumulative) {
            selected = i;
            break;
        }
    }
    res->selected = static_cast<std::uint32_t>(selected);
    res->token = (*kept)[selected].t;
    return 0;
}

int prepare_impl(std::uint32_t vocab, const q38o_row_params& p, int dtype,
                 const void* logits, const std::uint32_t* counts,
                 const std::int32_t* extra, std::size_t n_extra, int tie_mode,
                 q38o_result* res, std::vector<Cand>* kept,
                 std::vector<double>* w) {
    std::memset(res, 0, sizeof(*res));
    res->token = -1;
    int st = validate(vocab, p);
    if (st == 0 && dtype != 1 && dtype != 2) st = 1;
    std::vector<Cand> c;
    if (st == 0)
        st = build_candidates(vocab, 0, vocab, p, dtype, logits, counts, extra,
                              n_extra, &c);
    if (st == 0) {
        select_sort(&c, p.top_k, tie_mode);
        st = finish(c, p, kept, w, res);
    }
    res->status = st;
    if (st != 0) res->token = -1;
    return st;
}

void copy_out(const std::vector<Cand>& kept, const std::vector<double>& w,
              std::int32_t* ct, float* cv, double* cw, std::uint32_t cap) {
    const std::size_t m = std::min<std::size_t>(cap, kept.size());
    for (std::size_t i = 0; i < m; ++i) {
        if (ct) ct[i] = kept[i].t;
        if (cv) cv[i] = kept[i].v;
        if (cw) cw[i] = w[i];
    }
}

// A row's full distribution after top-k, min-p and top-p: the retained
// tokens in sorted order with probability w_i / total.
struct Dist {
    std::vector<std::int32_t> tok;
    std::vector<double> prob;
    std::vector<double> w;
    double total = 0.0;
    int status = 0;
};

Dist distribution(std::uint32_t vocab, const q38o_row_params& p, int dtype,
                  const void* logits, const std::uint32_t* counts,
                  const std::int32_t* extra, std::size_t n_extra, int tie_mode) {
    Dist d;
    q38o_result r;
    std::vector<Cand> kept;
    std::vector<double> w;
    d.status = prepare_impl(vocab, p, dtype, logits, counts, extra, n_extra,
                            tie_mode, &r, &kept, &w);
    if (d.status != 0) return d;
    d.total = r.total;
    for (std::uint32_t i = 0; i < r.n_retained; ++i) {
        d.tok.push_back(kept[i].t);
        d.w.push_back(w[i]);
        d.prob.push_back(w[i] / r.total);
    }
    return d;
}

}  // namespace

extern "C" {

// One sampling decision for one row (sampling.cc:59-146 plus extensions).
// `counts` is the per-token committed history count array (may be null),
// `extra` the additional penalty tokens of this call.  The sorted candidate
// list after top-k and min-p is copied into (cand_tokens, cand_values,
// cand_weights), up to `cap` entries (any pointer may be null).
int q38o_prepare_row(std::uint32_t vocab, const q38o_row_params* p, int dtype,
                     const void* logits, const std::uint32_t* counts,
                     const std::int32_t* extra, std::size_t n_extra,
                     int tie_mode, q38o_result* res, std::int32_t* cand_tokens,
                     float* cand_values, double* cand_weights,
                     std::uint32_t cap) {
    std::vector<Cand> kept;
    std::vector<double> w;
    const int st = prepare_impl(vocab, *p, dtype, logits, counts, extra, n_extra,
                                tie_mode, res, &kept, &w);
    if (st == 0) copy_out(kept, w, cand_tokens, cand_values, cand_weights, cap);
    return st;
}

// Many independent rows (row r: params[r], logits row r, counts row r or
// none), spread over `threads` threads.  Used for large parity sweeps and as
// the "port" CPU baseline.  Only tokens and statuses are returned.
void q38o_prepare_rows(std::uint32_t vocab, std::uint32_t rows,
                       const q38o_row_params* params, int dtype,
                       const void* logits, std::size_t row_stride_elems,
                       const std::uint32_t* const* counts, int tie_mode,
                       std::int32_t* tokens, std::int32_t* status,
                       int threads) {
    if (threads < 1) threads = 1;
    const std::size_t esize = dtype == 2 ? 4 : 2;
    auto work = [&](std::uint32_t b, std::uint32_t e) {
        std::vector<Cand> kept;
        std::vector<double> w;
        for (std::uint32_t r = b; r < e; ++r) {
            q38o_result res;
            const auto* row = static_cast<const char*>(logits) +
                              static_cast<std::size_t>(r) * row_stride_elems * esize;
            status[r] = prepare_impl(vocab, params[r], dtype, row,
                                     counts ? counts[r] : nullptr, nullptr, 0,
                                     tie_mode, &res, &kept, &w);
            tokens[r] = res.token;
        }
    };
    std::vector<std::thread> pool;
    const std::uint32_t per = (rows + threads - 1) / threads;
    for (int t = 0; t < threads; ++t) {
        const std::uint32_t b = t * per;
        const std::uint32_t e = std::min(rows, b + per);
        if (b >= e) break;
        pool.emplace_back(work, b, e);
    }
    for (auto& th : pool) th.join();
}

// Local top-K of one vocab shard: columns [col_begin, col_begin + n) of a
// row whose full vocabulary is `vocab`.  Penalties use counts (indexed by
// shard column) and temperature exactly as stage A; candidates are ordered
// canonically and carry global token ids.  Writes min(K, n) entries.
int q38o_shard_topk(std::uint32_t vocab, std::uint32_t col_begin,
                    std::uint32_t n, const q38o_row_params* p, int dtype,
                    const void* logits, const std::uint32_t* counts,
                    std::uint32_t K, float* values, std::int32_t* tokens) {
    if (validate(vocab, *p) != 0 || col_begin + n > vocab) return 1;
    std::vector<Cand> c;
    build_candidates(n, col_begin, vocab, *p, dtype, logits, counts, nullptr, 0, &c);
    select_sort(&c, K < n ? K : 0, 0);
    for (std::uint32_t i = 0; i < std::min<std::uint32_t>(K, n); ++i) {
        values[i] = c[i].v;
        tokens[i] = c[i].t;
    }
    return 0;
}

// Speculative verification of `n_draft` draft tokens against n_draft + 1
// target rows (row n_draft is the bonus row).  Row i of both target and
// draft is transformed by the same parameters with draft_tokens[0..i) added
// as extra penalty tokens, giving retained distributions p_i and q_i.
// Uniforms: state_i = rng_state + (i + 1) * gamma; acceptance of draft i uses
// uniform01(state_i ^ kAcceptDomain) and accepts iff u * q_i(d) < p_i(d);
// the residual / bonus draw uses uniform01(state_i), which is the reference
// draw of that position.  On rejection at row i the token is drawn from
// max(0, p_i - q_i) over p_i's sorted support (sequential sums, first
// cumulative above the draw); if that residual is empty the row falls back
// to the reference draw from p_i.  Writes the published tokens (accepted
// drafts then one sampled token), their count and the RNG state after the
// last published sample (rng_state + published * gamma).
int q38o_mtp_verify(std::uint32_t vocab, std::uint32_t n_draft,
                    const q38o_row_params* p, int dtype, const void* target,
                    const void* draft, const std::int32_t* draft_tokens,
                    const std::uint32_t* counts, int tie_mode,
                    std::int32_t* out_tokens, std::uint32_t* n_out,
                    std::uint32_t* n_accepted, std::uint64_t* rng_after) {
    const std::size_t esize = dtype == 2 ? 4 : 2;
    *n_out = 0;
    *n_accepted = 0;
    *rng_after = p->rng_state;
    for (std::uint32_t i = 0; i < n_draft; ++i)
        if (draft_tokens[i] < 0 || static_cast<std::uint32_t>(draft_tokens[i]) >= vocab)
            return 1;
    for (std::uint32_t i = 0; i <= n_draft; ++i) {
        const auto* trow = static_cast<const char*>(target) + i * vocab * esize;
        const Dist pd = distribution(vocab, *p, dtype, trow, counts, draft_tokens,
                                     i, tie_mode);
        if (pd.status != 0) return pd.status;
        const std::uint64_t state = p->rng_state + (static_cast<std::uint64_t>(i) + 1) * kGamma;
        if (i == n_draft) {  // bonus row: reference draw from p
            const double draw = uniform01(state) * pd.total;
            double cum = 0.0;
            std::size_t sel = pd.w.size() - 1;
            for (std::size_t j = 0; j < pd.w.size(); ++j) {
                cum += pd.w[j];
                if (draw < cum) { sel = j; break; }
            }
            out_tokens[(*n_out)++] = pd.tok[sel];
            *rng_after = state;
            return 0;
        }
        const auto* drow = static_cast<const char*>(draft) + i * vocab * esize;
        const Dist qd = distribution(vocab, *p, dtype, drow, counts, draft_tokens,
                                     i, tie_mode);
        if (qd.status != 0) return qd.status;
        const std::int32_t d = draft_tokens[i];
        double pp = 0.0, qq = 0.0;
        for (std::size_t j = 0; j < pd.tok.size(); ++j) if (pd.tok[j] == d) pp = pd.prob[j];
        for (std::size_t j = 0; j < qd.tok.size(); ++j) if (qd.tok[j] == d) qq = qd.prob[j];
        const double ua = uniform01(state ^ kAcceptDomain);
        if (ua * qq < pp) {
            out_tokens[(*n_out)++] = d;
            ++*n_accepted;
            continue;
        }
        // Rejected: draw from the residual max(0, p - q) in p's order.
        std::vector<double> res(pd.tok.size());
        double rtotal = 0.0;
        for (std::size_t j = 0; j < pd.tok.size(); ++j) {
            double qj = 0.0;
            for (std::size_t m = 0; m < qd.tok.size(); ++m)
                if (qd.tok[m] == pd.tok[j]) qj = qd.prob[m];
            res[j] = std::max(0.0, pd.prob[j] - qj);
            rtotal += res[j];
        }
        const bool residual = rtotal > 0.0;
        const std::vector<double>& ww = residual ? res : pd.w;
        const double tot = residual ? rtotal : pd.total;
        const double draw = uniform01(state) * tot;
        double cum = 0.0;
        std::size_t sel = ww.size() - 1;
        for (std::size_t j = 0; j < ww.size(); ++j) {
            cum += ww[j];
            if (draw < cum) { sel = j; break; }
        }
        out_tokens[(*n_out)++] = pd.tok[sel];
        *rng_after = state;
        return 0;
    }
    return 0;
}

// splitmix64 (sampling.cc:22-27), exposed so tests can check the RNG
// stream and the penalty checksum without the reference build.
std::uint64_t q38o_splitmix64(std::uint64_t x) { return splitmix64(x); }
double q38o_uniform01(std::uint64_t x) { return uniform01(x); }

}  // extern "C"
