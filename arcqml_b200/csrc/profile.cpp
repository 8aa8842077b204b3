// profile.cpp — optional CUDA-event timing of the runtime's own kernel launches.
//
// When enabled, each timed launch site records a start and a stop event on the stream it
// launches on; durations are resolved lazily (on read) and summed per category together with
// the launch's algorithmic HBM bytes. Every kernel launch of the runtime is also counted.
#include <mutex>
#include <vector>

#include "profile.h"
#include "rt_internal.h"

namespace arcqml {

namespace {

struct Pending {
    int cat;
    cudaEvent_t a, b;
    double bytes;
};

struct Totals {
    uint64_t launches = 0;
    double ms = 0.0;
    double bytes = 0.0;
};

std::mutex g_mu;
bool g_on = false;
std::vector<Pending> g_pending;
Totals g_tot[kProfCategories];
uint64_t g_launches = 0;

void resolve_locked() {
    for (auto &p : g_pending) {
        float ms = 0.f;
        if (cudaEventSynchronize(p.b) == cudaSuccess && cudaEventElapsedTime(&ms, p.a, p.b) == cudaSuccess) {
            g_tot[p.cat].launches += 1;
            g_tot[p.cat].ms += double(ms);
            g_tot[p.cat].bytes += p.bytes;
        }
        cudaEventDestroy(p.a);
        cudaEventDestroy(p.b);
    }
    g_pending.clear();
}

}  // namespace

void prof_count_launch() {
    std::lock_guard<std::mutex> l(g_mu);
    ++g_launches;
}

ProfToken prof_begin(int cat, cudaStream_t s) {
    ProfToken t;
    {
        std::lock_guard<std::mutex> l(g_mu);
        ++g_launches;
        if (!g_on) return t;
    }
    t.cat = cat;
    if (cudaEventCreate(&t.a) != cudaSuccess || cudaEventCreate(&t.b) != cudaSuccess) {
        t.cat = -1;
        return t;
    }
    cudaEventRecord(t.a, s);
    return t;
}

void prof_end(const ProfToken &t, cudaStream_t s, double bytes) {
    if (t.cat < 0) return;
    cudaEventRecord(t.b, s);
    std::lock_guard<std::mutex> l(g_mu);
    g_pending.push_back({t.cat, t.a, t.b, bytes});
}

void prof_enable(bool on) {
    std::lock_guard<std::mutex> l(g_mu);
    resolve_locked();
    g_on = on;
    for (auto &t : g_tot) t = Totals{};
}

void prof_read(int cat, uint64_t *launches, double *ms, double *bytes) {
    std::lock_guard<std::mutex> l(g_mu);
    resolve_locked();
    *launches = g_tot[cat].launches;
    *ms = g_tot[cat].ms;
    *bytes = g_tot[cat].bytes;
}

uint64_t prof_launch_count() {
    std::lock_guard<std::mutex> l(g_mu);
    return g_launches;
}

}  // namespace arcqml
