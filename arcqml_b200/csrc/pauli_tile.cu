// pauli_tile.cu — <psi|H|psi> and H|psi> for large states as a few passes over 12-qubit tiles.
//
// crates/arcqml-observable/src/compiled_hamiltonian.rs:104-132 defines
//   (H psi)[t] = sum over terms c * phase(t ^ f) * psi[t ^ f],
//   phase(s)   = i^(y mod 4) * (-1)^popc(s & z),
// with f the term's flip (X/Y) mask and z its phase (Y/Z) mask. A term whose flip bits all lie in
// a tile's qubits pairs amplitudes inside that tile. The host covers the observable's distinct
// flip masks with tile layouts (qubits 0-3, for 256-byte runs, plus eight more chosen greedily),
// and each layout becomes one pass: every CTA loads a tile of psi into shared memory, adds
// w * (-1)^popc(t & z) * psi[t ^ f] over the pass's
// groups for each of its amplitudes t, and writes (or adds to) H psi. Passes after the first
// read H psi back, so one evaluation moves 32 + 48 (passes - 1) bytes per amplitude instead of
// gathering psi once per distinct flip mask. The last pass, which holds the whole H psi, sums
// Re(conj(psi_t) (H psi)_t) = <psi|H|psi>; without an output every pass sums its own
// contribution.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <vector>

#include "launch.h"
#include "profile.h"
#include "rt_internal.h"

namespace arcqml {

namespace {

constexpr uint32_t kTileQ = 12;            // tile qubits
constexpr uint32_t kTileLow = 4;           // qubits 0-3 are always tile qubits
constexpr uint32_t kTileThreads = 256;     // 16 amplitudes per thread
constexpr uint32_t kTileMinQubits = 20;    // below this the state sits in L2 and k_pauli wins
constexpr uint32_t kTileMaxMembers = 4096; // terms per pass (shared-memory table)

struct TileMember {  // one term of a group, 32 bytes
    double2 w;       // coefficient * i^(y mod 4) * (-1)^popc(flip & z)
    uint64_t z;      // phase mask (global qubits)
    uint32_t zl;     // phase mask on the tile-local bits 0-7 (the thread-index bits)
    uint32_t h;      // phase mask on the tile-local bits 8-11 (the element bits), 0-15
};
static_assert(sizeof(TileMember) == 32, "TileMember layout");

struct TileArgs {
    uint8_t S[16];                  // tile qubits S[0..12), ascending, S[0..4) = 0..3
    const uint4 *groups;            // per group: {phys(local flip), first member, end member, 0}
    const TileMember *members;
    uint32_t ngroups, nmembers;
    uint32_t read_out;              // add to the H psi already in `out`
    // expectation terms of this pass: ev_sub subtracts <psi|out before the pass> (the first pass
    // that adds to an existing H psi), ev_add adds <psi|out after the pass> (every pass without
    // an output, else the last one: its H psi is the whole sum)
    uint32_t ev_sub, ev_add;
    // single-term groups come first, ordered by key 2 h + (weight imaginary), h their element
    // phase pattern: those of key k are [hbeg[k], hbeg[k + 1]); groups of several terms are
    // [hbeg[32], ngroups)
    uint32_t hbeg[33];
};

// A pass's group and term tables as a by-value kernel parameter (constant-bank reads, uniform
// over the warp), for passes small enough; larger ones are copied into shared memory.
constexpr uint32_t kInlineGroups = 128, kInlineMembers = 512;
struct TileTables {
    uint4 g[kInlineGroups];
    TileMember m[kInlineMembers];
};
struct NoTileTables {
    uint32_t unused;
};

__device__ __forceinline__ uint32_t tphys(uint32_t j) {
    return j ^ (((j >> 3) ^ (j >> 6) ^ (j >> 9)) & 7u);
}
__device__ __forceinline__ double2 tcfma(double2 a, double2 b, double2 c) {
    return make_double2(fma(a.x, b.x, fma(-a.y, b.y, c.x)), fma(a.x, b.y, fma(a.y, b.x, c.y)));
}
__device__ __forceinline__ uint32_t parity64(uint64_t x) { return uint32_t(__popcll(x) & 1); }
__host__ __device__ constexpr uint32_t cparity(uint32_t x) { return x ? (x & 1u) ^ cparity(x >> 1) : 0u; }
__device__ __forceinline__ double2 tneg(double2 a) { return make_double2(-a.x, -a.y); }

// The sign (-1)^popc(t & z) of a member for this thread's element i of the tile at `base`:
// (-1)^s0 * (-1)^parity(i & h), s0 from the tile base and the thread's own index bits.
__device__ __forceinline__ double2 member_weight(const TileMember &m, uint64_t base, uint32_t tid) {
    const uint32_t s0 = parity64(base & m.z) ^ (uint32_t(__popc(tid & m.zl)) & 1u);
    return s0 ? tneg(m.w) : m.w;
}

__device__ __forceinline__ void cp_async16t(void *smem, const void *gmem) {
    const unsigned a = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(a), "l"(gmem) : "memory");
}

// acc[i] += (-1)^parity(i & H) * w * psi[partner of element i] for the weight w of one term,
// real (IM false: w = (c, 0)) or imaginary (IM: w = (0, c)), so two FMAs per element: the
// element signs are constants of the code (one instantiation per phase pattern H on the element
// bits and kind of weight).
template <uint32_t H, bool IM>
__device__ __forceinline__ void add_group(double2 (&acc)[16], const double2 *tile, uint32_t x,
                                          double c) {
    const double cn = -c;
#pragma unroll
    for (uint32_t i = 0; i < 16; ++i) {
        const double s = cparity(i & H) ? cn : c;
        const double2 p = tile[x ^ tphys(i << 8)];
        if (IM) {
            acc[i].x = fma(-s, p.y, acc[i].x);
            acc[i].y = fma(s, p.x, acc[i].y);
        } else {
            acc[i].x = fma(s, p.x, acc[i].x);
            acc[i].y = fma(s, p.y, acc[i].y);
        }
    }
}

// wi[i] += (-1)^parity((i0 + i) & H) * w for elements i0..i0+7 (a group of several terms)
template <uint32_t H, uint32_t I0>
__device__ __forceinline__ void add_weight(double2 (&wi)[8], double2 w) {
#pragma unroll
    for (uint32_t i = 0; i < 8; ++i) {
        const bool neg = cparity((I0 + i) & H);
        wi[i] = make_double2(neg ? wi[i].x - w.x : wi[i].x + w.x,
                             neg ? wi[i].y - w.y : wi[i].y + w.y);
    }
}

#define ARCQML_H16(M) M(0) M(1) M(2) M(3) M(4) M(5) M(6) M(7) M(8) M(9) M(10) M(11) M(12) \
    M(13) M(14) M(15)

template <bool INL, class TT>
__global__ void __launch_bounds__(kTileThreads, 2)
    k_pauli_tile(const double2 *__restrict__ psi, double2 *__restrict__ out, uint32_t n,
                 uint64_t total_tiles, const __grid_constant__ TileArgs P,
                 const __grid_constant__ TT T, double *__restrict__ partials) {
    extern __shared__ __align__(16) unsigned char sm[];
    double2 *tile = reinterpret_cast<double2 *>(sm);                        // 64 KB
    uint64_t *hioff = reinterpret_cast<uint64_t *>(sm + (16u << kTileQ));  // 256 entries
    uint4 *sg = reinterpret_cast<uint4 *>(hioff + (1u << (kTileQ - kTileLow)));
    TileMember *smem_m = reinterpret_cast<TileMember *>(sg + P.ngroups);
    auto grp = [&](uint32_t gi) -> uint4 {
        if constexpr (INL) return T.g[gi];
        else return sg[gi];
    };
    auto mem = [&](uint32_t mi) -> const TileMember & {
        if constexpr (INL) return T.m[mi];
        else return smem_m[mi];
    };
    __shared__ double red[kTileThreads / 32];
    const uint32_t tid = threadIdx.x;
    for (uint32_t h = tid; h < (1u << (kTileQ - kTileLow)); h += blockDim.x) {
        uint64_t off = 0;
        for (uint32_t b = 0; b < kTileQ - kTileLow; ++b)
            if ((h >> b) & 1u) off |= uint64_t(1) << P.S[kTileLow + b];
        hioff[h] = off;
    }
    if constexpr (!INL) {
        for (uint32_t g = tid; g < P.ngroups; g += blockDim.x) sg[g] = P.groups[g];
        for (uint32_t m = tid; m < P.nmembers; m += blockDim.x) smem_m[m] = P.members[m];
    }
    __syncthreads();

    const uint32_t ptid = tphys(tid);
    const uint64_t tmask = (uint64_t(1) << (n - kTileQ)) - 1;
    auto tile_base = [&](uint64_t T) {
        uint64_t g = T & tmask;
        for (uint32_t b = 0; b < kTileQ; ++b) {
            const uint32_t p = P.S[b];
            g = ((g >> p) << (p + 1)) | (g & ((uint64_t(1) << p) - 1));
        }
        return g;
    };
    // element i of this thread: tile index j = tid | i << 8, state offset base + off(i)
    auto elem_off = [&](uint32_t i) { return uint64_t(tid & 15u) | hioff[(tid >> 4) | (i << 4)]; };
    const bool rd = P.read_out && out;

    double ev = 0.0;
    for (uint64_t T = blockIdx.x; T < total_tiles; T += gridDim.x) {
        const uint64_t base = tile_base(T);
        // psi's tile straight into shared memory; meanwhile this thread's H psi so far
#pragma unroll
        for (uint32_t i = 0; i < 16; ++i)
            cp_async16t(tile + (ptid ^ tphys(i << 8)), psi + base + elem_off(i));
        asm volatile("cp.async.commit_group;\n" ::: "memory");
        double2 acc[16];
#pragma unroll
        for (uint32_t i = 0; i < 16; ++i)
            acc[i] = rd ? out[base + elem_off(i)] : make_double2(0.0, 0.0);
        asm volatile("cp.async.wait_group 0;\n" ::: "memory");
        __syncthreads();
        if (P.ev_sub) {
#pragma unroll
            for (uint32_t i = 0; i < 16; ++i) {
                const double2 pi = tile[ptid ^ tphys(i << 8)];
                ev -= fma(pi.x, acc[i].x, pi.y * acc[i].y);
            }
        }
        // single-term groups: one loop per element phase pattern, its signs in the code
#define ARCQML_LOOP(H)                                                                     \
        _Pragma("unroll 1")                                                                \
        for (uint32_t gi = P.hbeg[2 * H]; gi < P.hbeg[2 * H + 1]; ++gi) {                  \
            const uint4 G = grp(gi);                                                       \
            add_group<H, false>(acc, tile, ptid ^ G.x,                                     \
                                member_weight(mem(G.y), base, tid).x);                     \
        }                                                                                  \
        _Pragma("unroll 1")                                                                \
        for (uint32_t gi = P.hbeg[2 * H + 1]; gi < P.hbeg[2 * H + 2]; ++gi) {              \
            const uint4 G = grp(gi);                                                       \
            add_group<H, true>(acc, tile, ptid ^ G.x,                                      \
                               member_weight(mem(G.y), base, tid).y);                      \
        }
        ARCQML_H16(ARCQML_LOOP)
#undef ARCQML_LOOP
        for (uint32_t gi = P.hbeg[32]; gi < P.ngroups; ++gi) {
            const uint4 G = grp(gi);
            const uint32_t x = ptid ^ G.x;
            {
                // several terms share the flip mask: per element the sum of their signed
                // weights, in two halves of eight elements (registers)
#pragma unroll
                for (uint32_t half = 0; half < 2; ++half) {
                    double2 wi[8];
#pragma unroll
                    for (uint32_t i = 0; i < 8; ++i) wi[i] = make_double2(0.0, 0.0);
                    for (uint32_t mi = G.y; mi < G.z; ++mi) {
                        const TileMember &m = mem(mi);
                        const double2 w = member_weight(m, base, tid);
                        if (half == 0) {
                            switch (m.h) {
#define ARCQML_CASE(H) \
                            case H: add_weight<H, 0>(wi, w); break;
                                ARCQML_H16(ARCQML_CASE)
#undef ARCQML_CASE
                            default: break;
                            }
                        } else {
                            switch (m.h) {
#define ARCQML_CASE(H) \
                            case H: add_weight<H, 8>(wi, w); break;
                                ARCQML_H16(ARCQML_CASE)
#undef ARCQML_CASE
                            default: break;
                            }
                        }
                    }
#pragma unroll
                    for (uint32_t i = 0; i < 8; ++i) {
                        const uint32_t e = half * 8 + i;
                        acc[e] = tcfma(wi[i], tile[x ^ tphys(e << 8)], acc[e]);
                    }
                }
            }
        }
        if (P.ev_add) {
#pragma unroll
            for (uint32_t i = 0; i < 16; ++i) {
                const double2 pi = tile[ptid ^ tphys(i << 8)];
                ev += fma(pi.x, acc[i].x, pi.y * acc[i].y);
            }
        }
        if (out) {
#pragma unroll
            for (uint32_t i = 0; i < 16; ++i) out[base + elem_off(i)] = acc[i];
        }
        __syncthreads();  // the tile is overwritten by the next iteration
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ev += __shfl_xor_sync(0xffffffffu, ev, o);
    if ((tid & 31u) == 0) red[tid >> 5] = ev;
    __syncthreads();
    if (tid == 0) {
        double s = 0.0;
        for (uint32_t w = 0; w < blockDim.x / 32u; ++w) s += red[w];
        partials[blockIdx.x] = s;
    }
}

// ---------------------------------------------------------------- host: tile cover

uint32_t host_phys(uint32_t j) { return j ^ (((j >> 3) ^ (j >> 6) ^ (j >> 9)) & 7u); }

// bit b of the result = bit S[b] of x
uint32_t compress(uint64_t x, const uint8_t *S) {
    uint32_t r = 0;
    for (uint32_t b = 0; b < kTileQ; ++b)
        if ((x >> S[b]) & 1u) r |= 1u << b;
    return r;
}

int popc64(uint64_t x) { return __builtin_popcountll(x); }

struct TilePass {
    uint8_t S[16] = {};
    std::vector<uint32_t> groups;  // indices into obs.groups
};

// Adds `picks` qubits to cand, each the one that completes the most of the masks in todo (ties:
// the one most of their qubits share; then the lowest).
void grow_by_qubits(const std::vector<uint64_t> &todo, uint32_t n, uint32_t picks,
                    uint64_t &cand) {
    for (uint32_t pick = 0; pick < picks; ++pick) {
        int best = -1;
        uint64_t best_score = 0;
        for (uint32_t q = kTileLow; q < n; ++q) {
            if ((cand >> q) & 1u) continue;
            const uint64_t c2 = cand | (uint64_t(1) << q);
            uint64_t done = 0, touch = 0;
            for (uint64_t f : todo) {
                if ((f & ~c2) == 0) ++done;
                touch += uint64_t(popc64(f & c2));
            }
            const uint64_t score = done * 4096 + touch;
            if (best < 0 || score > best_score) {
                best = int(q);
                best_score = score;
            }
        }
        if (best < 0) break;
        cand |= uint64_t(1) << best;
    }
}

// The qubits above the low four of one pass, chosen by masks: a widest remaining mask, then
// repeatedly the mask that completes the most remaining masks per qubit it adds (ties: the
// narrower union) while the union fits in `room` qubits. Among the widest masks `rule` picks
// the first (0) or last (1) in order, or the one sharing the most (2) or fewest (3) qubits
// with the others.
uint64_t pick_by_masks(const std::vector<uint64_t> &todo, uint32_t room, int rule) {
    int width = -1;
    for (uint64_t h : todo) width = std::max(width, popc64(h));
    uint64_t U = 0;
    bool have = false;
    uint64_t best_overlap = 0;
    for (uint64_t h : todo) {
        if (popc64(h) != width) continue;
        uint64_t overlap = 0;
        if (rule >= 2)
            for (uint64_t g : todo) overlap += uint64_t(popc64(h & g));
        const bool better = !have || rule == 1 || (rule == 2 && overlap > best_overlap) ||
                            (rule == 3 && overlap < best_overlap);
        if (better) {
            U = h;
            best_overlap = overlap;
            have = true;
        }
    }
    for (;;) {
        uint32_t inside = 0;
        for (uint64_t h : todo) inside += (h & ~U) == 0 ? 1u : 0u;
        bool found = false;
        double best_key = 0.0;
        int best_width = 0;
        uint64_t best = 0;
        for (uint64_t h : todo) {
            if ((h & ~U) == 0) continue;
            const uint64_t nu = U | h;
            const int wn = popc64(nu);
            if (wn > int(room)) continue;
            uint32_t in2 = 0;
            for (uint64_t g : todo) in2 += (g & ~nu) == 0 ? 1u : 0u;
            const double key = double(in2 - inside) / double(wn - popc64(U));
            if (!found || key > best_key || (key == best_key && wn < best_width)) {
                found = true;
                best_key = key;
                best_width = wn;
                best = h;
            }
        }
        if (!found) break;
        U |= best;
    }
    return U;
}

// Tile sets (12 qubits each, the low four included) covering every flip mask in `highs` (the
// distinct flip masks without their low four bits), by qubits (rule < 0) or by masks with the
// given seed rule.
std::vector<uint64_t> cover_sets(const std::vector<uint64_t> &highs, uint32_t n, int rule) {
    const uint64_t low = (uint64_t(1) << kTileLow) - 1;
    const uint32_t room = kTileQ - kTileLow;
    std::vector<uint64_t> todo = highs, sets;
    while (!todo.empty()) {
        uint64_t cand = low | (rule >= 0 ? pick_by_masks(todo, room, rule) : 0);
        grow_by_qubits(todo, n, kTileQ - uint32_t(popc64(cand)), cand);
        bool any = false;
        for (uint64_t h : todo) any = any || (h & ~cand) == 0;
        if (!any) {
            // the qubit greedy completed no mask: take the first one's qubits, fill up in order
            cand = low | todo[0];
            for (uint32_t q = kTileLow; q < n && popc64(cand) < int(kTileQ); ++q)
                cand |= uint64_t(1) << q;
        }
        // n >= 20: both ways reach 12 qubits
        if (popc64(cand) != int(kTileQ)) fail("internal: observable tile size");
        std::vector<uint64_t> rest;
        for (uint64_t h : todo)
            if (h & ~cand) rest.push_back(h);
        todo.swap(rest);
        sets.push_back(cand);
    }
    return sets;
}

// Covers the observable's groups with tile layouts: the fewest passes of the greedy by qubits
// and the greedy by masks with each seed rule (by masks only up to 256 distinct masks: its cost
// grows with their cube); false when a flip mask has more than eight qubits above qubit 3 (no
// 12-qubit tile holds it).
bool cover(const Observable &obs, uint32_t n, std::vector<TilePass> &passes) {
    const uint64_t low = (uint64_t(1) << kTileLow) - 1;
    std::vector<uint64_t> highs;
    int diag = -1;
    for (uint32_t g = 0; g < obs.groups.size(); ++g) {
        const uint64_t f = obs.groups[g].flip;
        if (f == 0) {
            diag = int(g);
            continue;
        }
        if (popc64(f & ~low) > int(kTileQ - kTileLow)) return false;
        highs.push_back(f & ~low);
    }
    std::sort(highs.begin(), highs.end());
    highs.erase(std::unique(highs.begin(), highs.end()), highs.end());
    std::vector<uint64_t> sets = cover_sets(highs, n, -1);
    for (int rule = 0; rule < 4 && highs.size() <= 256; ++rule) {
        std::vector<uint64_t> by_masks = cover_sets(highs, n, rule);
        if (by_masks.size() < sets.size()) sets.swap(by_masks);
    }
    if (sets.empty() && diag >= 0) {  // only the diagonal group: one pass over the low qubits
        uint64_t cand = low;
        grow_by_qubits({}, n, kTileQ - kTileLow, cand);
        sets.push_back(cand);
    }
    passes.assign(sets.size(), TilePass{});
    std::vector<char> taken(obs.groups.size(), 0);
    for (size_t p = 0; p < sets.size(); ++p) {
        uint32_t k = 0;
        for (uint32_t q = 0; q < n; ++q)
            if ((sets[p] >> q) & 1u) passes[p].S[k++] = uint8_t(q);
        if (p == 0 && diag >= 0) {
            passes[p].groups.push_back(uint32_t(diag));
            taken[size_t(diag)] = 1;
        }
        for (uint32_t g = 0; g < obs.groups.size(); ++g)
            if (!taken[g] && (obs.groups[g].flip & ~sets[p]) == 0) {
                passes[p].groups.push_back(g);
                taken[g] = 1;
            }
    }
    return true;
}

double2 term_weight(const Observable &obs, uint64_t flip, uint32_t k) {
    const double c = (__builtin_popcountll(flip & obs.zmask[k]) & 1) ? -obs.coef[k] : obs.coef[k];
    switch (obs.ymod4[k] & 3u) {
    case 0: return make_double2(c, 0.0);
    case 1: return make_double2(0.0, c);
    case 2: return make_double2(-c, 0.0);
    default: return make_double2(0.0, -c);
    }
}

// Everything host-side of an observable's tile passes for one state size: the cover and the
// per-pass group and term tables (one blob, 16-byte aligned parts), built once per observable
// and size. ok == false: the gather kernel evaluates the observable.
struct TilePlan {
    bool ok = false;
    std::vector<TilePass> passes;
    std::vector<size_t> goff, moff;      // byte offsets of each pass's groups and members
    std::vector<uint32_t> nmem;          // members per pass
    std::vector<std::vector<uint32_t>> hbeg;
    std::vector<double2> blob;
    size_t max_smem = 0;
};

size_t tile_smem(size_t ngroups, size_t nmembers) {
    return (16u << kTileQ) + (8u << (kTileQ - kTileLow)) + ngroups * sizeof(uint4) +
           nmembers * sizeof(TileMember);
}

std::shared_ptr<const TilePlan> build_tile_plan(const Observable &obs, uint32_t n) {
    auto tp = std::make_shared<TilePlan>();
    // an observable without terms takes no pass: the gather kernel writes its zero H psi
    if (n < kTileMinQubits || n > 63 || !cover(obs, n, tp->passes) || tp->passes.empty())
        return tp;
    const std::vector<TilePass> &passes = tp->passes;
    const size_t np = passes.size();
    tp->goff.resize(np);
    tp->moff.resize(np);
    tp->nmem.resize(np);
    tp->hbeg.resize(np);
    size_t total = 0;
    for (size_t p = 0; p < np; ++p) {
        uint32_t m = 0;
        for (uint32_t g : passes[p].groups) m += obs.groups[g].count;
        if (m > kTileMaxMembers) return std::make_shared<TilePlan>();
        tp->nmem[p] = m;
        tp->goff[p] = total;
        total += passes[p].groups.size() * sizeof(uint4);
        tp->moff[p] = total;
        total += size_t(m) * sizeof(TileMember);
        tp->max_smem = std::max(tp->max_smem, tile_smem(passes[p].groups.size(), m));
    }
    tp->blob.assign((total + 15) / 16 + 1, make_double2(0.0, 0.0));
    char *hb = reinterpret_cast<char *>(tp->blob.data());
    for (size_t p = 0; p < np; ++p) {
        const uint8_t *S = passes[p].S;
        uint4 *gs = reinterpret_cast<uint4 *>(hb + tp->goff[p]);
        TileMember *ms = reinterpret_cast<TileMember *>(hb + tp->moff[p]);
        // order: single-term groups by the element phase pattern of their term and whether its
        // weight i^y c is imaginary, then the others
        std::vector<uint32_t> order(passes[p].groups.size());
        for (uint32_t gi = 0; gi < order.size(); ++gi) order[gi] = gi;
        auto key = [&](uint32_t gi) {
            const PauliGroup &grp = obs.groups[passes[p].groups[gi]];
            if (grp.count != 1) return 32u;
            const uint32_t k = grp.first;
            return 2u * (compress(obs.zmask[k], S) >> 8) + (obs.ymod4[k] & 1u);
        };
        std::stable_sort(order.begin(), order.end(),
                         [&](uint32_t a, uint32_t b) { return key(a) < key(b); });
        std::vector<uint32_t> &hbeg = tp->hbeg[p];
        hbeg.assign(33, uint32_t(order.size()));
        for (uint32_t i = order.size(); i-- > 0;) hbeg[key(order[i])] = i;
        for (uint32_t h = 32; h-- > 0;) hbeg[h] = std::min(hbeg[h], hbeg[h + 1]);
        uint32_t mi = 0;
        for (size_t oi = 0; oi < order.size(); ++oi) {
            const PauliGroup &grp = obs.groups[passes[p].groups[order[oi]]];
            gs[oi] = make_uint4(host_phys(compress(grp.flip, S)), mi, mi + grp.count, 0u);
            for (uint32_t k = grp.first; k < grp.first + grp.count; ++k, ++mi) {
                TileMember &m = ms[mi];
                m.w = term_weight(obs, grp.flip, k);
                m.z = obs.zmask[k];
                const uint32_t zl = compress(obs.zmask[k], S);
                m.zl = zl & 0xffu;
                m.h = zl >> 8;
            }
        }
    }
    tp->ok = true;
    return tp;
}

// The observable's tile plan for n qubits, built on first use.
std::shared_ptr<const TilePlan> tile_plan(const Observable &obs, uint32_t n) {
    std::lock_guard<std::mutex> lock(obs.cache_mu);
    for (const auto &e : obs.tile_cache)
        if (e.first == n) return std::static_pointer_cast<const TilePlan>(e.second);
    std::shared_ptr<const TilePlan> tp = build_tile_plan(obs, n);
    obs.tile_cache.emplace_back(n, tp);
    return tp;
}

// Whether passes small enough take their tables as a kernel parameter (on unless
// ARCQML_TILE_TABLES_SMEM=1: always through shared memory).
bool tile_tables_inline() {
    static const bool on = [] {
        const char *e = std::getenv("ARCQML_TILE_TABLES_SMEM");
        return !(e && e[0] == '1');
    }();
    return on;
}

}  // namespace

uint32_t observable_tile_passes(const Observable &obs, uint32_t n) {
    const std::shared_ptr<const TilePlan> tp = tile_plan(obs, n);
    return tp->ok ? uint32_t(tp->passes.size()) : 0u;
}

// <psi|H|psi> of one state (value into *value_host) and, when out is non-null, H psi written
// to out (or added to it with accumulate). Returns false (nothing launched) when the state is
// too small or a flip mask fits no tile; the caller then uses k_pauli.
bool observable_tiled(const Observable &obs, const double2 *psi, double2 *out, uint32_t n,
                      double *value_host, bool accumulate, ThreadContext &ctx, cudaStream_t s) {
    if (n < kTileMinQubits || n > 63) return false;
    const std::shared_ptr<const TilePlan> tp = tile_plan(obs, n);
    if (!tp->ok) return false;
    const std::vector<TilePass> &passes = tp->passes;
    std::vector<const std::vector<double2> *> refs{&tp->blob};
    const char *dev = reinterpret_cast<const char *>(upload_tables(refs, ctx, s)[0]);

    int d = 0, sms = 0;
    check_cuda(cudaGetDevice(&d), "cudaGetDevice");
    check_cuda(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, d),
               "cudaDeviceGetAttribute");
    const auto k_smem = k_pauli_tile<false, NoTileTables>;
    const auto k_inl = k_pauli_tile<true, TileTables>;
    check_cuda(cudaFuncSetAttribute(k_smem, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    int(tp->max_smem)),
               "cudaFuncSetAttribute");
    check_cuda(cudaFuncSetAttribute(k_inl, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    int(tile_smem(0, 0))),
               "cudaFuncSetAttribute");
    int per_sm = 0;  // the shared-memory kernel's occupancy; the other one needs less memory
    check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_smem,
                                                             int(kTileThreads), tp->max_smem),
               "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    std::vector<TileTables> tables(1);  // the inline tables of the pass being launched
    const uint64_t total_tiles = uint64_t(1) << (n - kTileQ);
    const uint32_t grid =
        uint32_t(std::min<uint64_t>(total_tiles, uint64_t(sms) * std::max(per_sm, 1)));
    double *partials = ctx_partials(ctx, passes.size() * size_t(grid));
    for (size_t p = 0; p < passes.size(); ++p) {
        TileArgs a;
        std::memset(&a, 0, sizeof(a));
        std::memcpy(a.S, passes[p].S, 16);
        a.groups = reinterpret_cast<const uint4 *>(dev + tp->goff[p]);
        a.members = reinterpret_cast<const TileMember *>(dev + tp->moff[p]);
        a.ngroups = uint32_t(passes[p].groups.size());
        a.nmembers = tp->nmem[p];
        a.read_out = (out && (p > 0 || accumulate)) ? 1u : 0u;
        a.ev_sub = (out && p == 0 && accumulate) ? 1u : 0u;
        a.ev_add = (!out || p + 1 == passes.size()) ? 1u : 0u;
        for (uint32_t h = 0; h < 33; ++h) a.hbeg[h] = tp->hbeg[p][h];
        const bool inl = tile_tables_inline() && a.ngroups <= kInlineGroups &&
                         a.nmembers <= kInlineMembers;
        const size_t smem = inl ? tile_smem(0, 0) : tile_smem(a.ngroups, a.nmembers);
        // algorithmic traffic of the pass: psi read, H psi written (and read back after pass 0)
        const double per_amp = 16.0 + (out ? (a.read_out ? 32.0 : 16.0) : 0.0);
        const ProfToken tok = prof_begin(PROF_PAULI, s);
        prof_count_launch();
        if (inl) {
            const char *hb = reinterpret_cast<const char *>(tp->blob.data());
            std::memcpy(tables[0].g, hb + tp->goff[p], a.ngroups * sizeof(uint4));
            std::memcpy(tables[0].m, hb + tp->moff[p], a.nmembers * sizeof(TileMember));
            k_inl<<<grid, kTileThreads, smem, s>>>(psi, out, n, total_tiles, a, tables[0],
                                                   partials + p * size_t(grid));
        } else {
            k_smem<<<grid, kTileThreads, smem, s>>>(psi, out, n, total_tiles, a, NoTileTables{},
                                                    partials + p * size_t(grid));
        }
        prof_end(tok, s, per_amp * double(uint64_t(1) << n));
        check_cuda(cudaGetLastError(), "observable tile pass launch");
    }
    double *sums = ctx_dgrads(ctx, 1);
    launch_reduce_rows(partials, 1u, uint32_t(passes.size()) * grid, sums, s);
    double *h = ctx_hvals(ctx, 1);
    check_cuda(cudaMemcpyAsync(h, sums, sizeof(double), cudaMemcpyDeviceToHost, s),
               "cudaMemcpyAsync (value)");
    check_cuda(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    *value_host = h[0];
    return true;
}

}  // namespace arcqml
