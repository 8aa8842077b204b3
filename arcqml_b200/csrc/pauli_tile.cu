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
#include <cstring>
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

__global__ void __launch_bounds__(kTileThreads, 2)
    k_pauli_tile(const double2 *__restrict__ psi, double2 *__restrict__ out, uint32_t n,
                 uint64_t total_tiles, const __grid_constant__ TileArgs P,
                 double *__restrict__ partials) {
    extern __shared__ __align__(16) unsigned char sm[];
    double2 *tile = reinterpret_cast<double2 *>(sm);                        // 64 KB
    uint64_t *hioff = reinterpret_cast<uint64_t *>(sm + (16u << kTileQ));  // 256 entries
    uint4 *sg = reinterpret_cast<uint4 *>(hioff + (1u << (kTileQ - kTileLow)));
    TileMember *smem_m = reinterpret_cast<TileMember *>(sg + P.ngroups);
    __shared__ double red[kTileThreads / 32];
    const uint32_t tid = threadIdx.x;
    for (uint32_t h = tid; h < (1u << (kTileQ - kTileLow)); h += blockDim.x) {
        uint64_t off = 0;
        for (uint32_t b = 0; b < kTileQ - kTileLow; ++b)
            if ((h >> b) & 1u) off |= uint64_t(1) << P.S[kTileLow + b];
        hioff[h] = off;
    }
    for (uint32_t g = tid; g < P.ngroups; g += blockDim.x) sg[g] = P.groups[g];
    for (uint32_t m = tid; m < P.nmembers; m += blockDim.x) smem_m[m] = P.members[m];
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
        const uint64_t Tn = T + gridDim.x;
        if (Tn < total_tiles) {  // the next tile into L2 while this one is computed
            const uint64_t nb = tile_base(Tn);
            for (uint32_t r = tid; r < 512u; r += blockDim.x) {
                const double2 *p = psi + nb + hioff[r >> 1] + (r & 1u) * 8u;
                asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
                if (rd) {
                    const double2 *q = out + nb + hioff[r >> 1] + (r & 1u) * 8u;
                    asm volatile("prefetch.global.L2 [%0];" ::"l"(q));
                }
            }
        }
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
            const uint4 G = sg[gi];                                                        \
            add_group<H, false>(acc, tile, ptid ^ G.x,                                     \
                                member_weight(smem_m[G.y], base, tid).x);                  \
        }                                                                                  \
        _Pragma("unroll 1")                                                                \
        for (uint32_t gi = P.hbeg[2 * H + 1]; gi < P.hbeg[2 * H + 2]; ++gi) {              \
            const uint4 G = sg[gi];                                                        \
            add_group<H, true>(acc, tile, ptid ^ G.x,                                      \
                               member_weight(smem_m[G.y], base, tid).y);                   \
        }
        ARCQML_H16(ARCQML_LOOP)
#undef ARCQML_LOOP
        for (uint32_t gi = P.hbeg[32]; gi < P.ngroups; ++gi) {
            const uint4 G = sg[gi];
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
                        const TileMember &m = smem_m[mi];
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

struct TilePass {
    uint8_t S[16] = {};
    std::vector<uint32_t> groups;  // indices into obs.groups
};

// Covers the observable's groups with tile layouts; false when a flip mask has more than eight
// qubits above qubit 3 (no 12-qubit tile holds it).
bool cover(const Observable &obs, uint32_t n, std::vector<TilePass> &passes) {
    const uint64_t low = (uint64_t(1) << kTileLow) - 1;
    std::vector<uint32_t> todo;
    int diag = -1;
    for (uint32_t g = 0; g < obs.groups.size(); ++g) {
        const uint64_t f = obs.groups[g].flip;
        if (f == 0) {
            diag = int(g);
            continue;
        }
        if (__builtin_popcountll(f & ~low) > int(kTileQ - kTileLow)) return false;
        todo.push_back(g);
    }
    passes.clear();
    while (!todo.empty() || (passes.empty() && diag >= 0)) {
        uint64_t cand = low;
        // eight more qubits, each the one that completes the most remaining flip masks (ties:
        // the one most of their qubits share)
        for (uint32_t pick = 0; pick < kTileQ - kTileLow; ++pick) {
            int best = -1;
            uint64_t best_score = 0;
            for (uint32_t q = kTileLow; q < n; ++q) {
                if ((cand >> q) & 1u) continue;
                const uint64_t c2 = cand | (uint64_t(1) << q);
                uint64_t done = 0, touch = 0;
                for (uint32_t g : todo) {
                    const uint64_t f = obs.groups[g].flip;
                    if ((f & ~c2) == 0) ++done;
                    touch += uint64_t(__builtin_popcountll(f & c2));
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
        TilePass p;
        std::vector<uint32_t> rest;
        for (uint32_t g : todo)
            ((obs.groups[g].flip & ~cand) == 0 ? p.groups : rest).push_back(g);
        if (p.groups.empty() && !todo.empty()) {
            // greedy found no complete mask: take the first one's qubits, fill up in order
            cand = low | obs.groups[todo[0]].flip;
            for (uint32_t q = kTileLow; q < n && __builtin_popcountll(cand) < int(kTileQ); ++q)
                cand |= uint64_t(1) << q;
            rest.clear();
            for (uint32_t g : todo)
                ((obs.groups[g].flip & ~cand) == 0 ? p.groups : rest).push_back(g);
        }
        // n >= 20: the greedy always adds eight qubits, the fill-up completes the forced case
        if (__builtin_popcountll(cand) != int(kTileQ)) fail("internal: observable tile size");
        uint32_t k = 0;
        for (uint32_t q = 0; q < n; ++q)
            if ((cand >> q) & 1u) p.S[k++] = uint8_t(q);
        if (passes.empty() && diag >= 0) p.groups.insert(p.groups.begin(), uint32_t(diag));
        passes.push_back(std::move(p));
        todo.swap(rest);
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

}  // namespace

uint32_t observable_tile_passes(const Observable &obs, uint32_t n) {
    std::vector<TilePass> passes;
    if (n < kTileMinQubits || n > 63 || !cover(obs, n, passes)) return 0;
    return uint32_t(passes.size());
}

// <psi|H|psi> of one state (value into *value_host) and, when out is non-null, H psi written
// to out (or added to it with accumulate). Returns false (nothing launched) when the state is
// too small or a flip mask fits no tile; the caller then uses k_pauli.
bool observable_tiled(const Observable &obs, const double2 *psi, double2 *out, uint32_t n,
                      double *value_host, bool accumulate, ThreadContext &ctx, cudaStream_t s) {
    if (n < kTileMinQubits || n > 63) return false;
    std::vector<TilePass> passes;
    // an observable without terms takes no pass: the gather kernel writes its zero H psi
    if (!cover(obs, n, passes) || passes.empty()) return false;
    // device tables: per pass its groups then its members, 16-byte aligned
    std::vector<size_t> goff(passes.size()), moff(passes.size());
    std::vector<uint32_t> nmem(passes.size());
    size_t total = 0;
    for (size_t p = 0; p < passes.size(); ++p) {
        uint32_t m = 0;
        for (uint32_t g : passes[p].groups) m += obs.groups[g].count;
        if (m > kTileMaxMembers) return false;
        nmem[p] = m;
        goff[p] = total;
        total += passes[p].groups.size() * sizeof(uint4);
        moff[p] = total;
        total += size_t(m) * sizeof(TileMember);
    }
    std::vector<double2> blob((total + 15) / 16 + 1);
    char *hb = reinterpret_cast<char *>(blob.data());
    std::vector<std::vector<uint32_t>> hbeg(passes.size());
    for (size_t p = 0; p < passes.size(); ++p) {
        const uint8_t *S = passes[p].S;
        uint4 *gs = reinterpret_cast<uint4 *>(hb + goff[p]);
        TileMember *ms = reinterpret_cast<TileMember *>(hb + moff[p]);
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
        hbeg[p].assign(33, uint32_t(order.size()));
        for (uint32_t i = order.size(); i-- > 0;) hbeg[p][key(order[i])] = i;
        for (uint32_t h = 32; h-- > 0;) hbeg[p][h] = std::min(hbeg[p][h], hbeg[p][h + 1]);
        uint32_t mi = 0;
        for (size_t oi = 0; oi < order.size(); ++oi) {
            const size_t gi = oi;
            const PauliGroup &grp = obs.groups[passes[p].groups[order[oi]]];
            gs[gi] = make_uint4(host_phys(compress(grp.flip, S)), mi, mi + grp.count, 0u);
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
    std::vector<const std::vector<double2> *> refs{&blob};
    const char *dev = reinterpret_cast<const char *>(upload_tables(refs, ctx, s)[0]);

    static int sms = 0;
    if (sms == 0) {
        int d = 0;
        check_cuda(cudaGetDevice(&d), "cudaGetDevice");
        check_cuda(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, d),
                   "cudaDeviceGetAttribute");
    }
    size_t max_smem = 0;
    for (size_t p = 0; p < passes.size(); ++p)
        max_smem = std::max(max_smem, (16u << kTileQ) + (8u << (kTileQ - kTileLow)) +
                                          passes[p].groups.size() * sizeof(uint4) +
                                          size_t(nmem[p]) * sizeof(TileMember));
    check_cuda(cudaFuncSetAttribute(k_pauli_tile, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    int(max_smem)),
               "cudaFuncSetAttribute");
    int per_sm = 0;
    check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_pauli_tile,
                                                             int(kTileThreads), max_smem),
               "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
    const uint64_t total_tiles = uint64_t(1) << (n - kTileQ);
    const uint32_t grid = uint32_t(std::min<uint64_t>(total_tiles, uint64_t(sms) * std::max(per_sm, 1)));
    double *partials = ctx_partials(ctx, passes.size() * size_t(grid));
    for (size_t p = 0; p < passes.size(); ++p) {
        TileArgs a;
        std::memset(&a, 0, sizeof(a));
        std::memcpy(a.S, passes[p].S, 16);
        a.groups = reinterpret_cast<const uint4 *>(dev + goff[p]);
        a.members = reinterpret_cast<const TileMember *>(dev + moff[p]);
        a.ngroups = uint32_t(passes[p].groups.size());
        a.nmembers = nmem[p];
        a.read_out = (out && (p > 0 || accumulate)) ? 1u : 0u;
        a.ev_sub = (out && p == 0 && accumulate) ? 1u : 0u;
        a.ev_add = (!out || p + 1 == passes.size()) ? 1u : 0u;
        for (uint32_t h = 0; h < 33; ++h) a.hbeg[h] = hbeg[p][h];
        const size_t smem = (16u << kTileQ) + (8u << (kTileQ - kTileLow)) +
                            a.ngroups * sizeof(uint4) + size_t(a.nmembers) * sizeof(TileMember);
        // algorithmic traffic of the pass: psi read, H psi written (and read back after pass 0)
        const double per_amp = 16.0 + (out ? (a.read_out ? 32.0 : 16.0) : 0.0);
        const ProfToken tok = prof_begin(PROF_PAULI, s);
        prof_count_launch();
        k_pauli_tile<<<grid, kTileThreads, smem, s>>>(psi, out, n, total_tiles, a,
                                                      partials + p * size_t(grid));
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
