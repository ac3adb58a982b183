// IQ2_XXS / IQ2_XS / IQ2_S / IQ3_XXS / IQ3_S lattice-search kernels (sm_100a).
//
// Reference: kernels/iq2.py:418-498 (IQ2_XXS), kernels/iq2xs_common.py:280-355 with
// iq2_xs.py:20-69 / iq2_s.py:21-62, kernels/iq3_xxs.py:31-134, kernels/iq3_s.py:31-140.
//
// Mapping. One thread per quantization group (16 or 32 values, in registers) runs the
// weights, the sign handling and the accept chain over the candidate scales. The grid
// projections are where the time goes: a subgroup's tentative code is either on the
// lattice (one table lookup) or needs a best-neighbour search over a list of 1..292
// candidates. All sweep steps' codes depend only on the group maximum, so each warp
// queues the off-grid searches of a batch of steps in shared memory, counting-sorts
// them by list length, and then gives one search to each lane: the 32 lanes of a warp
// walk lists of similar length in lockstep, with no synchronisation inside the walk.
// The weighted distance of one candidate is a sum over positions of terms that depend
// only on the position and the candidate's level there, so a lane first tabulates the
// 4 x 8 (IQ2) or 8 x 4 (IQ3) terms of its search, computed exactly as the reference
// does, and then needs one table read and one add per position and candidate. The
// tables of all lanes of a CTA share one array of 256-byte rows at the start of shared
// memory, column (warp * 32 + lane): a term's address is the candidate's level bits,
// shifted into bits 8..11, OR-ed with the lane's byte column, plus a constant row.
#include <algorithm>
#include <mutex>
#include <vector>

#include "iq_grids.h"
#include "qs_kquant.cuh"
#include "qs_kernels.h"

namespace qs {

// ---------------------------------------------------------------------------
// device tables
// ---------------------------------------------------------------------------
struct IqGridDev {
    const uint16_t* kgrid;  // grid index -> code
    const uint32_t* nbr;    // code index -> 0x80000000 | code (on grid) or quad offset << 9 | quads
    const uint16_t* list;   // neighbour lists as codes, (distance, index) order, padded to whole
                            // quads with copies of the last code (a copy never wins a strict <)
    const int16_t* kmap;    // code -> grid index (-1 off the grid)
    int grid;
};

struct IqTables {
    IqGridDev g[5];
    void* mem = nullptr;              // the five codebooks
    void* gmem[5] = {};               // each grid's neighbour tables, built on first use
    bool built[5] = {};
    std::mutex mu;
};

enum { G_IQ2XXS = 0, G_IQ2XS, G_IQ2S, G_IQ3XXS, G_IQ3S };

// Neighbour lists of every reachable off-grid code (the reference's Tables classes:
// iq2.py:31-74, iq2xs_common.py:41-95, iq3_common.py:29-68). IQ2 codes are indexed in
// base 3 because sweep levels are clamped to 0..2, IQ3 codes directly (levels 0..7).
static void build_grid(const uint16_t* kgrid, int G, int bits, int npos, int nwant, std::vector<uint32_t>& nbr,
                       std::vector<uint16_t>& list, std::vector<int16_t>& kmap16) {
    const int mask = (1 << bits) - 1;
    const int kmap_size = bits == 2 ? 43692 : 4096;
    std::vector<int> kmap(kmap_size, -1);
    for (int i = 0; i < G; i++) kmap[kgrid[i]] = i;
    kmap16.assign(kmap.begin(), kmap.end());
    const int nidx = bits == 2 ? 6561 : 4096;
    nbr.assign(nidx, 0);
    std::vector<int64_t> keys;
    std::vector<int> dist(G);
    for (int idx = 0; idx < nidx; idx++) {
        int code = 0;
        if (bits == 2) {
            int t = idx;
            for (int j = 0; j < npos; j++) { code |= (t % 3) << (2 * j); t /= 3; }
        } else {
            code = idx;
        }
        if (kmap[code] >= 0) {
            nbr[idx] = 0x80000000u | (uint32_t)code;
            continue;
        }
        // squared distances to every grid point; the list is every point within the nwant
        // smallest distinct distances, in (distance, index) order: find the thresholds in
        // one pass, then sort only the selected points
        int thr[3] = {INT32_MAX, INT32_MAX, INT32_MAX};  // nwant <= 3 smallest distinct distances
        for (int i = 0; i < G; i++) {
            int d2 = 0;
            for (int j = 0; j < npos; j++) {
                int p = 2 * ((code >> (bits * j)) & mask) + 1;
                int q = 2 * ((kgrid[i] >> (bits * j)) & mask) + 1;
                d2 += (p - q) * (p - q);
            }
            dist[i] = d2;
            for (int w = 0; w < nwant; w++) {
                if (d2 == thr[w]) break;
                if (d2 < thr[w]) {
                    for (int v = nwant - 1; v > w; v--) thr[v] = thr[v - 1];
                    thr[w] = d2;
                    break;
                }
            }
        }
        int lim = thr[0];  // the largest threshold found (fewer than nwant distinct distances: all)
        for (int w = 1; w < nwant; w++)
            if (thr[w] != INT32_MAX) lim = thr[w];
        keys.clear();
        for (int i = 0; i < G; i++)
            if (dist[i] <= lim) keys.push_back((int64_t)dist[i] * 65536 + i);
        std::sort(keys.begin(), keys.end());
        const int n = (int)keys.size();
        const int nq = (n + 3) / 4;  // quads of 4 codes, one 8-byte load each
        nbr[idx] = ((uint32_t)(list.size() / 4) << 9) | (uint32_t)nq;
        for (int i = 0; i < 4 * nq; i++) list.push_back(kgrid[keys[i < n ? i : n - 1] % 65536]);
    }
}

struct GridSpec { const uint16_t* grid; int G, bits, npos, nwant; };
static const GridSpec kGrids[5] = {
    {KGRID_2BIT_256, 256, 2, 8, 2}, {KGRID_2BIT_512, 512, 2, 8, 2}, {KGRID_2BIT_1024, 1024, 2, 8, 1},
    {KGRID_3BIT_256, 256, 3, 4, 2}, {KGRID_3BIT_512, 512, 3, 4, 3}};

static int grid_of(int type) {
    switch (type) {
    case QS_IQ2_XXS: return G_IQ2XXS;
    case QS_IQ2_XS: return G_IQ2XS;
    case QS_IQ2_S: return G_IQ2S;
    case QS_IQ3_XXS: return G_IQ3XXS;
    case QS_IQ3_S: return G_IQ3S;
    default: return -1;
    }
}

// Uploads the five codebooks; the neighbour tables of a grid are built by iq_tables_ensure.
cudaError_t iq_tables_create(IqTables** out) {
    size_t total = 0;
    for (const GridSpec& sp : kGrids) total += ((size_t)sp.G * 2 + 255) & ~(size_t)255;
    char* mem = nullptr;
    cudaError_t e = cudaMalloc(&mem, total);
    if (e != cudaSuccess) return e;
    IqTables* T = new IqTables;
    T->mem = mem;
    size_t o = 0;
    for (int t = 0; t < 5; t++) {
        uint16_t* kg = reinterpret_cast<uint16_t*>(mem + o);
        o += ((size_t)kGrids[t].G * 2 + 255) & ~(size_t)255;
        if ((e = cudaMemcpy(kg, kGrids[t].grid, kGrids[t].G * 2, cudaMemcpyHostToDevice)) != cudaSuccess) {
            cudaFree(mem);
            delete T;
            return e;
        }
        T->g[t] = IqGridDev{kg, nullptr, nullptr, nullptr, kGrids[t].G};
    }
    *out = T;
    return cudaSuccess;
}

// Builds and uploads the neighbour tables of `type`'s grid once (thread-safe; the device
// must be current).
cudaError_t iq_tables_ensure(IqTables* T, int type) {
    const int t = grid_of(type);
    if (t < 0) return cudaSuccess;
    std::lock_guard<std::mutex> lk(T->mu);
    if (T->built[t]) return cudaSuccess;
    std::vector<uint32_t> nbr;
    std::vector<uint16_t> list;
    std::vector<int16_t> kmap;
    const GridSpec& sp = kGrids[t];
    build_grid(sp.grid, sp.G, sp.bits, sp.npos, sp.nwant, nbr, list, kmap);
    if (list.size() / 4 > 65535) return cudaErrorInvalidValue;  // queue entries hold 16-bit quad offsets
    auto al = [](size_t n) { return (n + 255) & ~(size_t)255; };
    const size_t total = al(nbr.size() * 4) + al(list.size() * 2 + 16) + al(kmap.size() * 2);
    char* mem = nullptr;
    cudaError_t e = cudaMalloc(&mem, total);
    if (e != cudaSuccess) return e;
    uint32_t* nb = reinterpret_cast<uint32_t*>(mem);
    uint16_t* ls = reinterpret_cast<uint16_t*>(mem + al(nbr.size() * 4));
    int16_t* km = reinterpret_cast<int16_t*>(mem + al(nbr.size() * 4) + al(list.size() * 2 + 16));
    if ((e = cudaMemcpy(nb, nbr.data(), nbr.size() * 4, cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaMemcpy(ls, list.data(), list.size() * 2, cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaMemcpy(km, kmap.data(), kmap.size() * 2, cudaMemcpyHostToDevice)) != cudaSuccess) {
        cudaFree(mem);
        return e;
    }
    T->gmem[t] = mem;
    T->g[t].nbr = nb;
    T->g[t].list = ls;
    T->g[t].kmap = km;
    T->built[t] = true;
    return cudaSuccess;
}

const uint16_t* iq_kgrid(const IqTables* t, int type) {
    switch (type) {
    case QS_IQ2_XXS: return t->g[G_IQ2XXS].kgrid;
    case QS_IQ2_XS: return t->g[G_IQ2XS].kgrid;
    case QS_IQ2_S: return t->g[G_IQ2S].kgrid;
    case QS_IQ3_XXS: return t->g[G_IQ3XXS].kgrid;
    case QS_IQ3_S: return t->g[G_IQ3S].kgrid;
    default: return nullptr;
    }
}

void iq_tables_destroy(IqTables* t) {
    if (t) {
        for (void* m : t->gmem) cudaFree(m);
        cudaFree(t->mem);
        delete t;
    }
}

// ---------------------------------------------------------------------------
// per-type constants
// ---------------------------------------------------------------------------
enum SumKind { SUM_TORCH, SUM_TREE };
enum Reproj { RP_ALL_PROJ, RP_OFFGRID_NEED, RP_OFFGRID_REDO, RP_ALL_REDO };

// ONE_SEARCH_SITE: the final reprojection runs as the last pass of the sweep loop, so the
// search code is inlined once instead of twice (smaller code; measured faster for the IQ2
// grids, slower for IQ3, where the two sites stay).
template <int T> struct IqT;
template <> struct IqT<QS_IQ2_XXS> {
    static constexpr int GS = 32, NSUB = 4, NPOS = 8, BITS = 2, NLEV = 4, MAXL = 2, NSTEP = 13, BB = 66, GID = G_IQ2XXS;
    static constexpr bool PARITY = true, ACT_GT0 = false, INIT_QP = true, ONE_SEARCH_SITE = true;
    static constexpr int SUMK = SUM_TORCH, RP = RP_ALL_PROJ;
    static constexpr float EPS = EPS15, SIGFAC = 1.0f, DMUL = 1.0f;
};
template <> struct IqT<QS_IQ2_XS> {
    static constexpr int GS = 16, NSUB = 2, NPOS = 8, BITS = 2, NLEV = 4, MAXL = 2, NSTEP = 19, BB = 74, GID = G_IQ2XS;
    static constexpr bool PARITY = true, ACT_GT0 = false, INIT_QP = false, ONE_SEARCH_SITE = true;
    static constexpr int SUMK = SUM_TREE, RP = RP_OFFGRID_NEED;
    static constexpr float EPS = EPS15, SIGFAC = 1.0f, DMUL = 1.0f;
};
template <> struct IqT<QS_IQ2_S> {
    static constexpr int GS = 16, NSUB = 2, NPOS = 8, BITS = 2, NLEV = 4, MAXL = 2, NSTEP = 19, BB = 82, GID = G_IQ2S;
    static constexpr bool PARITY = false, ACT_GT0 = false, INIT_QP = false, ONE_SEARCH_SITE = true;
    static constexpr int SUMK = SUM_TREE, RP = RP_OFFGRID_NEED;
    static constexpr float EPS = EPS8, SIGFAC = 2.0f, DMUL = 0.9875f;
};
template <> struct IqT<QS_IQ3_XXS> {
    static constexpr int GS = 32, NSUB = 8, NPOS = 4, BITS = 3, NLEV = 8, MAXL = 7, NSTEP = 31, BB = 98, GID = G_IQ3XXS;
    static constexpr bool PARITY = true, ACT_GT0 = false, INIT_QP = false, ONE_SEARCH_SITE = false;
    static constexpr int SUMK = SUM_TREE, RP = RP_OFFGRID_REDO;
    static constexpr float EPS = EPS8, SIGFAC = 2.0f, DMUL = 1.0125f;
};
template <> struct IqT<QS_IQ3_S> {
    static constexpr int GS = 32, NSUB = 8, NPOS = 4, BITS = 3, NLEV = 8, MAXL = 7, NSTEP = 19, BB = 110, GID = G_IQ3S;
    static constexpr bool PARITY = false, ACT_GT0 = true, INIT_QP = false, ONE_SEARCH_SITE = false;
    static constexpr int SUMK = SUM_TREE, RP = RP_ALL_REDO;
    static constexpr float EPS = 0.0f, SIGFAC = 2.0f, DMUL = 1.033f;
};

struct IqParams {
    float c[32];   // sweep-step numerators
    float qp[8];   // make_qp numerators (IQ2_XXS initial scale)
};

constexpr int IQ_WARPS = 2;      // warps per CTA; each warp owns 32 groups
constexpr int IQ_CAP = 256;      // queued searches per warp
constexpr int IQ_MIN_CTAS = 6;   // resident CTAs per SM the register budget is sized for (12 warps)
constexpr int IQ_FINAL = 15;     // tag slot of the final reprojection
constexpr int IQ_BINS = 74;      // list lengths in quads, 1..73 (the longest IQ2_XS list has 292 codes)
constexpr uint32_t IQ_SEARCHED = 1u << 16;  // flag beside a resolved code: it came from a search

// Rows of the CTA term table (256 bytes each: 64 columns of f32, warp * 32 + lane).
// IQ2 (16-bit codes, 2 bits per position): rows 0..15 hold t0 + t1 for the pair of
// levels (code & 15); positions 3, 5, 7 have a level stride of 4 rows and interleave
// in rows 16..30; positions 2, 4, 6 have consecutive rows from 32, 36, 40.
// IQ3 (12-bit codes, 3 bits per position): positions 3 and 1 take the even and odd rows
// 0..15 (stride 2), positions 0 and 2 rows 16..23 and 24..31.
template <int NPOS> struct IqRows;
template <> struct IqRows<8> {
    static constexpr int N = 44;
    __host__ __device__ static constexpr int row(int j, int l) {
        return j == 2 ? 32 + l : j == 3 ? 16 + 4 * l : j == 4 ? 36 + l : j == 5 ? 17 + 4 * l : j == 6 ? 40 + l : 18 + 4 * l;
    }
};
template <> struct IqRows<4> {
    static constexpr int N = 32;
    __host__ __device__ static constexpr int row(int j, int l) {
        return j == 0 ? 16 + l : j == 1 ? 1 + 2 * l : j == 2 ? 24 + l : 2 * l;
    }
};

template <class Tr>
struct IqWarpSmem {
    static constexpr int NB = IQ_CAP / (32 * Tr::NSUB);  // sweep steps per batch
    static constexpr int XS = Tr::GS + 4;  // row pitch: 16-byte rows, and 8 lanes' float4s hit 8 distinct bank quads
    static constexpr int WINS = NB * Tr::NSUB + 1;  // odd word pitch: lane-indexed accesses are conflict-free
    __align__(16) float xv[32][XS];  // search-space values of every group (|x|, parity-folded);
                                     // holds the superblock squares while the weights are computed
    __align__(16) float wv[32][XS];  // sqrt of the weights
    float psc[32][NB + 1];       // per group: search scale of each batch step, then the final scale
    uint16_t off[IQ_CAP];        // list start, in quads (every list table has fewer than 65536 quads)
    uint16_t tag[IQ_CAP];        // group | slot << 5 | subgroup << 9
    uint8_t len[IQ_CAP];         // list length, in quads
    uint8_t ord[IQ_CAP];         // searches in order of list length
    uint8_t rank[IQ_CAP];
    uint32_t hist[(IQ_BINS + 1) / 2];  // two 16-bit counters (then bin starts) per word
    uint32_t win[32][WINS];      // per step j and subgroup q, at j * NSUB + q: the resolved code
                                 // (| IQ_SEARCHED when it came from a search)
    float part[4][8];
    int nq;
};

template <class Tr>
__host__ __device__ constexpr size_t iq_tbl_bytes() { return (size_t)IqRows<Tr::NPOS>::N * 256; }

template <class Tr>
constexpr size_t iq_smem_bytes() {
    return iq_tbl_bytes<Tr>() + IQ_WARPS * sizeof(IqWarpSmem<Tr>) + 64 * 4 + IQ_WARPS * 4 * Tr::BB + 64;
}

// One distance term: constant row R plus the lane's column byte and the level bits.
template <int R>
__device__ __forceinline__ float iq_term(const unsigned char* tb, uint32_t a) {
    return *reinterpret_cast<const float*>(tb + R * 256 + a);
}

// Weighted distance of the code in the low (HI = false) or high half of w; lb is the
// lane's column byte. The terms are added in the reference's order, position 0 first.
template <int NPOS, bool HI>
__device__ __forceinline__ float iq_dist(const unsigned char* tb, uint32_t w, uint32_t lb) {
    using R = IqRows<NPOS>;
    if (NPOS == 8) {
        const uint32_t a = HI ? w >> 8 : w << 8, b = HI ? w >> 12 : w << 4, c = HI ? w >> 16 : w,
                       d = HI ? w >> 20 : w >> 4;
        float s = iq_term<0>(tb, (a & 0xF00) | lb);
        s = __fadd_rn(s, iq_term<R::row(2, 0)>(tb, (b & 0x300) | lb));
        s = __fadd_rn(s, iq_term<R::row(3, 0)>(tb, (b & 0xC00) | lb));
        s = __fadd_rn(s, iq_term<R::row(4, 0)>(tb, (c & 0x300) | lb));
        s = __fadd_rn(s, iq_term<R::row(5, 0)>(tb, (c & 0xC00) | lb));
        s = __fadd_rn(s, iq_term<R::row(6, 0)>(tb, (d & 0x300) | lb));
        s = __fadd_rn(s, iq_term<R::row(7, 0)>(tb, (d & 0xC00) | lb));
        return s;
    } else {
        const uint32_t a = HI ? w >> 8 : w << 8, b = HI ? w >> 10 : w << 6, c = HI ? w >> 14 : w << 2,
                       d = HI ? w >> 16 : w;
        float s = iq_term<R::row(0, 0)>(tb, (a & 0x700) | lb);
        s = __fadd_rn(s, iq_term<R::row(1, 0)>(tb, (b & 0xE00) | lb));
        s = __fadd_rn(s, iq_term<R::row(2, 0)>(tb, (c & 0x700) | lb));
        s = __fadd_rn(s, iq_term<R::row(3, 0)>(tb, (d & 0xE00) | lb));
        return s;
    }
}

__device__ __forceinline__ int warp_excl_scan(int v, int lane, int& total) {
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    total = __shfl_sync(0xffffffffu, x, 31);
    return x - v;
}

// Solve every queued search of this warp, one search per lane, longest lists first.
template <class Tr>
__device__ void iq_flush(IqWarpSmem<Tr>& W, const IqGridDev& G, int lane) {
    using WS = IqWarpSmem<Tr>;
    const int P = W.nq;
    // counting sort by list length, longest first
    constexpr int HW = (IQ_BINS + 1) / 2, PER = 2 * ((HW + 31) / 32);  // bins per lane (even)
    for (int i = lane; i < HW; i += 32) W.hist[i] = 0;
    __syncwarp();
    for (int i = lane; i < P; i += 32) {
        const int bin = IQ_BINS - 1 - min(IQ_BINS - 1, (int)W.len[i]);
        const int sh = 16 * (bin & 1);
        W.rank[i] = (uint8_t)((atomicAdd(&W.hist[bin >> 1], 1u << sh) >> sh) & 0xFFFF);
    }
    __syncwarp();
    {
        int cnt[PER], sum = 0;
#pragma unroll
        for (int k = 0; k < PER; k++) {
            const int b = lane * PER + k;
            cnt[k] = b < IQ_BINS ? (int)((W.hist[b >> 1] >> (16 * (b & 1))) & 0xFFFF) : 0;
            sum += cnt[k];
        }
        int tot;
        int run = warp_excl_scan(sum, lane, tot);
        __syncwarp();
#pragma unroll
        for (int k = 0; k < PER; k += 2) {
            const int b = lane * PER + k;
            if (b < IQ_BINS) W.hist[b >> 1] = (uint32_t)run | ((uint32_t)(run + cnt[k]) << 16);
            run += cnt[k] + cnt[k + 1];
        }
    }
    __syncwarp();
    for (int i = lane; i < P; i += 32) {
        const int bin = IQ_BINS - 1 - min(IQ_BINS - 1, (int)W.len[i]);
        W.ord[((W.hist[bin >> 1] >> (16 * (bin & 1))) & 0xFFFF) + W.rank[i]] = (uint8_t)i;
    }
    __syncwarp();

    extern __shared__ __align__(16) unsigned char smem[];
    const unsigned char* tb = smem;
    const uint32_t lb = (uint32_t)(threadIdx.x & (IQ_WARPS * 32 - 1)) * 4;  // this lane's column byte
    using R = IqRows<Tr::NPOS>;
    for (int pb = 0; pb < P; pb += 32) {
        const int i = pb + lane;
        if (i < P) {
            const int p = W.ord[i];
            const uint32_t off = W.off[p];
            const int n = W.len[p];
            const int tg = W.tag[p], g = tg & 31, slot = (tg >> 5) & 15, q = tg >> 9;
            const float sc = W.psc[g][slot == IQ_FINAL ? WS::NB : slot];
            float sg[Tr::NLEV];
#pragma unroll
            for (int l = 0; l < Tr::NLEV; l++) sg[l] = sc * (float)(2 * l + 1);
            // the list's first quad is in flight while the terms are tabulated
            const uint2* lp = reinterpret_cast<const uint2*>(G.list) + off;
            const uint2 v0 = __ldg(lp);
            unsigned char* tw = smem + lb;
            auto put = [&](int row, float t) { *reinterpret_cast<float*>(tw + row * 256) = t; };
            // terms t_j(l) = (wv_j * (sc v_l - xv_j)) * (sc v_l - xv_j)
            float xs[Tr::NPOS], ws[Tr::NPOS];
#pragma unroll
            for (int j = 0; j < Tr::NPOS; j += 4) {
                const float4 xa = *reinterpret_cast<const float4*>(&W.xv[g][q * Tr::NPOS + j]);
                const float4 wa = *reinterpret_cast<const float4*>(&W.wv[g][q * Tr::NPOS + j]);
                xs[j] = xa.x; xs[j + 1] = xa.y; xs[j + 2] = xa.z; xs[j + 3] = xa.w;
                ws[j] = wa.x; ws[j + 1] = wa.y; ws[j + 2] = wa.z; ws[j + 3] = wa.w;
            }
            if (Tr::NPOS == 8) {
                float t0[4], t1[4];
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const float xj = xs[j], wj = ws[j];
#pragma unroll
                    for (int l = 0; l < 4; l++) {
                        const float df = sg[l] - xj;
                        const float t = (wj * df) * df;
                        if (j == 0) t0[l] = t;
                        else if (j == 1) t1[l] = t;
                        else put(R::row(j, l), t);
                    }
                }
#pragma unroll
                for (int l1 = 0; l1 < 4; l1++)
#pragma unroll
                    for (int l0 = 0; l0 < 4; l0++) put(l0 + 4 * l1, t0[l0] + t1[l1]);
            } else {
#pragma unroll
                for (int j = 0; j < Tr::NPOS; j++) {
                    const float xj = xs[j], wj = ws[j];
#pragma unroll
                    for (int l = 0; l < Tr::NLEV; l++) {
                        const float df = sg[l] - xj;
                        put(R::row(j, l), (wj * df) * df);
                    }
                }
            }
            // first candidate, then strict < over the rest: the first of equal distances wins
            float bd = iq_dist<Tr::NPOS, false>(tb, v0.x, lb);
            uint32_t bc = v0.x & 0xFFFF;
            auto take = [&](float d2, uint32_t code) {
                if (d2 < bd) { bd = d2; bc = code; }
            };
            auto quad = [&](const uint2 v) {
                take(iq_dist<Tr::NPOS, false>(tb, v.x, lb), v.x & 0xFFFF);
                take(iq_dist<Tr::NPOS, true>(tb, v.x, lb), v.x >> 16);
                take(iq_dist<Tr::NPOS, false>(tb, v.y, lb), v.y & 0xFFFF);
                take(iq_dist<Tr::NPOS, true>(tb, v.y, lb), v.y >> 16);
            };
            take(iq_dist<Tr::NPOS, true>(tb, v0.x, lb), v0.x >> 16);
            take(iq_dist<Tr::NPOS, false>(tb, v0.y, lb), v0.y & 0xFFFF);
            take(iq_dist<Tr::NPOS, true>(tb, v0.y, lb), v0.y >> 16);
            // quads are requested two iterations ahead of their use
            uint2 nx1 = n > 1 ? __ldg(lp + 1) : v0, nx2 = n > 2 ? __ldg(lp + 2) : v0;
            for (int c = 1; c < n; c++) {
                const uint2 cur = nx1;
                nx1 = nx2;
                if (c + 2 < n) nx2 = __ldg(lp + c + 2);
                quad(cur);
            }
            W.win[g][(slot == IQ_FINAL ? 0 : slot) * Tr::NSUB + q] = bc | IQ_SEARCHED;
        }
    }
    __syncwarp();
    if (lane == 0) W.nq = 0;
    __syncwarp();
}

// Index of the tentative code of subgroup q at inverse scale inv into the nbr table
// (base 3 for IQ2: sweep levels are clamped to 0..2; the code itself for IQ3).
template <class Tr>
__device__ __forceinline__ int iq_index(const float* xval, int q, float inv) {
    int idx = 0, mul = 1;
#pragma unroll
    for (int j = 0; j < Tr::NPOS; j++) {
        // clamp(rint(u), 0, MAXL) as an integer without the round and convert instructions (XU
        // pipe): u + 1.5 * 2^23 rounds u to an integer in the low mantissa bits (|u| is a few
        // units here); u is first raised to -1, which changes no level and sends NaN to 0 as
        // the float-to-int conversion did
        const float u = fmaxf(0.5f * (inv * xval[q * Tr::NPOS + j] - 1.0f), -1.0f);
        const int l = min(max(__float_as_int(__fadd_rn(u, 12582912.0f)) - 0x4B400000, 0), Tr::MAXL);
        if (Tr::BITS == 2) { idx += l * mul; mul *= 3; }
        else idx |= l << (3 * j);
    }
    return idx;
}

// Queue the off-grid subgroups of this lane's group (bit q of `mask` set: nbr entry v[q]).
template <class Tr>
__device__ __forceinline__ void iq_enqueue(IqWarpSmem<Tr>& W, int lane, uint32_t mask, const uint32_t* v, int slot) {
    int tot;
    int k = W.nq + warp_excl_scan(__popc(mask), lane, tot);
#pragma unroll
    for (int q = 0; q < Tr::NSUB; q++) {
        if (mask & (1u << q)) {
            W.off[k] = (uint16_t)(v[q] >> 9);
            W.len[k] = (uint8_t)(v[q] & 511);
            W.tag[k] = (uint16_t)(lane | (slot << 5) | (q << 9));
            k++;
        }
    }
    __syncwarp();
    if (lane == 0) W.nq += tot;
    __syncwarp();
}

// grid values (2l+1) of the resolved codes of one group -> q[GS]
template <class Tr>
__device__ __forceinline__ void iq_decode(const uint32_t* win, float* q) {
#pragma unroll
    for (int s = 0; s < Tr::NSUB; s++) {
        const int code = (int)(win[s] & 0xFFFF);
#pragma unroll
        for (int j = 0; j < Tr::NPOS; j++)  // 2l + 1 as a float: the bits of 2^23 + 2l + 1, minus 2^23
            q[s * Tr::NPOS + j] = __fadd_rn(__int_as_float(0x4B000001 + 2 * ((code >> (Tr::BITS * j)) & (Tr::NLEV - 1))),
                                            -8388608.0f);
    }
}

template <class Tr>
__device__ __forceinline__ void iq_sums(const float* w, const float* xval, const float* q, float& sumqx, float& sumq2) {
    float a[Tr::GS], b[Tr::GS];
#pragma unroll
    for (int i = 0; i < Tr::GS; i++) {
        a[i] = (w[i] * xval[i]) * q[i];
        b[i] = (w[i] * q[i]) * q[i];
    }
    if (Tr::SUMK == SUM_TORCH) {
        sumqx = torch_sum<Tr::GS>(a);
        sumq2 = torch_sum<Tr::GS>(b);
    } else {
        sumqx = tree_sum<Tr::GS>(a);
        sumq2 = tree_sum<Tr::GS>(b);
    }
}

template <int TYPE, bool IMAT>
__global__ void __launch_bounds__(IQ_WARPS * 32, IQ_MIN_CTAS) iq_kernel(QuantArgs a, IqGridDev G, IqParams prm) {
    using Tr = IqT<TYPE>;
    using WS = IqWarpSmem<Tr>;
    constexpr int GS = Tr::GS, NSUB = Tr::NSUB, SBG = QK_K / GS, SBW = 32 / SBG, SBT = IQ_WARPS * SBW, BB = Tr::BB;
    constexpr int NB = WS::NB;
    extern __shared__ __align__(16) unsigned char smem[];
    WS* wsm = reinterpret_cast<WS*>(smem + iq_tbl_bytes<Tr>());  // the term table comes first
    float* s_c = reinterpret_cast<float*>(smem + iq_tbl_bytes<Tr>() + IQ_WARPS * sizeof(WS));
    float* s_qp = s_c + 32;
    uint8_t* s_out = reinterpret_cast<uint8_t*>(s_qp + 32);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    WS& W = wsm[warp];
    if (tid < 32) s_c[tid] = prm.c[tid];
    if (tid < 8) s_qp[tid] = prm.qp[tid];
    if (lane == 0) W.nq = 0;
    __syncthreads();

    const int sbl = lane / SBG, gl = lane % SBG;  // superblock within the warp, group within it
    for (int64_t tile = blockIdx.x; tile * SBT < a.nblk; tile += gridDim.x) {
        const int64_t b = min(tile * SBT + warp * SBW + sbl, a.nblk - 1);
        float x[GS], w[GS], xval[GS];
        load_row<GS>(a.src, b * QK_K + gl * GS, a.src_type, x);

        // weights (iq2.py:429-431, iq2_xs.py:27-29, iq2_s.py:28-30, iq3_xxs.py:40-45)
        if (IMAT) {
            float* sq = &W.xv[0][0] + sbl * QK_K;  // xv is written only after the weights
#pragma unroll
            for (int i = 0; i < GS; i++) sq[gl * GS + i] = x[i] * x[i];
            __syncwarp();
            if (gl < 8) W.part[sbl][gl] = sb_sum256_partial(sq, gl);
            __syncwarp();
            const float sigma2 = __fdiv_rn(Tr::SIGFAC * sb_sum256_finish(W.part[sbl]), 256.0f);
            float qv[GS];
            load_f32<GS>(a.qw + (b % a.nblk_row) * QK_K + gl * GS, qv);
#pragma unroll
            for (int i = 0; i < GS; i++) w[i] = qv[i] * sqrtf(sigma2 + x[i] * x[i]);
            __syncwarp();
        } else {
#pragma unroll
            for (int i = 0; i < GS; i++) w[i] = x[i] * x[i];
        }

        // signs: parity fold (iq2.py:439-449) or explicit bits (iq2_s.py:32-34, iq3_s.py:51-55)
        uint32_t signs = 0;  // 7 or 8 bits per 8 values
#pragma unroll
        for (int s = 0; s < GS / 8; s++) {
            int sb = 0, nneg = 0;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                xval[8 * s + j] = fabsf(x[8 * s + j]);
                if (x[8 * s + j] < 0.0f) { sb |= 1 << j; nneg++; }
            }
            if (Tr::PARITY) {
                if (nneg & 1) {
                    int imin = 0;
                    float m = (w[8 * s] * x[8 * s]) * x[8 * s];
#pragma unroll
                    for (int j = 1; j < 8; j++) {
                        const float v = (w[8 * s + j] * x[8 * s + j]) * x[8 * s + j];
                        if (v < m) { m = v; imin = j; }
                    }
#pragma unroll
                    for (int j = 0; j < 8; j++)
                        if (j == imin) xval[8 * s + j] = -xval[8 * s + j];
                    sb ^= 1 << imin;
                }
                signs |= (uint32_t)(sb & 127) << (7 * s);
            } else {
                signs |= (uint32_t)sb << (8 * s);
            }
        }
#pragma unroll
        for (int i = 0; i < GS; i += 4) {
            *reinterpret_cast<float4*>(&W.xv[lane][i]) = make_float4(xval[i], xval[i + 1], xval[i + 2], xval[i + 3]);
            *reinterpret_cast<float4*>(&W.wv[lane][i]) =
                make_float4(sqrtf(w[i]), sqrtf(w[i + 1]), sqrtf(w[i + 2]), sqrtf(w[i + 3]));
        }

        const float gmax = max_of<GS>(xval);
        bool active = Tr::ACT_GT0 ? gmax > 0.0f : gmax >= Tr::EPS;
        float scale, r;
        if (Tr::INIT_QP) {  // iq2.py:458-463
            float Lq[GS];
            const float scale0 = qp_search<GS>(xval, w, 4.0f, s_qp, Lq);
            const float eff = scale0 * 3.0f;
            active = active && eff > 0.0f;
            r = rcp_rn(active ? eff : 1.0f);
            scale = scale0;
        } else {
            r = rcp_rn(active ? gmax : 1.0f);
            if (TYPE == QS_IQ2_XS || TYPE == QS_IQ2_S) scale = active ? __fdiv_rn(gmax, 5.0f) : 0.0f;
            else scale = __fdiv_rn(gmax, 15.0f);
        }
        float best = 0.0f;
        uint32_t cur[NSUB];
        const uint32_t cur0 = Tr::RP == RP_ALL_REDO ? (uint32_t)__ldg(G.kgrid) | IQ_SEARCHED : (uint32_t)__ldg(G.kgrid);
#pragma unroll
        for (int s = 0; s < NSUB; s++) cur[s] = cur0;  // grid index 0; og_init: IQ3_S starts off-grid
        __syncwarp();

        bool redo = false;
        if (Tr::ONE_SEARCH_SITE) {
            // sweep over the candidate scales, NB steps per batch of searches; the pass after the
            // last batch is the final reprojection at the accepted scale (one search call site)
            for (int s0 = 0;; s0 += NB) {
                const bool final_pass = s0 >= Tr::NSTEP;
                const int nb = final_pass ? 0 : min(NB, Tr::NSTEP - s0);
                if (!final_pass) {
                    // all codes of the batch first, so their table loads are in flight together
                    uint32_t nv[NB][NSUB];
    #pragma unroll
                    for (int j = 0; j < NB; j++) {
                        if (j < nb) {
                            const float inv = r * s_c[s0 + j];
                            W.psc[lane][j] = rcp_rn(inv);
    #pragma unroll
                            for (int q = 0; q < NSUB; q++) nv[j][q] = __ldg(G.nbr + iq_index<Tr>(xval, q, inv));
                        }
                    }
    #pragma unroll
                    for (int j = 0; j < NB; j++) {
                        if (j < nb) {
                            uint32_t mask = 0;
    #pragma unroll
                            for (int q = 0; q < NSUB; q++) {
                                const uint32_t v = nv[j][q];
                                if (v >> 31) W.win[lane][j * NSUB + q] = v & 0xFFFF;
                                else mask |= 1u << q;
                            }
                            iq_enqueue<Tr>(W, lane, mask, nv[j], j);
                        }
                    }
                } else {
                    // final reprojection at the accepted scale + least-squares refit
                    bool anyoff = false, allon = true;
    #pragma unroll
                    for (int q = 0; q < NSUB; q++) { anyoff |= (cur[q] & IQ_SEARCHED) != 0; allon &= (cur[q] & IQ_SEARCHED) == 0; }
                    float inv;
                    if (Tr::RP == RP_ALL_PROJ) {
                        redo = active && scale > 0.0f;
                        inv = rcp_rn(redo ? scale : 1.0f);
                    } else if (Tr::RP == RP_OFFGRID_NEED) {
                        redo = active && scale > 0.0f && !allon;
                        inv = rcp_rn(scale > 0.0f ? scale : 1.0f);
                    } else {
                        redo = active && anyoff && scale > 0.0f;
                        inv = rcp_rn(redo ? scale : 1.0f);
                    }
                    W.psc[lane][NB] = scale;
                    uint32_t v[NSUB], mask = 0;
    #pragma unroll
                    for (int q = 0; q < NSUB; q++) {
                        const bool want = redo && (Tr::RP == RP_ALL_PROJ || Tr::RP == RP_ALL_REDO || (cur[q] & IQ_SEARCHED));
                        // not reprojected: keep the current code (read back below without its flag)
                        v[q] = want ? __ldg(G.nbr + iq_index<Tr>(xval, q, inv)) : 0x80000000u | cur[q];
                    }
    #pragma unroll
                    for (int q = 0; q < NSUB; q++) {
                        if (v[q] >> 31) W.win[lane][q] = v[q] & 0xFFFF;
                        else mask |= 1u << q;
                    }
                    __syncwarp();
                    iq_enqueue<Tr>(W, lane, mask, v, IQ_FINAL);
                }
                iq_flush<Tr>(W, G, lane);
                if (final_pass) break;
                for (int j = 0; j < nb; j++) {
                    float qv[GS], sumqx, sumq2;
                    iq_decode<Tr>(&W.win[lane][j * NSUB], qv);
                    iq_sums<Tr>(w, xval, qv, sumqx, sumq2);
                    if (active && sumq2 > 0.0f && sumqx * sumqx > best * sumq2) {
                        const float ns = __fdiv_rn(sumqx, sumq2 < F32_TINY ? F32_TINY : sumq2);
                        scale = ns;
                        best = ns * sumqx;
    #pragma unroll
                        for (int q = 0; q < NSUB; q++) cur[q] = W.win[lane][j * NSUB + q];
                    }
                }
                __syncwarp();
            }
        } else {
            // sweep over the candidate scales, NB steps per batch of searches
            for (int s0 = 0; s0 < Tr::NSTEP; s0 += NB) {
                const int nb = min(NB, Tr::NSTEP - s0);
                // all codes of the batch first, so their table loads are in flight together
                uint32_t nv[NB][NSUB];
    #pragma unroll
                for (int j = 0; j < NB; j++) {
                    if (j < nb) {
                        const float inv = r * s_c[s0 + j];
                        W.psc[lane][j] = rcp_rn(inv);
    #pragma unroll
                        for (int q = 0; q < NSUB; q++) nv[j][q] = __ldg(G.nbr + iq_index<Tr>(xval, q, inv));
                    }
                }
    #pragma unroll
                for (int j = 0; j < NB; j++) {
                    if (j < nb) {
                        uint32_t mask = 0;
    #pragma unroll
                        for (int q = 0; q < NSUB; q++) {
                            const uint32_t v = nv[j][q];
                            if (v >> 31) W.win[lane][j * NSUB + q] = v & 0xFFFF;
                            else mask |= 1u << q;
                        }
                        iq_enqueue<Tr>(W, lane, mask, nv[j], j);
                    }
                }
                iq_flush<Tr>(W, G, lane);
                for (int j = 0; j < nb; j++) {
                    float qv[GS], sumqx, sumq2;
                    iq_decode<Tr>(&W.win[lane][j * NSUB], qv);
                    iq_sums<Tr>(w, xval, qv, sumqx, sumq2);
                    if (active && sumq2 > 0.0f && sumqx * sumqx > best * sumq2) {
                        const float ns = __fdiv_rn(sumqx, sumq2 < F32_TINY ? F32_TINY : sumq2);
                        scale = ns;
                        best = ns * sumqx;
    #pragma unroll
                        for (int q = 0; q < NSUB; q++) cur[q] = W.win[lane][j * NSUB + q];
                    }
                }
                __syncwarp();
            }

            // final reprojection at the accepted scale + least-squares refit
            bool anyoff = false, allon = true;
    #pragma unroll
            for (int q = 0; q < NSUB; q++) { anyoff |= (cur[q] & IQ_SEARCHED) != 0; allon &= (cur[q] & IQ_SEARCHED) == 0; }
            float inv;
            if (Tr::RP == RP_ALL_PROJ) {
                redo = active && scale > 0.0f;
                inv = rcp_rn(redo ? scale : 1.0f);
            } else if (Tr::RP == RP_OFFGRID_NEED) {
                redo = active && scale > 0.0f && !allon;
                inv = rcp_rn(scale > 0.0f ? scale : 1.0f);
            } else {
                redo = active && anyoff && scale > 0.0f;
                inv = rcp_rn(redo ? scale : 1.0f);
            }
            W.psc[lane][NB] = scale;
            {
                uint32_t v[NSUB], mask = 0;
    #pragma unroll
                for (int q = 0; q < NSUB; q++) {
                    const bool want = redo && (Tr::RP == RP_ALL_PROJ || Tr::RP == RP_ALL_REDO || (cur[q] & IQ_SEARCHED));
                    // not reprojected: keep the current code (read back below without its flag)
                    v[q] = want ? __ldg(G.nbr + iq_index<Tr>(xval, q, inv)) : 0x80000000u | cur[q];
                }
    #pragma unroll
                for (int q = 0; q < NSUB; q++) {
                    if (v[q] >> 31) W.win[lane][q] = v[q] & 0xFFFF;
                    else mask |= 1u << q;
                }
                __syncwarp();
                iq_enqueue<Tr>(W, lane, mask, v, IQ_FINAL);
            }
            iq_flush<Tr>(W, G, lane);
        }
        uint32_t fin[NSUB];
#pragma unroll
        for (int q = 0; q < NSUB; q++) fin[q] = W.win[lane][q] & 0xFFFF;
        {
            float qv[GS], sumqx, sumq2;
            iq_decode<Tr>(fin, qv);
            iq_sums<Tr>(w, xval, qv, sumqx, sumq2);
            if (redo && sumq2 > 0.0f) scale = __fdiv_rn(sumqx, sumq2 < F32_TINY ? F32_TINY : sumq2);
        }
        if (!redo) {
#pragma unroll
            for (int q = 0; q < NSUB; q++) fin[q] = cur[q] & 0xFFFF;
        }
#pragma unroll
        for (int q = 0; q < NSUB; q++) fin[q] = (uint32_t)__ldg(G.kmap + fin[q]);  // code -> grid index
        // negative least-squares scale: flip the scale and all the signs
        if (active && scale < 0.0f) {
            scale = -scale;
            signs = ~signs & (Tr::PARITY ? (GS == 32 ? 0x0FFFFFFFu : 0x3FFFu) : (GS == 32 ? 0xFFFFFFFFu : 0xFFFFu));
        }
        const float sc_g = active ? scale : 0.0f;

        // superblock: d = max_scale / 31, 4-bit sub-scales (iq2.py:87-108, iq2xs_common.py:345-355)
        float max_scale = sc_g;
#pragma unroll
        for (int o = 1; o < SBG; o <<= 1) {
            const float t = __shfl_xor_sync(0xffffffffu, max_scale, o);
            max_scale = t > max_scale ? t : max_scale;
        }
        const bool has = max_scale > 0.0f;
        const float d = __fdiv_rn(max_scale, 31.0f);
        const float inv_d = rcp_rn(has ? d : 1.0f);
        const int lnib = has ? (int)clampf(rintf(0.5f * (inv_d * sc_g - 1.0f)), 0.0f, 15.0f) : 0;
        uint8_t* o = s_out + (warp * SBW + sbl) * BB;
        if (gl == 0) {
            const uint16_t dh = f16_bits(has ? (Tr::DMUL == 1.0f ? d : d * Tr::DMUL) : 0.0f);
            o[0] = (uint8_t)dh;
            o[1] = (uint8_t)(dh >> 8);
        }
        if (TYPE == QS_IQ2_XXS) {
            uint32_t lo = 0, hi = 0;
            if (active && has) {
#pragma unroll
                for (int q = 0; q < 4; q++) lo |= (uint32_t)fin[q] << (8 * q);
                hi = signs;
            }
            if (has) hi |= (uint32_t)lnib << 28;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                o[2 + 8 * gl + i] = (uint8_t)(lo >> (8 * i));
                o[6 + 8 * gl + i] = (uint8_t)(hi >> (8 * i));
            }
        } else if (TYPE == QS_IQ2_XS) {
#pragma unroll
            for (int q = 0; q < 2; q++) {
                const uint32_t v = (active && has) ? ((uint32_t)fin[q] | (((signs >> (7 * q)) & 127) << 9)) : 0;
                o[2 + 4 * gl + 2 * q] = (uint8_t)v;
                o[3 + 4 * gl + 2 * q] = (uint8_t)(v >> 8);
            }
            const int ln1 = __shfl_down_sync(0xffffffffu, lnib, 1);
            if ((gl & 1) == 0) o[66 + gl / 2] = (uint8_t)(lnib | (ln1 << 4));
        } else if (TYPE == QS_IQ2_S) {
            int qh = 0;
#pragma unroll
            for (int q = 0; q < 2; q++) {
                const int gi = active ? fin[q] : 0;
                o[2 + 2 * gl + q] = (uint8_t)(gi & 255);
                o[34 + 2 * gl + q] = (uint8_t)(active ? (signs >> (8 * q)) & 255 : 0);
                qh |= (gi >> 8) << (2 * (2 * (gl & 1) + q));
            }
            const int qh1 = __shfl_down_sync(0xffffffffu, qh, 1);
            const int ln1 = __shfl_down_sync(0xffffffffu, lnib, 1);
            if ((gl & 1) == 0) {
                o[66 + gl / 2] = (uint8_t)(qh | qh1);
                o[74 + gl / 2] = (uint8_t)(lnib | (ln1 << 4));
            }
        } else if (TYPE == QS_IQ3_XXS) {
#pragma unroll
            for (int q = 0; q < 8; q++) o[2 + 8 * gl + q] = (uint8_t)((active && has) ? fin[q] : 0);
            const uint32_t word = has ? ((active ? signs : 0) | ((uint32_t)lnib << 28)) : 0;
#pragma unroll
            for (int i = 0; i < 4; i++) o[66 + 4 * gl + i] = (uint8_t)(word >> (8 * i));
        } else {  // IQ3_S: live groups compact toward the front of qs / signs (iq3_s.py:113-122)
#pragma unroll
            for (int i = 0; i < 8; i++) o[2 + 8 * gl + i] = 0;
#pragma unroll
            for (int i = 0; i < 4; i++) o[74 + 4 * gl + i] = 0;
            const unsigned act = __ballot_sync(0xffffffffu, active);
            const unsigned mine = (act >> (sbl * SBG)) & ((1u << SBG) - 1);
            const int slot = __popc(mine & ((1u << gl) - 1));
            __syncwarp();
            int qh = 0;
            if (active) {
#pragma unroll
                for (int q = 0; q < 8; q++) {
                    o[2 + 8 * slot + q] = (uint8_t)(fin[q] & 255);
                    qh |= (fin[q] >> 8) << q;
                }
#pragma unroll
                for (int i = 0; i < 4; i++) o[74 + 4 * slot + i] = (uint8_t)(signs >> (8 * i));
            }
            o[66 + gl] = (uint8_t)qh;
            const int ln1 = __shfl_down_sync(0xffffffffu, lnib, 1);
            if ((gl & 1) == 0) o[106 + gl / 2] = (uint8_t)(lnib | (ln1 << 4));
        }
        __syncthreads();
        store_tile(a, s_out, tile * SBT, (int)min((int64_t)SBT, a.nblk - tile * SBT), BB, tid, blockDim.x);
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// host launch
// ---------------------------------------------------------------------------
template <int TYPE, bool IMAT>
static cudaError_t launch_one(const QuantArgs& a, const LaunchCtx& ctx, const IqTables* t, const IqParams& p) {
    using Tr = IqT<TYPE>;
    constexpr size_t smem = iq_smem_bytes<Tr>();
    auto k = iq_kernel<TYPE, IMAT>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, IQ_WARPS * 32, smem) != cudaSuccess || per_sm < 1)
        per_sm = 1;
    constexpr int SBT = IQ_WARPS * (32 / (QK_K / Tr::GS));
    const int64_t tiles = (a.nblk + SBT - 1) / SBT;
    const int64_t g = (int64_t)per_sm * ctx.num_sms;
    const int grid = (int)(tiles < g ? tiles : g);
    k<<<grid, IQ_WARPS * 32, smem, ctx.stream>>>(a, t->g[Tr::GID], p);
    return cudaGetLastError();
}

cudaError_t launch_iq(int type, const QuantArgs& a, const LaunchCtx& ctx, const IqTables* t) {
    IqParams p;
    memset(&p, 0, sizeof(p));
    const bool imat = a.qw != nullptr;
    switch (type) {
    case QS_IQ2_XXS: {
        for (int s = -6; s <= 6; s++) p.c[s + 6] = (float)(5.0 + 0.1 * s);  // iq2.py:470 (double, then f32)
        int j = 0;
        for (int s = -4; s <= 4; s++) if (s) p.qp[j++] = (float)(0.1 * s + 4.0);  // iq2.py:387
        return imat ? launch_one<QS_IQ2_XXS, true>(a, ctx, t, p) : cudaErrorInvalidValue;
    }
    case QS_IQ2_XS:
    case QS_IQ2_S:
        for (int s = -9; s <= 9; s++) p.c[s + 9] = 5.0f + (float)s * 0.1f;  // iq2xs_common.py:21
        if (!imat) return cudaErrorInvalidValue;
        return type == QS_IQ2_XS ? launch_one<QS_IQ2_XS, true>(a, ctx, t, p) : launch_one<QS_IQ2_S, true>(a, ctx, t, p);
    case QS_IQ3_XXS:
        for (int s = -15; s <= 15; s++) p.c[s + 15] = 15.0f + (float)s * 0.2f;  // iq3_xxs.py:22
        return imat ? launch_one<QS_IQ3_XXS, true>(a, ctx, t, p) : launch_one<QS_IQ3_XXS, false>(a, ctx, t, p);
    case QS_IQ3_S:
        for (int s = -9; s <= 9; s++) p.c[s + 9] = 15.0f + (float)s * 0.2f;  // iq3_s.py:22
        return imat ? launch_one<QS_IQ3_S, true>(a, ctx, t, p) : launch_one<QS_IQ3_S, false>(a, ctx, t, p);
    default:
        return cudaErrorInvalidValue;
    }
}

}  // namespace qs
