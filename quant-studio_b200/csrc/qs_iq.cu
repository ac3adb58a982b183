// IQ2_XXS / IQ2_XS / IQ2_S / IQ3_XXS / IQ3_S lattice-search kernels (sm_100a).
//
// Reference: kernels/iq2.py:418-498 (IQ2_XXS), kernels/iq2xs_common.py:280-355 with
// iq2_xs.py:20-69 / iq2_s.py:21-62, kernels/iq3_xxs.py:31-134, kernels/iq3_s.py:31-140.
//
// Mapping. One thread per quantization group (16 or 32 values, in registers) runs the
// weights, the sign handling and the accept chain over the candidate scales; a warp owns 32
// groups. The grid projections are where the time goes: at every sweep step a subgroup's
// tentative code is either on the lattice (one table lookup) or needs the nearest grid point
// of a list of 1..292 candidates under the weighted distance d2 = sum_j s_j (sc g_j - x_j)^2
// in the reference's float arithmetic (the first of equal distances wins).
//
// Certified runs. The tentative code of a subgroup changes only every few sweep steps while
// the scale moves by about 1 % a step. In real arithmetic d2 = sc^2 A - 2 sc B + C with
// A = sum s g^2 and B = sum s x g independent of sc, so the candidates of one list rank as
// lines in sc. A "job" is a run of up to 8 consecutive steps at which a subgroup has the
// same off-grid code: one pass over the list computes each candidate's A and
// B (as A' and L below) and scores it at the run's first and last step. When the same
// candidate wins at both ends by more than a bound on every rounding error involved (the
// reference's float d2 against the real distance, and this pass's own arithmetic), it is the
// reference's choice at every step of the run: the score gaps are linear in sc and the bound
// is convex (see cert_q). A job that fails is scored again at each of its steps, and a step
// that still fails is searched exactly as the reference does; so is the final reprojection.
//
// Lockstep. Jobs and exact searches are queued per warp in shared memory, counting-sorted by
// list length and handed out one per lane, so the 32 lanes walk lists of similar length
// together with no synchronisation inside a walk. An exact IQ2 search first tabulates the
// 4 x 8 distance terms of its subgroup (the CTA's term table: one 256-byte row per term, one
// column per lane) and then needs one table read and one add per position and candidate; an
// exact IQ3 search evaluates its few candidates directly.
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
    const uint32_t* nbr;    // code index -> 0x80000000 | grid index (on the grid), else
                            // list start in quads << 9 | list length in codes
    const uint16_t* list;   // neighbour lists as codes, (distance, index) order, padded to whole
                            // quads with copies of the last code (a copy never wins a strict <)
    const uint32_t* lvl;    // per list entry, the candidate's level at each position, one byte
                            // each (IQ3: one word, IQ2: two words)
    const uint16_t* gidx;   // per list entry, the candidate's grid index
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
                       std::vector<uint16_t>& list, std::vector<uint32_t>& lvl, std::vector<uint16_t>& gidx) {
    const int mask = (1 << bits) - 1;
    const int kmap_size = bits == 2 ? 43692 : 4096;
    std::vector<int> kmap(kmap_size, -1);
    for (int i = 0; i < G; i++) kmap[kgrid[i]] = i;
    const int nidx = bits == 2 ? 6561 : 4096;
    const int nw = npos / 4;  // level words per entry
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
            nbr[idx] = 0x80000000u | (uint32_t)kmap[code];
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
        nbr[idx] = ((uint32_t)(list.size() / 4) << 9) | (uint32_t)n;
        for (int i = 0; i < 4 * nq; i++) {
            const int k = (int)(keys[i < n ? i : n - 1] % 65536);
            list.push_back(kgrid[k]);
            gidx.push_back((uint16_t)k);
            for (int w = 0; w < nw; w++) {
                uint32_t word = 0;
                for (int b = 0; b < 4; b++) word |= (uint32_t)((kgrid[k] >> (bits * (4 * w + b))) & mask) << (8 * b);
                lvl.push_back(word);
            }
        }
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
        T->g[t] = IqGridDev{kg, nullptr, nullptr, nullptr, nullptr, kGrids[t].G};
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
    std::vector<uint32_t> nbr, lvl;
    std::vector<uint16_t> list, gidx;
    const GridSpec& sp = kGrids[t];
    build_grid(sp.grid, sp.G, sp.bits, sp.npos, sp.nwant, nbr, list, lvl, gidx);
    if (list.size() / 4 >= (1u << 23)) return cudaErrorInvalidValue;  // nbr entries hold 23-bit quad offsets
    auto al = [](size_t n) { return (n + 255) & ~(size_t)255; };
    const size_t o_list = al(nbr.size() * 4), o_lvl = o_list + al(list.size() * 2 + 16),
                 o_gidx = o_lvl + al(lvl.size() * 4), total = o_gidx + al(gidx.size() * 2);
    char* mem = nullptr;
    cudaError_t e = cudaMalloc(&mem, total);
    if (e != cudaSuccess) return e;
    uint32_t* nb = reinterpret_cast<uint32_t*>(mem);
    uint16_t* ls = reinterpret_cast<uint16_t*>(mem + o_list);
    uint32_t* lv = reinterpret_cast<uint32_t*>(mem + o_lvl);
    uint16_t* gi = reinterpret_cast<uint16_t*>(mem + o_gidx);
    if ((e = cudaMemcpy(nb, nbr.data(), nbr.size() * 4, cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaMemcpy(ls, list.data(), list.size() * 2, cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaMemcpy(lv, lvl.data(), lvl.size() * 4, cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaMemcpy(gi, gidx.data(), gidx.size() * 2, cudaMemcpyHostToDevice)) != cudaSuccess) {
        cudaFree(mem);
        return e;
    }
    T->gmem[t] = mem;
    T->g[t].nbr = nb;
    T->g[t].list = ls;
    T->g[t].lvl = lv;
    T->g[t].gidx = gi;
    T->built[t] = true;
    return cudaSuccess;
}

const uint16_t* iq_kgrid(const IqTables* t, int type) {
    const int g = grid_of(type);
    return g < 0 ? nullptr : t->g[g].kgrid;
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

// SW: sweep steps resolved before their accept chain runs (a window; SW * NSUB <= 64): the
// whole sweep for IQ2, 8 steps for IQ3 (whose result table would not fit otherwise);
// CUT8: jobs end at every 8th step of the window (else only after 8 steps): shorter runs
// certify more often, which pays where lists are short (measured per type);
// BINS: list-length classes of the counting sort (the longest list in quads of 4, plus one);
// MIN_CTAS: resident CTAs per SM (shared memory allows it) and MAXREG the register cap that fits them.
template <int T> struct IqT;
template <> struct IqT<QS_IQ2_XXS> {
    static constexpr int GS = 32, NSUB = 4, NPOS = 8, BITS = 2, NLEV = 4, MAXL = 2, NSTEP = 13, BB = 66, GID = G_IQ2XXS;
    static constexpr int GRID = 256, SW = 13, BINS = 39, MIN_CTAS = 5, MAXREG = 200;
    static constexpr bool CUT8 = false;
    static constexpr bool PARITY = true, ACT_GT0 = false, INIT_QP = true;
    static constexpr int SUMK = SUM_TORCH, RP = RP_ALL_PROJ;
    static constexpr float EPS = EPS15, SIGFAC = 1.0f, DMUL = 1.0f;
};
template <> struct IqT<QS_IQ2_XS> {
    static constexpr int GS = 16, NSUB = 2, NPOS = 8, BITS = 2, NLEV = 4, MAXL = 2, NSTEP = 19, BB = 74, GID = G_IQ2XS;
    static constexpr int GRID = 512, SW = 19, BINS = 74, MIN_CTAS = 6, MAXREG = 168;
    static constexpr bool CUT8 = false;
    static constexpr bool PARITY = true, ACT_GT0 = false, INIT_QP = false;
    static constexpr int SUMK = SUM_TREE, RP = RP_OFFGRID_NEED;
    static constexpr float EPS = EPS15, SIGFAC = 1.0f, DMUL = 1.0f;
};
template <> struct IqT<QS_IQ2_S> {
    static constexpr int GS = 16, NSUB = 2, NPOS = 8, BITS = 2, NLEV = 4, MAXL = 2, NSTEP = 19, BB = 82, GID = G_IQ2S;
    static constexpr int GRID = 1024, SW = 19, BINS = 19, MIN_CTAS = 6, MAXREG = 168;
    static constexpr bool CUT8 = true;
    static constexpr bool PARITY = false, ACT_GT0 = false, INIT_QP = false;
    static constexpr int SUMK = SUM_TREE, RP = RP_OFFGRID_NEED;
    static constexpr float EPS = EPS8, SIGFAC = 2.0f, DMUL = 0.9875f;
};
template <> struct IqT<QS_IQ3_XXS> {
    static constexpr int GS = 32, NSUB = 8, NPOS = 4, BITS = 3, NLEV = 8, MAXL = 7, NSTEP = 31, BB = 98, GID = G_IQ3XXS;
    static constexpr int GRID = 256, SW = 8, BINS = 10, MIN_CTAS = 6, MAXREG = 168;
    static constexpr bool CUT8 = false;
    static constexpr bool PARITY = true, ACT_GT0 = false, INIT_QP = false;
    static constexpr int SUMK = SUM_TREE, RP = RP_OFFGRID_REDO;
    static constexpr float EPS = EPS8, SIGFAC = 2.0f, DMUL = 1.0125f;
};
template <> struct IqT<QS_IQ3_S> {
    static constexpr int GS = 32, NSUB = 8, NPOS = 4, BITS = 3, NLEV = 8, MAXL = 7, NSTEP = 19, BB = 110, GID = G_IQ3S;
    static constexpr int GRID = 512, SW = 8, BINS = 11, MIN_CTAS = 6, MAXREG = 168;
    static constexpr bool CUT8 = false;
    static constexpr bool PARITY = false, ACT_GT0 = true, INIT_QP = false;
    static constexpr int SUMK = SUM_TREE, RP = RP_ALL_REDO;
    static constexpr float EPS = 0.0f, SIGFAC = 2.0f, DMUL = 1.033f;
};

struct IqParams {
    float c[32];   // sweep-step numerators
    float qp[8];   // make_qp numerators (IQ2_XXS initial scale)
};

constexpr int IQ_WARPS = 2;       // warps per CTA; each warp owns 32 groups
constexpr int IQ_CAP = 256;       // queued jobs or exact searches per warp
constexpr int IQ_RUN = 8;         // steps per job at most
constexpr int IQ_FINAL = 31;      // slot of the final reprojection in an exact search's tag
constexpr uint16_t IQ_SEARCHED = 0x8000;     // flag beside a resolved grid index: it came from a search
constexpr uint32_t IQ_ONGRID = 0x80000000u;  // nbr entry of an on-grid code (| grid index)
constexpr unsigned IQ_FULL = 0xffffffffu;

// Rows of the CTA term table of the exact IQ2 searches (256 bytes each: 64 columns of f32,
// warp * 32 + lane; 16-bit codes, 2 bits per position): rows 0..15 hold t0 + t1 for the pair
// of levels (code & 15); positions 3, 5, 7 have a level stride of 4 rows and interleave in
// rows 16..30; positions 2, 4, 6 have consecutive rows from 32, 36, 40.
struct IqRows8 {
    static constexpr int N = 44;
    __host__ __device__ static constexpr int row(int j, int l) {
        return j == 2 ? 32 + l : j == 3 ? 16 + 4 * l : j == 4 ? 36 + l : j == 5 ? 17 + 4 * l : j == 6 ? 40 + l : 18 + 4 * l;
    }
};

template <class Tr>
struct IqWarpSmem {
    static constexpr int SW = Tr::SW;
    static constexpr int XS = Tr::GS + 4;  // row pitch: 16-byte rows, and 8 lanes' own-row float4s hit 8 bank quads
    static constexpr int WINS = 2 * (((SW * Tr::NSUB + 1) / 2) | 1);  // an odd number of words: lane rows conflict-free
    __align__(16) float xv[32][XS];  // search-space values of every group (|x|, parity-folded);
                                     // holds the superblock squares while the weights are computed
    __align__(16) float wv[32][XS];  // sqrt of the weights
    float rg[32];                    // per group: r, the search scale of step j being 1 / (r c_j)
    float psc[32][Tr::SW <= 8 ? Tr::SW + 1 : 1];  // short windows: those scales (odd pitch: random groups
                                                  // read by the lanes spread over the banks)
    float fsc[32];                   // per group: the scale of the final reprojection
    unsigned long long xflag[32];    // per group: steps (bit j * NSUB + q) left to an exact search
    uint32_t rec[IQ_CAP];            // queue: the code's nbr entry (list start and length)
    uint16_t tag[IQ_CAP];            // job: group | subgroup << 5 | first step << 8 | (steps - 1) << 13;
                                     // exact search: group | step (or IQ_FINAL) << 5 | subgroup << 10
    uint8_t ord[IQ_CAP];             // queue entries in order of list length
    uint8_t rank[IQ_CAP];            // counting-sort ranks, then the jobs to score step by step
    uint32_t hist[(Tr::BINS + 1) / 2];  // two 16-bit counters (then bin starts) per word
    uint16_t win[32][WINS];          // per step j and subgroup q, at j * NSUB + q: the resolved grid
                                     // index (| IQ_SEARCHED when it came from a search)
    float part[4][8];
};

template <class Tr>
__host__ __device__ constexpr size_t iq_tbl_bytes() { return Tr::NPOS == 8 ? (size_t)IqRows8::N * 256 : 0; }
template <class Tr>
__host__ __device__ constexpr size_t iq_kg_bytes() { return ((size_t)Tr::GRID * 2 + 15) & ~(size_t)15; }

template <class Tr>
constexpr size_t iq_smem_bytes() {
    return iq_tbl_bytes<Tr>() + IQ_WARPS * sizeof(IqWarpSmem<Tr>) + 64 * 4 + iq_kg_bytes<Tr>() +
           IQ_WARPS * 4 * Tr::BB + 64;
}

// ---------------------------------------------------------------------------
// queue and counting sort
// ---------------------------------------------------------------------------
__device__ __forceinline__ int warp_excl_scan(int v, int lane, int& total) {
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(IQ_FULL, x, o);
        if (lane >= o) x += y;
    }
    total = __shfl_sync(IQ_FULL, x, 31);
    return x - v;
}

// Append (rec, tag) for every lane whose `pred` is set; nq (warp-uniform) counts the queue.
template <class Tr>
__device__ __forceinline__ void iq_push(IqWarpSmem<Tr>& W, int& nq, int lane, bool pred, uint32_t rec, uint32_t tag) {
    const unsigned b = __ballot_sync(IQ_FULL, pred);
    if (pred) {
        const int k = nq + __popc(b & ((1u << lane) - 1u));
        W.rec[k] = rec;
        W.tag[k] = (uint16_t)tag;
    }
    nq += __popc(b);
}

template <class Tr>
__device__ __forceinline__ int iq_bin(uint32_t rec) {
    return Tr::BINS - 1 - min(Tr::BINS - 1, (int)(((rec & 511) + 3) >> 2));
}

// Counting sort of the P queued entries by list length, longest first: W.ord.
template <class Tr>
__device__ void iq_sort(IqWarpSmem<Tr>& W, int P, int lane) {
    constexpr int HW = (Tr::BINS + 1) / 2, PER = 2 * ((HW + 31) / 32);  // bins per lane (even)
    for (int i = lane; i < HW; i += 32) W.hist[i] = 0;
    __syncwarp();
    for (int i = lane; i < P; i += 32) {
        const int bin = iq_bin<Tr>(W.rec[i]);
        const int sh = 16 * (bin & 1);
        W.rank[i] = (uint8_t)((atomicAdd(&W.hist[bin >> 1], 1u << sh) >> sh) & 0xFFFF);
    }
    __syncwarp();
    {
        int cnt[PER], sum = 0;
#pragma unroll
        for (int k = 0; k < PER; k++) {
            const int b = lane * PER + k;
            cnt[k] = b < Tr::BINS ? (int)((W.hist[b >> 1] >> (16 * (b & 1))) & 0xFFFF) : 0;
            sum += cnt[k];
        }
        int tot;
        int run = warp_excl_scan(sum, lane, tot);
        __syncwarp();
#pragma unroll
        for (int k = 0; k < PER; k += 2) {
            const int b = lane * PER + k;
            if (b < Tr::BINS) W.hist[b >> 1] = (uint32_t)run | ((uint32_t)(run + cnt[k]) << 16);
            run += cnt[k] + cnt[k + 1];
        }
    }
    __syncwarp();
    for (int i = lane; i < P; i += 32) {
        const int bin = iq_bin<Tr>(W.rec[i]);
        W.ord[((W.hist[bin >> 1] >> (16 * (bin & 1))) & 0xFFFF) + W.rank[i]] = (uint8_t)i;
    }
    __syncwarp();
}

// The NPOS search-space values and weight roots of subgroup q of group g.
template <class Tr>
__device__ __forceinline__ void iq_load_sub(const IqWarpSmem<Tr>& W, int g, int q, float* xs, float* ws) {
#pragma unroll
    for (int j = 0; j < Tr::NPOS; j += 4) {
        const float4 xa = *reinterpret_cast<const float4*>(&W.xv[g][q * Tr::NPOS + j]);
        const float4 wa = *reinterpret_cast<const float4*>(&W.wv[g][q * Tr::NPOS + j]);
        xs[j] = xa.x; xs[j + 1] = xa.y; xs[j + 2] = xa.z; xs[j + 3] = xa.w;
        ws[j] = wa.x; ws[j + 1] = wa.y; ws[j + 2] = wa.z; ws[j + 3] = wa.w;
    }
}

// ---------------------------------------------------------------------------
// certified search
// ---------------------------------------------------------------------------
// Notation: a subgroup's values x_j and weight roots s_j >= 0 (j < NPOS), a candidate's
// levels l_j and grid values g_j = 2 l_j + 1, the scale sc > 0, and u = 2^-24. The reference
// computes d2 = sum_j fl(fl(s_j fl(fl(sc g_j) - x_j)) fl(sc g_j) - x_j) ...) in float, adds
// in some order, and keeps the first least d2. The real distance is
//   D = sum_j s_j (sc g_j - x_j)^2 = sc^2 A - 2 sc B + C,
//   A = sum s g^2 = 4 A' + S0,  B = sum s x g = 2 L + sum s x,  C = sum s x^2,
//   A' = sum s l (l + 1),  L = sum (s x) l,  S0 = sum s,
// so D_k - D_m = 4 sc (S_k - S_m) with the score S = sc A' - L, and S is what this pass ranks.
//
// Error bounds, with b_j = sc g_j + |x_j| and M = sum_j s_j b_j^2 <= 2 (sc^2 A + C) =: 2 Q:
//  - reference: fl(sc g) and the subtraction give diff = d + e with |e| <= 2 u b (1 + u);
//    each term then carries at most 6.0001 u s b^2, the NPOS - 1 additions at most
//    (NPOS - 1) u (1 + 7 u) sum s b^2: |d2 - D| <= (NPOS + 5.01) u M;
//  - this pass (one rounding per multiply, fused multiply-add and add): A' to NPOS u A',
//    s x to u and L to (NPOS + 1) u sum |s x| l; with 4 sc^2 A' <= sum s (sc g)^2 and
//    4 sc l |x| <= 2 sc g |x|, |4 sc (S~ - S)| <= (NPOS + 1) u M, and the rounding of the score
//    itself adds u M.
// Two candidates compared: 2 (NPOS + 5.01 + NPOS + 1 + 1) u 2 Q = (8 NPOS + 28.04) u Q in D
// units, i.e. tau = K u Q / (4 sc) in score units with K = 64 (NPOS 4, needs 60.04) or 96
// (NPOS 8, needs 92.04); the slack covers the roundings of tau, Q, A'max and the gap
// themselves. A gap in S at sc above tau(sc) therefore orders the two candidates' reference
// d2 the same way, strictly. tau(sc) = (K u / 4)(A sc + C / sc) is convex in sc and a gap in S
// is linear in sc, so a gap above max(tau) at both ends of a run holds at every step between.
// The guards keep every quantity of both computations in the normal range with no overflow
// (|x|, s <= 2^40, sc in [2^-40, 2^16], Q in [2^-40, 2^60]): what underflow can add is below
// 2^-100 against a slack above 2^-64, and NaN or infinite inputs fail the guards.
struct IqCertSub { float S0, C, XM; };  // sum s, sum s x^2, max |x|

template <int NPOS>
__device__ __forceinline__ IqCertSub cert_setup(const float* xs, const float* ws, float* sx) {
    IqCertSub c{0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < NPOS; j++) {
        sx[j] = __fmul_rn(ws[j], xs[j]);
        c.S0 = __fadd_rn(c.S0, ws[j]);
        c.C = __fmaf_rn(sx[j], xs[j], c.C);
        c.XM = fmaxf(c.XM, fabsf(xs[j]));
    }
    return c;
}

template <class Tr>
__device__ __forceinline__ float cert_q(const IqCertSub& c, float sc, float apmax) {
    return __fmaf_rn(__fmul_rn(sc, sc), __fmaf_rn(4.0f, apmax, c.S0), c.C);
}

// the guards, false for NaN
template <class Tr>
__device__ __forceinline__ bool cert_ok(const IqCertSub& c, float sc, float apmax) {
    const float Q = cert_q<Tr>(c, sc, apmax);
    return sc >= 0x1p-40f && sc <= 0x1p16f && c.S0 <= 0x1p40f && c.XM <= 0x1p40f && Q >= 0x1p-40f && Q <= 0x1p60f;
}

// The certified pass uses the packed f32x2 arithmetic of qs_common.cuh: its bound counts one
// rounding per operation and term, whatever the order.

// A' and L of one candidate from its level bytes (one per position), two positions per
// packed operation; ws2 / sx2 hold s and s x of positions 2k, 2k + 1.
template <int NPOS>
__device__ __forceinline__ void cert_terms(const uint32_t* lw, const f32x2* ws2, const f32x2* sx2, float& ap, float& lx) {
    constexpr f32x2 M223 = 0xCB000000CB000000ull;  // (-2^23, -2^23)
    f32x2 a2 = 0, b2 = 0;
#pragma unroll
    for (int k = 0; k < NPOS / 2; k++) {
        // the bytes as the low bits of 2^23, minus 2^23: the levels as floats
        const uint32_t w = lw[k >> 1];
        const f32x2 lf = f2_add(f2_pack(__int_as_float((int)__byte_perm(w, 0x4B000000u, 0x7440u | ((2 * k) & 3))),
                                        __int_as_float((int)__byte_perm(w, 0x4B000000u, 0x7440u | ((2 * k + 1) & 3)))),
                                M223);
        const f32x2 p = f2_fma(lf, lf, lf);
        a2 = k == 0 ? f2_mul_z(ws2[0], p) : f2_fma(ws2[k], p, a2);
        b2 = k == 0 ? f2_mul_z(sx2[0], lf) : f2_fma(sx2[k], lf, b2);
    }
    float a0, a1, b0, b1;
    f2_unpack(a2, a0, a1);
    f2_unpack(b2, b0, b1);
    ap = __fadd_rn(a0, a1);
    lx = __fadd_rn(b0, b1);
}

// least and second least score, and the first candidate with the least
struct IqBest { float m1, m2; int w; };
__device__ __forceinline__ void best_init(IqBest& b) {
    b.m1 = b.m2 = __int_as_float(0x7f800000);
    b.w = 0;
}
// a NaN score leaves m2 == m1 (no certificate)
__device__ __forceinline__ void best_take(IqBest& b, float s, int c) {
    b.m2 = fminf(b.m2, fmaxf(b.m1, s));
    b.w = s < b.m1 ? c : b.w;
    b.m1 = fminf(b.m1, s);
}

// Level words of one quad of list entries (4 candidates, NW words each).
template <int NW> struct IqLvlQuad { uint4 h[NW]; };
template <int NW>
__device__ __forceinline__ IqLvlQuad<NW> lvl_quad(const uint4* lq, int qd) {
    IqLvlQuad<NW> r;
#pragma unroll
    for (int k = 0; k < NW; k++) r.h[k] = __ldg(lq + qd * NW + k);
    return r;
}

// A' and L of the n candidates of a list, in list order, to f(A', L, position). The loop is
// rolled (one candidate per iteration, a small body for the instruction cache): the current
// quad's level words rotate down by one candidate per step while the next quad is in flight
// (q0, the first, is requested by the caller). The padding copies of the last candidate are
// never visited: a copy would tie with it.
template <int NPOS, class F>
__device__ __forceinline__ void cert_walk(const uint4* lq, const IqLvlQuad<NPOS / 4>& q0, int n, const f32x2* ws2,
                                          const f32x2* sx2, F&& f) {
    constexpr int NW = NPOS / 4;
    const int nq4 = (n + 3) >> 2;
    IqLvlQuad<NW> cur = q0, nx = q0;
    if (nq4 > 1) nx = lvl_quad<NW>(lq, 1);
#pragma unroll 1
    for (int c = 0; c < n; c++) {
        uint32_t lw[NW];
        lw[0] = cur.h[0].x;
        if (NW == 2) lw[NW - 1] = cur.h[0].y;
        if ((c & 3) == 3) {
            cur = nx;
            if ((c >> 2) + 2 < nq4) nx = lvl_quad<NW>(lq, (c >> 2) + 2);
        } else if (NW == 1) {
            cur.h[0] = make_uint4(cur.h[0].y, cur.h[0].z, cur.h[0].w, 0u);
        } else {
            cur.h[0] = make_uint4(cur.h[0].z, cur.h[0].w, cur.h[NW - 1].x, cur.h[NW - 1].y);
            cur.h[NW - 1] = make_uint4(cur.h[NW - 1].z, cur.h[NW - 1].w, 0u, 0u);
        }
        float ap, lx;
        cert_terms<NPOS>(lw, ws2, sx2, ap, lx);
        f(ap, lx, c);
    }
}

// Search scale of window step j of group g: 1 / (r c_j), from the table for short windows
template <class Tr>
__device__ __forceinline__ float iq_step_scale(const IqWarpSmem<Tr>& W, int g, int j, const float* cw) {
    if (Tr::SW <= 8) return W.psc[g][Tr::SW <= 8 ? j : 0];
    return rcp_rn(W.rg[g] * cw[j]);
}

// Solve the P queued jobs: certified at the ends of each run, then step by step for the
// runs that failed; the steps that fail again get their bit in W.xflag. Returns (warp-
// uniform) whether any did. A job's tag: group | subgroup << 5 | first step << 8 |
// (steps - 1) << 13, steps counted within the window, whose step numerators are cw[].
template <class Tr>
__device__ bool iq_job_flush(IqWarpSmem<Tr>& W, const IqGridDev& G, int lane, int P, const float* cw) {
    constexpr int NPOS = Tr::NPOS, SW = Tr::SW, NSUB = Tr::NSUB, NW = NPOS / 4;
    constexpr float KU4 = (NPOS == 4 ? 64.0f : 96.0f) * 0x1p-24f * 0.25f;
    iq_sort<Tr>(W, P, lane);
    int nretry = 0;
    for (int pb = 0; pb < P; pb += 32) {
        const int i = pb + lane;
        bool retry = false;
        int p = 0;
        if (i < P) {
            p = W.ord[i];
            const uint32_t rec = W.rec[p], tg = W.tag[p];
            const int g = tg & 31, q = (tg >> 5) & 7, j0 = (tg >> 8) & 31, len = ((tg >> 13) & 7) + 1;
            const uint4* lq = reinterpret_cast<const uint4*>(G.lvl) + (size_t)(rec >> 9) * NW;
            const IqLvlQuad<NW> q0 = lvl_quad<NW>(lq, 0);
            const float sa = iq_step_scale<Tr>(W, g, j0, cw), sb = iq_step_scale<Tr>(W, g, j0 + len - 1, cw);
            float xs[NPOS], ws[NPOS], sx[NPOS];
            iq_load_sub<Tr>(W, g, q, xs, ws);
            const IqCertSub cs = cert_setup<NPOS>(xs, ws, sx);
            f32x2 ws2[NPOS / 2], sx2[NPOS / 2];
#pragma unroll
            for (int k = 0; k < NPOS / 2; k++) {
                ws2[k] = f2_pack(ws[2 * k], ws[2 * k + 1]);
                sx2[k] = f2_pack(sx[2 * k], sx[2 * k + 1]);
            }
            const uint32_t e0 = (rec >> 9) * 4;
            const int n = rec & 511;
            IqBest ba, bb;
            best_init(ba);
            best_init(bb);
            float apmax = 0.0f;
            cert_walk<NPOS>(lq, q0, n, ws2, sx2, [&](float ap, float lx, int c) {
                apmax = fmaxf(apmax, ap);
                best_take(ba, __fmaf_rn(sa, ap, -lx), c);
                best_take(bb, __fmaf_rn(sb, ap, -lx), c);
            });
            // both gaps above tau at both ends, i.e. gap * sc > (K u / 4) Q(sc) for each pair
            const float kqa = __fmul_rn(KU4, cert_q<Tr>(cs, sa, apmax)), kqb = __fmul_rn(KU4, cert_q<Tr>(cs, sb, apmax));
            const float ga = __fsub_rn(ba.m2, ba.m1), gb = __fsub_rn(bb.m2, bb.m1);
            const bool ok = ba.w == bb.w && cert_ok<Tr>(cs, sa, apmax) && cert_ok<Tr>(cs, sb, apmax) &&
                            __fmul_rn(ga, sa) > kqa && __fmul_rn(ga, sb) > kqb && __fmul_rn(gb, sa) > kqa &&
                            __fmul_rn(gb, sb) > kqb;
            if (ok) {
                const uint16_t v = (uint16_t)(__ldg(G.gidx + e0 + ba.w) | IQ_SEARCHED);
#pragma unroll
                for (int k = 0; k < IQ_RUN; k++)
                    if (k < len) W.win[g][(j0 + k) * NSUB + q] = v;
            }
            retry = !ok;
        }
        // the runs to score step by step, in the same (length) order
        const unsigned rb = __ballot_sync(IQ_FULL, retry);
        if (retry) W.rank[nretry + __popc(rb & ((1u << lane) - 1u))] = (uint8_t)p;
        nretry += __popc(rb);
    }
    __syncwarp();
    bool anyx = false;
    for (int pb = 0; pb < nretry; pb += 32) {
        const int i = pb + lane;
        if (i < nretry) {
            const int p = W.rank[i];
            const uint32_t rec = W.rec[p], tg = W.tag[p];
            const int g = tg & 31, q = (tg >> 5) & 7, j0 = (tg >> 8) & 31, len = ((tg >> 13) & 7) + 1;
            const uint4* lq = reinterpret_cast<const uint4*>(G.lvl) + (size_t)(rec >> 9) * NW;
            const IqLvlQuad<NW> q0 = lvl_quad<NW>(lq, 0);
            float sc[IQ_RUN];
#pragma unroll
            for (int k = 0; k < IQ_RUN; k++) sc[k] = iq_step_scale<Tr>(W, g, min(j0 + k, SW - 1), cw);  // past the run: unused
            float xs[NPOS], ws[NPOS], sx[NPOS];
            iq_load_sub<Tr>(W, g, q, xs, ws);
            const IqCertSub cs = cert_setup<NPOS>(xs, ws, sx);
            f32x2 ws2[NPOS / 2], sx2[NPOS / 2], sc2[IQ_RUN / 2];
#pragma unroll
            for (int k = 0; k < NPOS / 2; k++) {
                ws2[k] = f2_pack(ws[2 * k], ws[2 * k + 1]);
                sx2[k] = f2_pack(sx[2 * k], sx[2 * k + 1]);
            }
#pragma unroll
            for (int k = 0; k < IQ_RUN / 2; k++) sc2[k] = f2_pack(sc[2 * k], sc[2 * k + 1]);
            const uint32_t e0 = (rec >> 9) * 4;
            const int n = rec & 511;
            IqBest b[IQ_RUN];
#pragma unroll
            for (int k = 0; k < IQ_RUN; k++) best_init(b[k]);
            float apmax = 0.0f;
            cert_walk<NPOS>(lq, q0, n, ws2, sx2, [&](float ap, float lx, int c) {
                apmax = fmaxf(apmax, ap);
                const f32x2 ap2 = f2_pack(ap, ap), ml2 = f2_pack(-lx, -lx);
#pragma unroll
                for (int k = 0; k < IQ_RUN / 2; k++) {
                    float s0, s1;
                    f2_unpack(f2_fma(sc2[k], ap2, ml2), s0, s1);
                    best_take(b[2 * k], s0, c);
                    best_take(b[2 * k + 1], s1, c);
                }
            });
#pragma unroll
            for (int k = 0; k < IQ_RUN; k++) {
                if (k < len) {
                    const bool ok = cert_ok<Tr>(cs, sc[k], apmax) &&
                                    __fmul_rn(__fsub_rn(b[k].m2, b[k].m1), sc[k]) > __fmul_rn(KU4, cert_q<Tr>(cs, sc[k], apmax));
                    if (ok) {
                        W.win[g][(j0 + k) * NSUB + q] = (uint16_t)(__ldg(G.gidx + e0 + b[k].w) | IQ_SEARCHED);
                    } else {
                        atomicOr(&W.xflag[g], 1ull << ((j0 + k) * NSUB + q));
                        anyx = true;
                    }
                }
            }
        }
    }
    __syncwarp();
    return __any_sync(IQ_FULL, anyx);
}

// ---------------------------------------------------------------------------
// exact search (the reference's float distances)
// ---------------------------------------------------------------------------
// One distance term of the IQ2 term table: constant row R plus the lane's column byte and the
// level bits.
template <int R>
__device__ __forceinline__ float iq_term(const unsigned char* tb, uint32_t a) {
    return *reinterpret_cast<const float*>(tb + R * 256 + a);
}

// Weighted distance of the IQ2 code in the low (HI = false) or high half of w; lb is the
// lane's column byte. The terms are added in the reference's order, position 0 first.
template <bool HI>
__device__ __forceinline__ float iq2_dist(const unsigned char* tb, uint32_t w, uint32_t lb) {
    using R = IqRows8;
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
}

// Weighted distance of an IQ3 code (3 bits per position), term by term as the reference:
// t_j = (s_j (sc g_j - x_j)) (sc g_j - x_j), added position 0 first.
__device__ __forceinline__ float iq3_dist(uint32_t code, const float* xs, const float* ws, float sc) {
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const int l = (int)((code >> (3 * j)) & 7);
        const float g = __fadd_rn(__int_as_float(0x4B000001 + 2 * l), -8388608.0f);  // 2 l + 1
        const float df = __fsub_rn(__fmul_rn(sc, g), xs[j]);
        const float t = __fmul_rn(__fmul_rn(ws[j], df), df);
        s = j == 0 ? t : __fadd_rn(s, t);
    }
    return s;
}

// Solve the P queued exact searches, one per lane, longest lists first (window step
// numerators cw[]).
template <class Tr>
__device__ void iq_exact_flush(IqWarpSmem<Tr>& W, const IqGridDev& G, int lane, int P, const float* cw) {
    constexpr int NPOS = Tr::NPOS, NSUB = Tr::NSUB;
    iq_sort<Tr>(W, P, lane);
    extern __shared__ __align__(16) unsigned char smem[];
    const unsigned char* tb = smem;
    const uint32_t lb = (uint32_t)(threadIdx.x & (IQ_WARPS * 32 - 1)) * 4;  // this lane's column byte
    for (int pb = 0; pb < P; pb += 32) {
        const int i = pb + lane;
        if (i < P) {
            const int p = W.ord[i];
            const uint32_t rec = W.rec[p], e0 = (rec >> 9) * 4;
            const int n = rec & 511;
            const int tg = W.tag[p], g = tg & 31, slot = (tg >> 5) & 31, q = (tg >> 10) & 7;
            const uint2* lp = reinterpret_cast<const uint2*>(G.list + e0);  // quads of 4 codes
            uint2 nx = __ldg(lp);
            const float sc = slot == IQ_FINAL ? W.fsc[g] : iq_step_scale<Tr>(W, g, slot, cw);
            float xs[NPOS], ws[NPOS];
            iq_load_sub<Tr>(W, g, q, xs, ws);
            int bp = 0;  // list position of the first least distance
            if (NPOS == 4) {
                // the first candidate, then strict < over the rest; rolled, the codes of the
                // current quad shifting down by one per step, the next quad in flight
                const int nq4 = (n + 3) >> 2;
                uint2 cur = nx;
                if (nq4 > 1) nx = __ldg(lp + 1);
                float bd = 0.0f;
#pragma unroll 1
                for (int c = 0; c < n; c++) {
                    const float d2 = iq3_dist(cur.x & 0xFFFF, xs, ws, sc);
                    if (c == 0 || d2 < bd) { bd = d2; bp = c; }
                    if ((c & 3) == 3) {
                        cur = nx;
                        if ((c >> 2) + 2 < nq4) nx = __ldg(lp + (c >> 2) + 2);
                    } else {
                        cur.x = __funnelshift_r(cur.x, cur.y, 16);
                        cur.y >>= 16;
                    }
                }
            } else {
                using R = IqRows8;
                float sg[Tr::NLEV];
#pragma unroll
                for (int l = 0; l < Tr::NLEV; l++) sg[l] = __fmul_rn(sc, (float)(2 * l + 1));
                // the list's first quad is in flight while the terms are tabulated
                const uint2 v0 = nx;
                unsigned char* tw = smem + lb;
                auto put = [&](int row, float t) { *reinterpret_cast<float*>(tw + row * 256) = t; };
                // terms t_j(l) = (s_j * (sc g_l - x_j)) * (sc g_l - x_j)
                float t0[4], t1[4];
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const float xj = xs[j], wj = ws[j];
#pragma unroll
                    for (int l = 0; l < 4; l++) {
                        const float df = __fsub_rn(sg[l], xj);
                        const float t = __fmul_rn(__fmul_rn(wj, df), df);
                        if (j == 0) t0[l] = t;
                        else if (j == 1) t1[l] = t;
                        else put(R::row(j, l), t);
                    }
                }
#pragma unroll
                for (int l1 = 0; l1 < 4; l1++)
#pragma unroll
                    for (int l0 = 0; l0 < 4; l0++) put(l0 + 4 * l1, __fadd_rn(t0[l0], t1[l1]));
                // the first candidate, then strict < over the rest (the first of equal distances
                // wins; a padding copy of the last code never wins); quads are requested two
                // iterations ahead of their use
                float bd = 0.0f;
                auto take = [&](float d2, int c) {
                    if (c == 0 || d2 < bd) { bd = d2; bp = c; }
                };
                const int nq4 = (n + 3) >> 2;
                uint2 nx1 = nq4 > 1 ? __ldg(lp + 1) : v0, nx2 = nq4 > 2 ? __ldg(lp + 2) : v0, cur = v0;
#pragma unroll 1
                for (int c = 0; c < nq4; c++) {
                    take(iq2_dist<false>(tb, cur.x, lb), 4 * c);
                    take(iq2_dist<true>(tb, cur.x, lb), 4 * c + 1);
                    take(iq2_dist<false>(tb, cur.y, lb), 4 * c + 2);
                    take(iq2_dist<true>(tb, cur.y, lb), 4 * c + 3);
                    cur = nx1;
                    nx1 = nx2;
                    if (c + 3 < nq4) nx2 = __ldg(lp + c + 3);
                }
            }
            W.win[g][(slot == IQ_FINAL ? 0 : slot) * NSUB + q] = (uint16_t)(__ldg(G.gidx + e0 + bp) | IQ_SEARCHED);
        }
    }
    __syncwarp();
}

// Index of the tentative code of the subgroup with values xq at inverse scale inv into the nbr
// table (base 3 for IQ2: sweep levels are clamped to 0..2; the code itself for IQ3).
template <class Tr>
__device__ __forceinline__ int iq_index(const float* xq, float inv) {
    int idx = 0, mul = 1;
#pragma unroll
    for (int j = 0; j < Tr::NPOS; j++) {
        // clamp(rint(0.5 t), 0, MAXL), t = fl(inv x) - 1, without round or convert instructions (XU
        // pipe): 0.5 t is exact (|t| is 0 or at least 2^-24), so one fused multiply-add
        // 0.5 t + 1.5 * 2^23 rounds it to an integer in the low mantissa bits, ties to even as
        // rint; the clamps are taken on that float, and send NaN to level 0 as the float-to-int
        // conversion did
        const float t = __fadd_rn(__fmul_rn(inv, xq[j]), -1.0f);
        const float v = fminf(fmaxf(__fmaf_rn(t, 0.5f, 12582912.0f), 12582912.0f), 12582912.0f + (float)Tr::MAXL);
        const int l = __float_as_int(v) & 7;  // the low bits of 1.5 * 2^23 are zero
        if (Tr::BITS == 2) { idx += l * mul; mul *= 3; }
        else idx |= l << (3 * j);
    }
    return idx;
}

// grid values (2l+1) of the resolved grid indexes of one group -> q[GS]
template <class Tr>
__device__ __forceinline__ void iq_decode(const uint16_t* win, const uint16_t* kg, float* q) {
#pragma unroll
    for (int s = 0; s < Tr::NSUB; s++) {
        const int code = kg[win[s] & 0x7FFF];
#pragma unroll
        for (int j = 0; j < Tr::NPOS; j++)  // 2l + 1 as a float: the bits of 2^23 + 2l + 1, minus 2^23
            q[s * Tr::NPOS + j] = __fadd_rn(__int_as_float(0x4B000001 + 2 * ((code >> (Tr::BITS * j)) & (Tr::NLEV - 1))),
                                            -8388608.0f);
    }
}

template <class Tr>
__device__ __forceinline__ void iq_sums(const float* w, const float* wx, const float* q, float& sumqx, float& sumq2) {
    if constexpr (Tr::SUMK == SUM_TREE) {
        // on f32x2 pairs (v[k], v[k + H]), tree_sum2 keeping the adjacent-pair order. The grid
        // values are positive, so a product is zero only for a zero weight or value, and
        // f2_mul_z's +0 for -0 changes only an all-zero sum's sign: sumq2 <= 0 is rejected
        // either way, and sumqx == 0 is never accepted (best >= 0) and refits to a zero scale,
        // which neither flips the signs nor changes the 4-bit sub-scale
        constexpr int H = Tr::GS / 2;
        f32x2 a2[H], b2[H];
#pragma unroll
        for (int k = 0; k < H; k++) {
            const f32x2 q2 = f2_pack(q[k], q[k + H]);
            a2[k] = f2_mul_z(f2_pack(wx[k], wx[k + H]), q2);
            b2[k] = f2_mul_z(f2_mul_z(f2_pack(w[k], w[k + H]), q2), q2);
        }
        sumqx = tree_sum2<H>(a2);
        sumq2 = tree_sum2<H>(b2);
    } else {  // torch's `.sum(-1)` order (IQ2_XXS), scalar
        float a[Tr::GS], b[Tr::GS];
#pragma unroll
        for (int i = 0; i < Tr::GS; i++) {
            a[i] = wx[i] * q[i];  // (w x) q
            b[i] = (w[i] * q[i]) * q[i];
        }
        sumqx = torch_sum<Tr::GS>(a);
        sumq2 = torch_sum<Tr::GS>(b);
    }
}

template <int TYPE, bool IMAT>
__global__ void __maxnreg__(IqT<TYPE>::MAXREG) iq_kernel(QuantArgs a, IqGridDev G, IqParams prm) {
    using Tr = IqT<TYPE>;
    using WS = IqWarpSmem<Tr>;
    constexpr int GS = Tr::GS, NSUB = Tr::NSUB, NPOS = Tr::NPOS, SBG = QK_K / GS, SBW = 32 / SBG,
                  SBT = IQ_WARPS * SBW, BB = Tr::BB;
    constexpr int SW = Tr::SW;
    extern __shared__ __align__(16) unsigned char smem[];
    WS* wsm = reinterpret_cast<WS*>(smem + iq_tbl_bytes<Tr>());  // the IQ2 term table comes first
    float* s_c = reinterpret_cast<float*>(smem + iq_tbl_bytes<Tr>() + IQ_WARPS * sizeof(WS));
    float* s_qp = s_c + 32;
    uint16_t* s_kg = reinterpret_cast<uint16_t*>(s_qp + 32);
    uint8_t* s_out = reinterpret_cast<uint8_t*>(s_kg) + iq_kg_bytes<Tr>();

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    WS& W = wsm[warp];
    if (tid < 32) s_c[tid] = prm.c[tid];
    if (tid < 8) s_qp[tid] = prm.qp[tid];
    for (int i = tid; i < Tr::GRID; i += blockDim.x) s_kg[i] = __ldg(G.kgrid + i);
    __syncthreads();

    const int sbl = lane / SBG, gl = lane % SBG;  // superblock within the warp, group within it
    for (int64_t tile = blockIdx.x; tile * SBT < a.nblk; tile += gridDim.x) {
        const int64_t b = min(tile * SBT + warp * SBW + sbl, a.nblk - 1);
        float x[GS], w[GS], xval[GS];
        load_row<GS>(a.src, b * QK_K + gl * GS, a.src_type, x);

        // weights (iq2.py:429-431, iq2_xs.py:27-29, iq2_s.py:28-30, iq3_xxs.py:40-45)
        if (IMAT) {
            float* sq = &W.xv[0][0] + sbl * QK_K;  // xv is written only after the weights
            if constexpr (GS == 32) {
                sb_put_sq32(sq, gl, x);
                __syncwarp();
                W.part[sbl][gl] = sb_sum256_partial32(sq, gl);
            } else {
                sb_put_sq16(sq, gl, x);
                __syncwarp();
                if (gl < 8) W.part[sbl][gl] = sb_sum256_partial16(sq, gl);
            }
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
        float wx[GS];  // w x, the first product of each sumqx term
#pragma unroll
        for (int i = 0; i < GS; i++) wx[i] = w[i] * xval[i];
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
        uint16_t cur[NSUB];
        const uint16_t cur0 = Tr::RP == RP_ALL_REDO ? IQ_SEARCHED : 0;  // grid index 0; og_init: IQ3_S starts off-grid
#pragma unroll
        for (int s = 0; s < NSUB; s++) cur[s] = cur0;
        __syncwarp();

        // the sweep over the candidate scales, SW steps per window; the pass after the last
        // window is the final reprojection at the accepted scale
        bool redo = false;
        for (int s0 = 0;; s0 += SW) {
            const bool final_pass = s0 >= Tr::NSTEP;
            const int nw = final_pass ? 0 : min(SW, Tr::NSTEP - s0);
            bool anyx = false;
            if (!final_pass) {
                W.xflag[lane] = 0ull;
                W.rg[lane] = r;
                if (SW <= 8) {
#pragma unroll
                    for (int j = 0; j < (SW <= 8 ? SW : 1); j++) W.psc[lane][j] = rcp_rn(r * s_c[s0 + min(j, nw - 1)]);
                }
                __syncwarp();
                // jobs: per subgroup, the runs of equal off-grid codes within the window, split
                // every 8 steps; the queue is solved when the next subgroup's jobs would not fit,
                // and after the last
                int nq = 0, q = 0;
                for (;;) {
#pragma unroll 1
                    for (; q < NSUB; q++) {
                        float xq[NPOS];
#pragma unroll
                        for (int j = 0; j < NPOS; j += 4) {
                            const float4 f4 = *reinterpret_cast<const float4*>(&W.xv[lane][q * NPOS + j]);
                            xq[j] = f4.x; xq[j + 1] = f4.y; xq[j + 2] = f4.z; xq[j + 3] = f4.w;
                        }
                        uint32_t v[SW];
#pragma unroll
                        for (int j = 0; j < SW; j++)
                            v[j] = j < nw ? __ldg(G.nbr + iq_index<Tr>(xq, r * s_c[s0 + j])) : IQ_ONGRID;
                        // step j continues the job of step j - 1 when both are off the grid with the
                        // same code and no cut falls between them (that job has 8 steps, or with
                        // CUT8 j is a multiple of 8); a job's last step is one the next step does
                        // not continue
                        auto runs = [&](auto&& at) {
                            int run = 0;
#pragma unroll
                            for (int j = 0; j < SW; j++) {
                                const bool off = !(v[j] >> 31);
                                const bool cut = Tr::CUT8 ? j % IQ_RUN == 0 : run >= IQ_RUN;
                                run = off ? (j > 0 && run > 0 && !cut && v[j] == v[j > 0 ? j - 1 : 0] ? run + 1 : 1) : 0;
                                const bool cutn = Tr::CUT8 ? (j + 1) % IQ_RUN == 0 : run >= IQ_RUN;
                                const bool next = j + 1 < SW && run > 0 && !cutn && v[j + 1 < SW ? j + 1 : j] == v[j];
                                at(j, off, off && !next, run);
                            }
                        };
                        unsigned njobs = 0;
                        runs([&](int j, bool off, bool last, int run) {
                            njobs += last;
                            if (!off && j < nw) W.win[lane][j * NSUB + q] = (uint16_t)(v[j] & 0x7FFF);
                        });
                        if (nq + (int)__reduce_add_sync(IQ_FULL, njobs) > IQ_CAP) break;
                        runs([&](int j, bool, bool last, int run) {
                            iq_push(W, nq, lane, last, v[j],
                                    (uint32_t)lane | (uint32_t)q << 5 | (uint32_t)(j - run + 1) << 8 | (uint32_t)(run - 1) << 13);
                        });
                    }
                    __syncwarp();
                    if (nq > 0) anyx |= iq_job_flush<Tr>(W, G, lane, nq, s_c + s0);
                    nq = 0;
                    if (q >= NSUB) break;
                }
            }

            // exact searches: the steps no certificate covered, or the final reprojection
            unsigned long long xm = anyx ? W.xflag[lane] : 0ull;
            bool fin_todo = final_pass;
            while (fin_todo || __any_sync(IQ_FULL, xm != 0ull)) {
                int nq = 0;
                if (fin_todo) {
                    bool anyoff = false, allon = true;
#pragma unroll
                    for (int q = 0; q < NSUB; q++) {
                        anyoff |= (cur[q] & IQ_SEARCHED) != 0;
                        allon &= (cur[q] & IQ_SEARCHED) == 0;
                    }
                    float finv;
                    if (Tr::RP == RP_ALL_PROJ) {
                        redo = active && scale > 0.0f;
                        finv = rcp_rn(redo ? scale : 1.0f);
                    } else if (Tr::RP == RP_OFFGRID_NEED) {
                        redo = active && scale > 0.0f && !allon;
                        finv = rcp_rn(scale > 0.0f ? scale : 1.0f);
                    } else {
                        redo = active && anyoff && scale > 0.0f;
                        finv = rcp_rn(redo ? scale : 1.0f);
                    }
                    W.fsc[lane] = scale;
#pragma unroll
                    for (int q = 0; q < NSUB; q++) {
                        const bool want = redo && (Tr::RP == RP_ALL_PROJ || Tr::RP == RP_ALL_REDO || (cur[q] & IQ_SEARCHED));
                        // not reprojected: keep the current grid index (read back below without its flag)
                        float xq[NPOS];
#pragma unroll
                        for (int t = 0; t < NPOS; t += 4) {
                            const float4 f4 = *reinterpret_cast<const float4*>(&W.xv[lane][q * NPOS + t]);
                            xq[t] = f4.x; xq[t + 1] = f4.y; xq[t + 2] = f4.z; xq[t + 3] = f4.w;
                        }
                        const uint32_t v = want ? __ldg(G.nbr + iq_index<Tr>(xq, finv))
                                                : IQ_ONGRID | (uint32_t)(cur[q] & 0x7FFF);
                        if (v >> 31) W.win[lane][q] = (uint16_t)(v & 0x7FFF);
                        iq_push(W, nq, lane, !(v >> 31), v, (uint32_t)lane | (uint32_t)IQ_FINAL << 5 | (uint32_t)q << 10);
                    }
                    fin_todo = false;
                } else {
                    // up to 8 of this lane's flagged steps per pass
#pragma unroll 1
                    for (int k = 0; k < 8; k++) {
                        const bool has = xm != 0ull;
                        const int bit = has ? __ffsll((long long)xm) - 1 : 0;
                        xm &= xm - 1ull;
                        const int j = bit / NSUB, qq = bit % NSUB;
                        uint32_t v = 0;
                        if (has) {
                            float xq[NPOS];
#pragma unroll
                            for (int t = 0; t < NPOS; t += 4) {
                                const float4 f = *reinterpret_cast<const float4*>(&W.xv[lane][qq * NPOS + t]);
                                xq[t] = f.x; xq[t + 1] = f.y; xq[t + 2] = f.z; xq[t + 3] = f.w;
                            }
                            v = __ldg(G.nbr + iq_index<Tr>(xq, r * s_c[s0 + j]));
                        }
                        iq_push(W, nq, lane, has, v, (uint32_t)lane | (uint32_t)j << 5 | (uint32_t)qq << 10);
                    }
                }
                __syncwarp();
                iq_exact_flush<Tr>(W, G, lane, nq, s_c + s0);
            }
            if (final_pass) break;

            // the accept chain over the window's steps
            for (int j = 0; j < nw; j++) {
                float qv[GS], sumqx, sumq2;
                iq_decode<Tr>(&W.win[lane][j * NSUB], s_kg, qv);
                iq_sums<Tr>(w, wx, qv, sumqx, sumq2);
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
        uint16_t fin[NSUB];
#pragma unroll
        for (int q = 0; q < NSUB; q++) fin[q] = W.win[lane][q] & 0x7FFF;
        {
            float qv[GS], sumqx, sumq2;
            iq_decode<Tr>(fin, s_kg, qv);
            iq_sums<Tr>(w, wx, qv, sumqx, sumq2);
            if (redo && sumq2 > 0.0f) scale = __fdiv_rn(sumqx, sumq2 < F32_TINY ? F32_TINY : sumq2);
        }
        if (!redo) {
#pragma unroll
            for (int q = 0; q < NSUB; q++) fin[q] = cur[q] & 0x7FFF;
        }
        // fin holds grid indexes
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
