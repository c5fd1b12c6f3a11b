// Periodic cell-list neighbour build on the device.
//
// Pair-set contract: every (i, j, S) with |R_j + S.cell - R_i| < max(rc_radial, rc_angular),
// excluding (i, i, 0) — the ASE neighbor_list("ijS") semantics used by the reference
// BatchBuilder (rune/mobius/interface/batch.py:42-102) and the training builder
// (rune/datasets/neighbor.py:36-134). Membership is decided in float64 from the caller's
// positions; the stored edge vector is then formed in float32 exactly as the reference model
// does (positions and S.cell cast to float32, r = (R_j + off) - R_i; descriptor.py:813-817).
//
// Layout: edges are grouped by centre atom (CSR, row_ptr), each row holding the edges inside
// the smaller cutoff first, so the radial and angular lists share one array: the list with the
// larger cutoff is the whole row, the other one its prefix.
//
// Binning: per structure, bins along each periodic axis = floor(thickness / rc) (>= 1); the
// stencil reaches ceil(rc / bin thickness) bins, wrapping with an integer image shift, so cells
// thinner than the cutoff produce every periodic image (the small-box case of
// rune/mobius/src/mobius.cu:170-201). A non-periodic axis has one bin and no images.
// Bin contents are sorted by atom index, so the edge order is deterministic.

#include <cub/cub.cuh>

#include "engine.cuh"

namespace rune {

namespace {

__device__ __forceinline__ int floordiv(int a, int b) {
    int q = a / b;
    if ((a % b != 0) && ((a < 0) != (b < 0))) --q;
    return q;
}

// Bin every atom; record its structure, integer wrap (floor of the fractional coordinate on
// periodic axes, so that shifts refer to the caller's unwrapped positions) and bin.
__global__ void k_bin_atoms(int n_atoms, int n_types, int n_structures,
                            const int* __restrict__ atom_ptr, const double* __restrict__ pos,
                            const int* __restrict__ types, const StructGeom* __restrict__ geom,
                            int* __restrict__ tsafe, int* __restrict__ sid_out, int4* __restrict__ binc,
                            int4* __restrict__ wrap, int* __restrict__ bin_count,
                            unsigned int* __restrict__ flags) {
    int a = blockIdx.x * blockDim.x + threadIdx.x;
    if (a >= n_atoms) return;
    int lo = 0, hi = n_structures - 1;
    while (lo < hi) {  // last structure whose first atom <= a
        int mid = (lo + hi + 1) >> 1;
        if (atom_ptr[mid] <= a) lo = mid; else hi = mid - 1;
    }
    sid_out[a] = lo;
    const StructGeom& g = geom[lo];
    double p[3] = {pos[3 * a], pos[3 * a + 1], pos[3 * a + 2]};
    int t = types[a];
    if (t < 0 || t >= n_types) {
        atomicOr(flags, 1u);
        t = 0;  // keep every table read in bounds; the call reports the error at its end
    }
    tsafe[a] = t;
    int b[3], w[3];
    bool finite = isfinite(p[0]) && isfinite(p[1]) && isfinite(p[2]);
    if (!finite) atomicOr(flags, 2u);
    for (int k = 0; k < 3; ++k) {
        double f = p[0] * g.inv[0 * 3 + k] + p[1] * g.inv[1 * 3 + k] + p[2] * g.inv[2 * 3 + k];
        if (!finite) f = 0.0;
        if (g.pbc[k]) {
            double fl = floor(f);
            if (fabs(fl) > 1.0e5) { atomicOr(flags, 2u); fl = 0.0; }
            w[k] = (int)fl;
            double fw = f - fl;
            int bk = (int)(fw * g.nb[k]);
            b[k] = min(max(bk, 0), g.nb[k] - 1);
        } else {
            w[k] = 0;
            b[k] = 0;
        }
    }
    int bin = g.bin_offset + (b[0] * g.nb[1] + b[1]) * g.nb[2] + b[2];
    binc[a] = make_int4(b[0], b[1], b[2], bin);
    wrap[a] = make_int4(w[0], w[1], w[2], 0);
    atomicAdd(&bin_count[bin], 1);
}

__global__ void k_fill_bins(int n_atoms, const int4* __restrict__ binc,
                            const int* __restrict__ bin_start, int* __restrict__ bin_fill,
                            int* __restrict__ bin_atoms) {
    int a = blockIdx.x * blockDim.x + threadIdx.x;
    if (a >= n_atoms) return;
    int bin = binc[a].w;
    int slot = atomicAdd(&bin_fill[bin], 1);
    bin_atoms[bin_start[bin] + slot] = a;
}

// Candidate record in bin order: float64 position and the packed integer wrap.
__device__ __forceinline__ double pack_wrap(int4 w) {
    unsigned long long u = ((unsigned long long)(w.x & 0x1fffff)) |
                           ((unsigned long long)(w.y & 0x1fffff) << 21) |
                           ((unsigned long long)(w.z & 0x1fffff) << 42);
    return __longlong_as_double((long long)u);
}
__device__ __forceinline__ int3 unpack_wrap(double d) {
    unsigned long long u = (unsigned long long)__double_as_longlong(d);
    auto ext = [](unsigned long long v) { int x = (int)(v & 0x1fffff); return x >= (1 << 20) ? x - (1 << 21) : x; };
    return make_int3(ext(u), ext(u >> 21), ext(u >> 42));
}

// Sort each bin's atom list ascending (rank sort; atom indices are unique), warp per bin, and
// write the bin-ordered candidate arrays (atom index; position and wrap).
__global__ void k_sort_bins(int n_bins, const int* __restrict__ bin_start,
                            const int* __restrict__ bin_count, const int* __restrict__ unsorted,
                            const double* __restrict__ pos, const int4* __restrict__ wrap,
                            int* __restrict__ batom, double4* __restrict__ bpos) {
    int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (warp >= n_bins) return;
    int start = bin_start[warp], n = bin_count[warp];
    for (int base = 0; base < n; base += 32) {
        int k = base + lane;
        int v = k < n ? unsorted[start + k] : 0;
        int rank = 0;
        for (int m = 0; m < n; ++m) rank += unsorted[start + m] < v;
        if (k < n) {
            batom[start + rank] = v;
            bpos[start + rank] = make_double4(pos[3 * v], pos[3 * v + 1], pos[3 * v + 2],
                                              pack_wrap(wrap[v]));
        }
    }
}

struct Traverse {
    const StructGeom* geom;
    const double* pos;
    const int4* binc;
    const int4* wrap;
    const int* sid;
    const int* bin_start;
    const int* batom;
    const double4* bpos;
    double rc_max2, rc_min2;
};

// Visit every candidate j of atom i in a fixed order; `visit(j, S, d, d^2, valid)` is called by
// all 32 lanes once per round (valid = this lane holds a candidate inside rc_max). Along z the
// bins of one image are consecutive, so their candidates form one contiguous range.
template <typename Visit>
__device__ __forceinline__ void traverse(const Traverse& tv, int i, int lane, Visit&& visit) {
    const StructGeom& g = tv.geom[tv.sid[i]];
    int4 bc = tv.binc[i];
    int4 wi = tv.wrap[i];
    double pi0 = tv.pos[3 * i], pi1 = tv.pos[3 * i + 1], pi2 = tv.pos[3 * i + 2];
    for (int dx = -g.reach[0]; dx <= g.reach[0]; ++dx) {
        int tx = bc.x + dx, ix = 0;
        if (g.pbc[0]) { ix = floordiv(tx, g.nb[0]); tx -= ix * g.nb[0]; }
        else if (tx < 0 || tx >= g.nb[0]) continue;
        for (int dy = -g.reach[1]; dy <= g.reach[1]; ++dy) {
            int ty = bc.y + dy, iy = 0;
            if (g.pbc[1]) { iy = floordiv(ty, g.nb[1]); ty -= iy * g.nb[1]; }
            else if (ty < 0 || ty >= g.nb[1]) continue;
            int column = g.bin_offset + (tx * g.nb[1] + ty) * g.nb[2];
            int z = bc.z - g.reach[2], zend = bc.z + g.reach[2];
            while (z <= zend) {
                int iz = 0, tz0, seg_end;
                if (g.pbc[2]) {
                    iz = floordiv(z, g.nb[2]);
                    tz0 = z - iz * g.nb[2];
                    seg_end = min(zend, (iz + 1) * g.nb[2] - 1);
                } else {
                    tz0 = z;
                    seg_end = zend;
                    if (z < 0) { z = 0; continue; }
                    if (z >= g.nb[2]) break;
                    seg_end = min(seg_end, g.nb[2] - 1);
                }
                int tz1 = tz0 + (seg_end - z);
                int a0 = tv.bin_start[column + tz0], a1 = tv.bin_start[column + tz1 + 1];
                for (int base = a0; base < a1; base += 32) {
                    int k = base + lane;
                    bool valid = k < a1;
                    int j = 0;
                    double4 pj = make_double4(pi0, pi1, pi2, 0.0);
                    if (valid) {
                        j = tv.batom[k];
                        pj = tv.bpos[k];
                    }
                    int3 wj = unpack_wrap(pj.w);
                    int s0 = g.pbc[0] ? ix - wj.x + wi.x : 0;
                    int s1 = g.pbc[1] ? iy - wj.y + wi.y : 0;
                    int s2 = g.pbc[2] ? iz - wj.z + wi.z : 0;
                    // (R_j - R_i) + S.cell: exactly antisymmetric under i <-> j, S -> -S
                    double d0 = (pj.x - pi0) + (s0 * g.cell[0] + s1 * g.cell[3] + s2 * g.cell[6]);
                    double d1 = (pj.y - pi1) + (s0 * g.cell[1] + s1 * g.cell[4] + s2 * g.cell[7]);
                    double d2v = (pj.z - pi2) + (s0 * g.cell[2] + s1 * g.cell[5] + s2 * g.cell[8]);
                    double r2 = d0 * d0 + d1 * d1 + d2v * d2v;
                    valid = valid && r2 < tv.rc_max2 && !(j == i && s0 == 0 && s1 == 0 && s2 == 0);
                    visit(j, s0, s1, s2, d0, d1, d2v, r2, valid);
                }
                z = seg_end + 1;
            }
        }
    }
}

// Per-atom counts (inside the smaller cutoff, total) plus, per block, the largest radial and
// angular counts (packed count << 32 | ~atom, so the first atom wins) and their sums.
__global__ void k_nbr_count(int n_atoms, Traverse tv, bool radial_is_full,
                            int* __restrict__ cnt_short, int* __restrict__ cnt_total,
                            unsigned long long* __restrict__ summary) {
    __shared__ unsigned long long red[4][8];
    int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int ns = 0, nt = 0;
    if (i < n_atoms) {
        traverse(tv, i, lane, [&](int, int, int, int, double, double, double, double r2,
                                  bool valid) {
            unsigned m_all = __ballot_sync(0xffffffffu, valid);
            unsigned m_short = __ballot_sync(0xffffffffu, valid && r2 < tv.rc_min2);
            nt += __popc(m_all);
            ns += __popc(m_short);
        });
        if (lane == 0) {
            cnt_short[i] = ns;
            cnt_total[i] = nt;
        }
    }
    if (lane == 0) {
        int nr = radial_is_full ? nt : ns, na = radial_is_full ? ns : nt;
        unsigned long long inv = i < n_atoms ? 0xffffffffull - (unsigned long long)i : 0ull;
        red[0][warp] = i < n_atoms ? ((unsigned long long)nr << 32) | inv : 0ull;
        red[1][warp] = i < n_atoms ? ((unsigned long long)na << 32) | inv : 0ull;
        red[2][warp] = i < n_atoms ? (unsigned long long)nr : 0ull;
        red[3][warp] = i < n_atoms ? (unsigned long long)na : 0ull;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int nw = blockDim.x >> 5;
        unsigned long long m0 = 0, m1 = 0, s0 = 0, s1 = 0;
        for (int w = 0; w < nw; ++w) {
            m0 = max(m0, red[0][w]);
            m1 = max(m1, red[1][w]);
            s0 += red[2][w];
            s1 += red[3][w];
        }
        atomicMax(&summary[0], m0);
        atomicMax(&summary[1], m1);
        atomicAdd(&summary[2], s0);
        atomicAdd(&summary[3], s1);
    }
}

__global__ void k_nbr_fill(int n_atoms, Traverse tv, const int* __restrict__ row_ptr,
                           const int* __restrict__ cnt_short, long long capacity,
                           float4* __restrict__ edges, int* __restrict__ shifts,
                           unsigned int* __restrict__ flags) {
    int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (i >= n_atoms) return;
    int base_s = row_ptr[i];
    int base_l = row_ptr[i] + cnt_short[i];
    if ((long long)row_ptr[i + 1] > capacity) {  // the edge buffer is too small: rerun
        if (lane == 0) atomicOr(flags, 16u);
        return;
    }
    unsigned lt = (1u << lane) - 1u;
    traverse(tv, i, lane, [&](int j, int s0, int s1, int s2, double d0, double d1, double d2,
                              double r2, bool valid) {
        bool is_short = valid && r2 < tv.rc_min2;
        bool is_long = valid && !is_short;
        unsigned ms = __ballot_sync(0xffffffffu, is_short);
        unsigned ml = __ballot_sync(0xffffffffu, is_long);
        if (valid) {
            int slot = is_short ? base_s + __popc(ms & lt) : base_l + __popc(ml & lt);
            // the float64 pair vector rounded once to float32: its error is relative to |r|,
            // not to the magnitude of the absolute positions
            edges[slot] = make_float4((float)d0, (float)d1, (float)d2, __int_as_float(j));
            shifts[slot] = (s0 & 1023) | ((s1 & 1023) << 10) | ((s2 & 1023) << 20);
        }
        base_s += __popc(ms);
        base_l += __popc(ml);
    });
}

// After an edge-buffer overflow nothing may read past the buffer: empty every row. The call is
// then repeated with a larger buffer.
__global__ void k_guard_rows(int n_atoms, const unsigned int* __restrict__ flags,
                             int* __restrict__ cnt_a, int* __restrict__ cnt_b) {
    if (!(*flags & 16u)) return;
    for (int a = blockIdx.x * blockDim.x + threadIdx.x; a < n_atoms; a += gridDim.x * blockDim.x) {
        cnt_a[a] = 0;
        cnt_b[a] = 0;
    }
}

// Padded reference rows -> CSR. Entries equal to -1 are skipped wherever they sit in a row.
__global__ void k_padded_count(int n_atoms, int width, const int64_t* __restrict__ nbr,
                               int n_atoms_check, const int* __restrict__ types, int n_types,
                               int* __restrict__ cnt, unsigned int* __restrict__ flags) {
    int a = blockIdx.x * blockDim.x + threadIdx.x;
    if (a >= n_atoms) return;
    if (types[a] < 0 || types[a] >= n_types) atomicOr(flags, 1u);
    int c = 0;
    for (int k = 0; k < width; ++k) {
        int64_t j = nbr[(int64_t)a * width + k];
        if (j == -1) continue;
        if (j < 0 || j >= n_atoms_check) atomicOr(flags, 4u);
        ++c;
    }
    cnt[a] = c;
}

__global__ void k_padded_fill(int n_atoms, int width, const int64_t* __restrict__ nbr,
                              const float* __restrict__ off, const float* __restrict__ pos,
                              const int* __restrict__ row_ptr, float4* __restrict__ edges) {
    int a = blockIdx.x * blockDim.x + threadIdx.x;
    if (a >= n_atoms) return;
    int o = row_ptr[a];
    for (int k = 0; k < width; ++k) {
        int64_t jj = nbr[(int64_t)a * width + k];
        if (jj < 0 || jj >= n_atoms) continue;
        int j = (int)jj;
        const float* of = off + ((int64_t)a * width + k) * 3;
        // (R_j - R_i) + off formed exactly in float64 from the float32 inputs, rounded once, so
        // the error is relative to |r| (the reference's float32 (R_j + off) - R_i rounds at |R|)
        float r0 = (float)(((double)pos[3 * j] - (double)pos[3 * a]) + (double)of[0]);
        float r1 = (float)(((double)pos[3 * j + 1] - (double)pos[3 * a + 1]) + (double)of[1]);
        float r2 = (float)(((double)pos[3 * j + 2] - (double)pos[3 * a + 2]) + (double)of[2]);
        edges[o++] = make_float4(r0, r1, r2, __int_as_float(j));
    }
}

// Reverse-edge index: for edge e = (i -> j, r) find (j -> i, ~-r) in row j. Distinct periodic
// images of one atom differ by a lattice vector, so a 1e-4 A match is unambiguous.
__global__ void k_rev_index(int n_atoms, EdgeList L, int* __restrict__ rev,
                            unsigned int* __restrict__ flags) {
    int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (i >= n_atoms) return;
    int b = L.row_ptr[i], n = L.cnt[i];
    for (int k = lane; k < n; k += 32) {
        float4 e = L.e[b + k];
        int j = edge_j(e);
        int bj = L.row_ptr[j], nj = L.cnt[j];
        int found = -1;
        for (int m = 0; m < nj; ++m) {
            float4 f = L.e[bj + m];
            if (edge_j(f) != i) continue;
            float x = e.x + f.x, y = e.y + f.y, z = e.z + f.z;
            if (x * x + y * y + z * z < 1.0e-8f) { found = bj + m; break; }
        }
        if (found < 0) atomicOr(flags, 8u);
        rev[b + k] = found < 0 ? b + k : found;
    }
}

inline int blocks_for(long long n, int per) { return (int)((n + per - 1) / per); }

}  // namespace

// ----------------------------------------------------------------------------- host side
static void structure_geometry(const double* cells, const uint8_t* pbc, int n_structures,
                               double rc, std::vector<StructGeom>& out, int& total_bins) {
    out.resize(n_structures);
    total_bins = 0;
    for (int s = 0; s < n_structures; ++s) {
        StructGeom& g = out[s];
        const double* c = cells + 9 * s;
        bool any = pbc[3 * s] || pbc[3 * s + 1] || pbc[3 * s + 2];
        double m[9];
        for (int k = 0; k < 9; ++k) m[k] = c[k];
        double det = m[0] * (m[4] * m[8] - m[5] * m[7]) - m[1] * (m[3] * m[8] - m[5] * m[6]) +
                     m[2] * (m[3] * m[7] - m[4] * m[6]);
        if (!any && std::fabs(det) < 1e-12) {
            for (int k = 0; k < 9; ++k) m[k] = (k % 4 == 0) ? 1.0 : 0.0;
            det = 1.0;
        }
        if (std::fabs(det) < 1e-12)
            throw Error(RUNE_ERR_INVALID,
                        "Degenerate cell is not supported for periodic neighbor construction.");
        for (int k = 0; k < 9; ++k) g.cell[k] = m[k];
        // inverse (frac = pos @ inv)
        double id = 1.0 / det;
        g.inv[0] = (m[4] * m[8] - m[5] * m[7]) * id;
        g.inv[1] = (m[2] * m[7] - m[1] * m[8]) * id;
        g.inv[2] = (m[1] * m[5] - m[2] * m[4]) * id;
        g.inv[3] = (m[5] * m[6] - m[3] * m[8]) * id;
        g.inv[4] = (m[0] * m[8] - m[2] * m[6]) * id;
        g.inv[5] = (m[2] * m[3] - m[0] * m[5]) * id;
        g.inv[6] = (m[3] * m[7] - m[4] * m[6]) * id;
        g.inv[7] = (m[1] * m[6] - m[0] * m[7]) * id;
        g.inv[8] = (m[0] * m[4] - m[1] * m[3]) * id;
        // plane spacings: volume / |b x c| etc.
        auto cross_norm = [&](int u, int v) {
            double x = m[3 * u + 1] * m[3 * v + 2] - m[3 * u + 2] * m[3 * v + 1];
            double y = m[3 * u + 2] * m[3 * v + 0] - m[3 * u + 0] * m[3 * v + 2];
            double z = m[3 * u + 0] * m[3 * v + 1] - m[3 * u + 1] * m[3 * v + 0];
            return std::sqrt(x * x + y * y + z * z);
        };
        double vol = std::fabs(det);
        double h[3] = {vol / cross_norm(1, 2), vol / cross_norm(2, 0), vol / cross_norm(0, 1)};
        int bins = 1;
        for (int k = 0; k < 3; ++k) {
            g.pbc[k] = pbc[3 * s + k] ? 1 : 0;
            if (g.pbc[k]) {
                long long nb = (long long)std::floor(h[k] / rc);
                nb = std::max(1LL, std::min(nb, 1024LL));
                g.nb[k] = (int)nb;
                g.reach[k] = (int)std::ceil(rc * nb / h[k] - 1e-12);
                if (g.reach[k] < 1) g.reach[k] = 1;
                if (g.reach[k] > 400)
                    throw Error(RUNE_ERR_INVALID, "Periodic cell is too thin for the cutoff.");
            } else {
                g.nb[k] = 1;
                g.reach[k] = 0;
            }
            bins *= g.nb[k];
        }
        g.bin_offset = total_bins;
        total_bins += bins;
    }
}

template <typename T>
static void exclusive_scan(Engine& eng, const T* in, T* out, int n, cudaStream_t stream) {
    size_t bytes = 0;
    RUNE_CUDA_TRY(cub::DeviceScan::ExclusiveSum(nullptr, bytes, in, out, n, stream));
    void* tmp = eng.ws.take(bytes + 256);
    KernelScope ks("cub_exclusive_scan", stream, 2);
    RUNE_CUDA_TRY(cub::DeviceScan::ExclusiveSum(tmp, bytes, in, out, n, stream));
}

void build_neighbors(Engine& eng, const BatchInput& in, NeighborData& nd, cudaStream_t stream) {
    const rune_model_config& cfg = eng.cfg;
    int n = in.n_atoms;
    double rc_max = std::max(cfg.rc_radial, cfg.rc_angular);
    double rc_min = std::min(cfg.rc_radial, cfg.rc_angular);
    std::vector<StructGeom> geom;
    int total_bins = 0;
    structure_geometry(in.cells, in.pbc, in.n_structures, rc_max, geom, total_bins);

    StructGeom* d_geom = eng.ws.take_n<StructGeom>(geom.size());
    eng.upload(d_geom, geom.data(), sizeof(StructGeom) * geom.size(), stream);
    int* d_atom_ptr = eng.ws.take_n<int>(in.n_structures + 1);
    eng.upload(d_atom_ptr, in.atom_ptr, sizeof(int) * (in.n_structures + 1), stream);
    int* sid = eng.ws.take_n<int>(n);
    int* tsafe = eng.ws.take_n<int>(n);
    int4* binc = eng.ws.take_n<int4>(n);
    int4* wrap = eng.ws.take_n<int4>(n);
    int* bin_count = eng.ws.take_n<int>(total_bins + 1);
    int* bin_start = eng.ws.take_n<int>(total_bins + 1);
    int* bin_fill = eng.ws.take_n<int>(total_bins + 1);
    int* bin_tmp = eng.ws.take_n<int>(n);
    int* batom = eng.ws.take_n<int>(n);
    double4* bpos = eng.ws.take_n<double4>(n);
    int* cnt_short = eng.ws.take_n<int>(n + 1);
    int* cnt_total = eng.ws.take_n<int>(n + 1);
    int* row_ptr = eng.ws.take_n<int>(n + 1);
    unsigned long long* summary = eng.ws.take_n<unsigned long long>(4);
    long long capacity = eng.edge_capacity > 0 ? eng.edge_capacity : (long long)n * 64 + 1024;
    float4* edges = eng.ws.take_n<float4>((size_t)capacity);
    int* shifts = eng.ws.take_n<int>((size_t)capacity);
    RUNE_CUDA_TRY(cudaMemsetAsync(bin_count, 0, sizeof(int) * (total_bins + 1), stream));
    RUNE_CUDA_TRY(cudaMemsetAsync(bin_fill, 0, sizeof(int) * (total_bins + 1), stream));
    RUNE_CUDA_TRY(cudaMemsetAsync(summary, 0, sizeof(unsigned long long) * 4, stream));
    RUNE_CUDA_TRY(cudaMemsetAsync(cnt_total + n, 0, sizeof(int), stream));

    const int tpb = 256;
    if (n > 0) {
        RUNE_KERNEL("k_bin_atoms", stream,
                    k_bin_atoms<<<blocks_for(n, tpb), tpb, 0, stream>>>(
                        n, cfg.n_types, in.n_structures, d_atom_ptr, in.positions, in.types,
                        d_geom, tsafe, sid, binc, wrap, bin_count, eng.d_flags));
        RUNE_LAUNCH_CHECK();
    }
    exclusive_scan(eng, bin_count, bin_start, total_bins + 1, stream);
    if (n > 0) {
        RUNE_KERNEL("k_fill_bins", stream,
                    k_fill_bins<<<blocks_for(n, tpb), tpb, 0, stream>>>(n, binc, bin_start,
                                                                          bin_fill, bin_tmp));
        RUNE_KERNEL("k_sort_bins", stream,
                    k_sort_bins<<<blocks_for((long long)total_bins * 32, tpb), tpb, 0, stream>>>(
                        total_bins, bin_start, bin_count, bin_tmp, in.positions, wrap, batom,
                        bpos));
        RUNE_LAUNCH_CHECK();
    }
    Traverse tv{d_geom, in.positions, binc, wrap, sid, bin_start, batom, bpos,
                rc_max * rc_max, rc_min * rc_min};
    bool radial_is_full = cfg.rc_radial >= cfg.rc_angular;
    if (n > 0) {
        RUNE_KERNEL("k_nbr_count", stream,
                    k_nbr_count<<<blocks_for((long long)n * 32, tpb), tpb, 0, stream>>>(
                        n, tv, radial_is_full, cnt_short, cnt_total, summary));
        RUNE_LAUNCH_CHECK();
    }
    exclusive_scan(eng, cnt_total, row_ptr, n + 1, stream);
    const int* cnt_r = radial_is_full ? cnt_total : cnt_short;
    const int* cnt_a = radial_is_full ? cnt_short : cnt_total;
    if (n > 0) {
        RUNE_KERNEL("k_nbr_fill", stream,
                    k_nbr_fill<<<blocks_for((long long)n * 32, tpb), tpb, 0, stream>>>(
                        n, tv, row_ptr, cnt_short, capacity, edges, shifts, eng.d_flags));
        RUNE_KERNEL("k_guard_rows", stream,
                    k_guard_rows<<<std::min(blocks_for(n, tpb), 1024), tpb, 0, stream>>>(
                        n, eng.d_flags, cnt_short, cnt_total));
        RUNE_LAUNCH_CHECK();
    }
    nd.n_atoms = n;
    nd.total_edges = (int)std::min<long long>(capacity, INT32_MAX);
    nd.edges = edges;
    nd.shifts = shifts;
    nd.row_ptr = row_ptr;
    nd.radial = EdgeList{edges, row_ptr, cnt_r, nullptr};
    nd.angular = EdgeList{edges, row_ptr, cnt_a, nullptr};
    nd.cnt_r = cnt_r;
    nd.cnt_a = cnt_a;
    nd.positions64 = in.positions;
    nd.sid = sid;
    nd.geom = d_geom;
    nd.summary = summary;
    nd.capacity = capacity;
    nd.types = tsafe;
    eng.stats.neighbor_builds++;
}

// End-of-call checks of a device-built list (after the stream synchronisation): capacity
// overflow (returns false: rerun), invalid inputs, neighbour limits; records the statistics.
bool finish_neighbors(Engine& eng, const NeighborData& nd, const HostSync& hs) {
    const rune_model_config& cfg = eng.cfg;
    if (hs.flags & 16u) {
        eng.edge_capacity = (long long)hs.total + hs.total / 8 + 1024;
        return false;
    }
    for (int which = 0; which < 2; ++which) {
        unsigned long long v = hs.maxc[which];
        int count = (int)(v >> 32);
        int atom = (int)(0xffffffffull - (v & 0xffffffffull));
        int limit = which == 0 ? cfg.max_neighbors_radial : cfg.max_neighbors_angular;
        if (nd.n_atoms > 0 && count > limit) {
            throw Error(RUNE_ERR_NEIGHBOR_OVERFLOW,
                        "Neighbor count " + std::to_string(count) + " for atom " +
                            std::to_string(atom) + " exceeds max_neighbors=" +
                            std::to_string(limit) +
                            ". Increase max_neighbors_radial or max_neighbors_angular.");
        }
    }
    if (hs.total > eng.edge_capacity) eng.edge_capacity = hs.total;
    eng.stats.last_edges = hs.total;
    eng.stats.last_radial_edges = (int64_t)hs.maxc[2];
    eng.stats.last_angular_edges = (int64_t)hs.maxc[3];
    return true;
}

void build_padded(Engine& eng, const PaddedInput& in, NeighborData& nd, cudaStream_t stream) {
    int n = in.n_atoms;
    const int tpb = 256;
    EdgeList lists[2];
    int totals[2] = {0, 0};
    const int64_t* nbr[2] = {in.radial_neighbors, in.angular_neighbors};
    const float* off[2] = {in.radial_offsets, in.angular_offsets};
    int width[2] = {in.radial_width, in.angular_width};
    int* cnt[2];
    int* rp[2];
    for (int w = 0; w < 2; ++w) {
        cnt[w] = eng.ws.take_n<int>(n + 1);
        rp[w] = eng.ws.take_n<int>(n + 1);
        RUNE_CUDA_TRY(cudaMemsetAsync(cnt[w] + n, 0, sizeof(int), stream));
        if (n > 0 && width[w] > 0) {
            RUNE_KERNEL("k_padded_count", stream, k_padded_count<<<blocks_for(n, tpb), tpb, 0, stream>>>(n, width[w], nbr[w], n,
                                                                     in.types, eng.cfg.n_types,
                                                                     cnt[w], eng.d_flags));
            RUNE_LAUNCH_CHECK();
        } else if (n > 0) {
            RUNE_CUDA_TRY(cudaMemsetAsync(cnt[w], 0, sizeof(int) * n, stream));
        }
        exclusive_scan(eng, cnt[w], rp[w], n + 1, stream);
    }
    HostSync* hs = eng.host_sync;
    RUNE_CUDA_TRY(cudaMemcpyAsync(&hs->total, rp[0] + n, sizeof(int), cudaMemcpyDeviceToHost,
                                  stream));
    RUNE_CUDA_TRY(cudaMemcpyAsync(&hs->total2, rp[1] + n, sizeof(int), cudaMemcpyDeviceToHost,
                                  stream));
    RUNE_CUDA_TRY(cudaMemcpyAsync(&hs->flags, eng.d_flags, sizeof(unsigned int),
                                  cudaMemcpyDeviceToHost, stream));
    RUNE_CUDA_TRY(cudaStreamSynchronize(stream));
    eng.check_flags(hs->flags, stream);
    totals[0] = hs->total;
    totals[1] = hs->total2;
    for (int w = 0; w < 2; ++w) {
        float4* e = eng.ws.take_n<float4>(totals[w] + 1);
        if (n > 0 && totals[w] > 0) {
            RUNE_KERNEL("k_padded_fill", stream, k_padded_fill<<<blocks_for(n, tpb), tpb, 0, stream>>>(n, width[w], nbr[w], off[w],
                                                                    in.positions, rp[w], e));
            RUNE_LAUNCH_CHECK();
        }
        lists[w] = EdgeList{e, rp[w], cnt[w], nullptr};
    }
    nd.n_atoms = n;
    nd.total_edges = totals[0];
    nd.total_angular = totals[1];
    nd.edges = nullptr;
    nd.shifts = nullptr;
    nd.row_ptr = nullptr;
    nd.radial = lists[0];
    nd.angular = lists[1];
    nd.cnt_r = cnt[0];
    nd.cnt_a = cnt[1];
    eng.stats.last_edges = totals[0];
    eng.stats.last_radial_edges = totals[0];
    eng.stats.last_angular_edges = totals[1];
}

void build_reverse(Engine& eng, NeighborData& nd, EdgeList& list, int n_edges,
                   cudaStream_t stream) {
    int* rev = eng.ws.take_n<int>(n_edges + 1);
    if (nd.n_atoms > 0 && n_edges > 0) {
        RUNE_KERNEL("k_rev_index", stream, k_rev_index<<<blocks_for((long long)nd.n_atoms * 32, 256), 256, 0, stream>>>(
            nd.n_atoms, list, rev, eng.d_flags));
        RUNE_LAUNCH_CHECK();
    }
    list.rev = rev;
}

}  // namespace rune
