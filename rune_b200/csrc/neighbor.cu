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

__global__ void k_atom_structure(int n_atoms, int n_structures, const int* __restrict__ atom_ptr,
                                 int* __restrict__ sid) {
    int a = blockIdx.x * blockDim.x + threadIdx.x;
    if (a >= n_atoms) return;
    int lo = 0, hi = n_structures - 1;
    while (lo < hi) {  // last structure whose start <= a
        int mid = (lo + hi + 1) >> 1;
        if (atom_ptr[mid] <= a) lo = mid; else hi = mid - 1;
    }
    sid[a] = lo;
}

// Bin every atom; record its integer wrap (floor of the fractional coordinate on periodic
// axes) so that shifts refer to the caller's unwrapped positions.
__global__ void k_bin_atoms(int n_atoms, int n_types, const double* __restrict__ pos,
                            const int* __restrict__ types, const int* __restrict__ sid,
                            const StructGeom* __restrict__ geom, int4* __restrict__ binc,
                            int4* __restrict__ wrap, int* __restrict__ bin_count,
                            unsigned int* __restrict__ flags) {
    int a = blockIdx.x * blockDim.x + threadIdx.x;
    if (a >= n_atoms) return;
    const StructGeom& g = geom[sid[a]];
    double p[3] = {pos[3 * a], pos[3 * a + 1], pos[3 * a + 2]};
    int t = types[a];
    if (t < 0 || t >= n_types) atomicOr(flags, 1u);
    int b[3], w[3];
    bool finite = isfinite(p[0]) && isfinite(p[1]) && isfinite(p[2]);
    if (!finite) atomicOr(flags, 2u);
    for (int k = 0; k < 3; ++k) {
        double f = p[0] * g.inv[0 * 3 + k] + p[1] * g.inv[1 * 3 + k] + p[2] * g.inv[2 * 3 + k];
        if (!finite) f = 0.0;
        if (g.pbc[k]) {
            double fl = floor(f);
            if (fabs(fl) > 1.0e6) { atomicOr(flags, 2u); fl = 0.0; }
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

// Sort each bin's atom list ascending (rank sort; atom indices are unique), warp per bin.
__global__ void k_sort_bins(int n_bins, const int* __restrict__ bin_start,
                            const int* __restrict__ bin_count, const int* __restrict__ unsorted,
                            int* __restrict__ sorted) {
    int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (warp >= n_bins) return;
    int start = bin_start[warp], n = bin_count[warp];
    for (int base = 0; base < n; base += 32) {
        int k = base + lane;
        int v = k < n ? unsorted[start + k] : 0;
        int rank = 0;
        for (int m = 0; m < n; ++m) rank += unsorted[start + m] < v;
        if (k < n) sorted[start + rank] = v;
    }
}

struct Traverse {
    const StructGeom* geom;
    const double* pos;
    const int4* binc;
    const int4* wrap;
    const int* sid;
    const int* bin_start;
    const int* bin_count;
    const int* bin_atoms;
    double rc_max2, rc_min2;
};

// Visit every candidate j of atom i in a fixed order; `visit(j, S, d, d^2, valid)` is called by
// all 32 lanes once per round (valid = this lane holds a candidate inside rc_max).
template <typename Visit>
__device__ __forceinline__ void traverse(const Traverse& tv, int i, int lane, Visit&& visit) {
    const StructGeom& g = tv.geom[tv.sid[i]];
    int4 bc = tv.binc[i];
    int4 wi = tv.wrap[i];
    double pi0 = tv.pos[3 * i], pi1 = tv.pos[3 * i + 1], pi2 = tv.pos[3 * i + 2];
    int bi[3] = {bc.x, bc.y, bc.z};
    for (int dx = -g.reach[0]; dx <= g.reach[0]; ++dx) {
        int tx = bi[0] + dx, ix = 0;
        if (g.pbc[0]) { ix = floordiv(tx, g.nb[0]); tx -= ix * g.nb[0]; }
        else if (tx < 0 || tx >= g.nb[0]) continue;
        for (int dy = -g.reach[1]; dy <= g.reach[1]; ++dy) {
            int ty = bi[1] + dy, iy = 0;
            if (g.pbc[1]) { iy = floordiv(ty, g.nb[1]); ty -= iy * g.nb[1]; }
            else if (ty < 0 || ty >= g.nb[1]) continue;
            for (int dz = -g.reach[2]; dz <= g.reach[2]; ++dz) {
                int tz = bi[2] + dz, iz = 0;
                if (g.pbc[2]) { iz = floordiv(tz, g.nb[2]); tz -= iz * g.nb[2]; }
                else if (tz < 0 || tz >= g.nb[2]) continue;
                int tb = g.bin_offset + (tx * g.nb[1] + ty) * g.nb[2] + tz;
                int start = tv.bin_start[tb], cnt = tv.bin_count[tb];
                for (int base = 0; base < cnt; base += 32) {
                    int k = base + lane;
                    bool valid = k < cnt;
                    int j = valid ? tv.bin_atoms[start + k] : 0;
                    int4 wj = tv.wrap[j];
                    int s0 = g.pbc[0] ? ix - wj.x + wi.x : 0;
                    int s1 = g.pbc[1] ? iy - wj.y + wi.y : 0;
                    int s2 = g.pbc[2] ? iz - wj.z + wi.z : 0;
                    // (R_j - R_i) + S.cell: exactly antisymmetric under i <-> j, S -> -S
                    double d0 = (tv.pos[3 * j] - pi0) +
                                (s0 * g.cell[0] + s1 * g.cell[3] + s2 * g.cell[6]);
                    double d1 = (tv.pos[3 * j + 1] - pi1) +
                                (s0 * g.cell[1] + s1 * g.cell[4] + s2 * g.cell[7]);
                    double d2v = (tv.pos[3 * j + 2] - pi2) +
                                 (s0 * g.cell[2] + s1 * g.cell[5] + s2 * g.cell[8]);
                    double r2 = d0 * d0 + d1 * d1 + d2v * d2v;
                    valid = valid && r2 < tv.rc_max2 && !(j == i && s0 == 0 && s1 == 0 && s2 == 0);
                    visit(j, s0, s1, s2, d0, d1, d2v, r2, valid);
                }
            }
        }
    }
}

__global__ void k_nbr_count(int n_atoms, Traverse tv, int* __restrict__ cnt_short,
                            int* __restrict__ cnt_total) {
    int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (i >= n_atoms) return;
    int ns = 0, nt = 0;
    traverse(tv, i, lane, [&](int, int, int, int, double, double, double, double r2, bool valid) {
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

__global__ void k_nbr_fill(int n_atoms, Traverse tv, const int* __restrict__ row_ptr,
                           const int* __restrict__ cnt_short, const StructGeom* __restrict__ geom,
                           float4* __restrict__ edges, int* __restrict__ shifts) {
    int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (i >= n_atoms) return;
    int base_s = row_ptr[i];
    int base_l = row_ptr[i] + cnt_short[i];
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

// Largest per-atom radial / angular count, packed (count << 32 | ~atom) so the first atom wins.
__global__ void k_max_counts(int n_atoms, const int* __restrict__ ra, const int* __restrict__ an,
                             unsigned long long* __restrict__ out) {
    int a = blockIdx.x * blockDim.x + threadIdx.x;
    if (a >= n_atoms) return;
    unsigned long long inv = 0xffffffffull - (unsigned long long)a;
    atomicMax(&out[0], ((unsigned long long)ra[a] << 32) | inv);
    atomicMax(&out[1], ((unsigned long long)an[a] << 32) | inv);
    atomicAdd(&out[2], (unsigned long long)ra[a]);
    atomicAdd(&out[3], (unsigned long long)an[a]);
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
    RUNE_CUDA_TRY(cudaMemcpyAsync(d_geom, geom.data(), sizeof(StructGeom) * geom.size(),
                                  cudaMemcpyHostToDevice, stream));
    int* d_atom_ptr = eng.ws.take_n<int>(in.n_structures + 1);
    RUNE_CUDA_TRY(cudaMemcpyAsync(d_atom_ptr, in.atom_ptr, sizeof(int) * (in.n_structures + 1),
                                  cudaMemcpyHostToDevice, stream));
    int* sid = eng.ws.take_n<int>(n);
    int4* binc = eng.ws.take_n<int4>(n);
    int4* wrap = eng.ws.take_n<int4>(n);
    int* bin_count = eng.ws.take_n<int>(total_bins + 1);
    int* bin_start = eng.ws.take_n<int>(total_bins + 1);
    int* bin_fill = eng.ws.take_n<int>(total_bins + 1);
    int* bin_tmp = eng.ws.take_n<int>(n);
    int* bin_atoms = eng.ws.take_n<int>(n);
    int* cnt_short = eng.ws.take_n<int>(n + 1);
    int* cnt_total = eng.ws.take_n<int>(n + 1);
    int* row_ptr = eng.ws.take_n<int>(n + 1);
    unsigned long long* maxc = eng.ws.take_n<unsigned long long>(4);
    RUNE_CUDA_TRY(cudaMemsetAsync(bin_count, 0, sizeof(int) * (total_bins + 1), stream));
    RUNE_CUDA_TRY(cudaMemsetAsync(bin_fill, 0, sizeof(int) * (total_bins + 1), stream));
    RUNE_CUDA_TRY(cudaMemsetAsync(maxc, 0, sizeof(unsigned long long) * 4, stream));
    RUNE_CUDA_TRY(cudaMemsetAsync(cnt_total + n, 0, sizeof(int), stream));

    const int tpb = 256;
    if (n > 0) {
        RUNE_KERNEL("k_atom_structure", stream, k_atom_structure<<<blocks_for(n, tpb), tpb, 0, stream>>>(n, in.n_structures, d_atom_ptr,
                                                                   sid));
        RUNE_KERNEL("k_bin_atoms", stream, k_bin_atoms<<<blocks_for(n, tpb), tpb, 0, stream>>>(n, cfg.n_types, in.positions,
                                                              in.types, sid, d_geom, binc, wrap,
                                                              bin_count, eng.d_flags));
        RUNE_LAUNCH_CHECK();
    }
    exclusive_scan(eng, bin_count, bin_start, total_bins + 1, stream);
    if (n > 0) {
        RUNE_KERNEL("k_fill_bins", stream, k_fill_bins<<<blocks_for(n, tpb), tpb, 0, stream>>>(n, binc, bin_start, bin_fill, bin_tmp));
        RUNE_KERNEL("k_sort_bins", stream, k_sort_bins<<<blocks_for((long long)total_bins * 32, tpb), tpb, 0, stream>>>(
            total_bins, bin_start, bin_count, bin_tmp, bin_atoms));
        RUNE_LAUNCH_CHECK();
    }
    Traverse tv{d_geom, in.positions, binc, wrap, sid, bin_start, bin_count, bin_atoms,
                rc_max * rc_max, rc_min * rc_min};
    if (n > 0) {
        RUNE_KERNEL("k_nbr_count", stream, k_nbr_count<<<blocks_for((long long)n * 32, tpb), tpb, 0, stream>>>(n, tv, cnt_short,
                                                                             cnt_total));
        RUNE_LAUNCH_CHECK();
    }
    exclusive_scan(eng, cnt_total, row_ptr, n + 1, stream);
    bool radial_is_full = cfg.rc_radial >= cfg.rc_angular;
    const int* cnt_r = radial_is_full ? cnt_total : cnt_short;
    const int* cnt_a = radial_is_full ? cnt_short : cnt_total;
    if (n > 0) {
        RUNE_KERNEL("k_max_counts", stream, k_max_counts<<<blocks_for(n, tpb), tpb, 0, stream>>>(n, cnt_r, cnt_a, maxc));
        RUNE_LAUNCH_CHECK();
    }
    // one synchronisation: edge total, max counts and error flags
    HostSync* hs = eng.host_sync;
    RUNE_CUDA_TRY(cudaMemcpyAsync(&hs->total, row_ptr + n, sizeof(int), cudaMemcpyDeviceToHost,
                                  stream));
    RUNE_CUDA_TRY(cudaMemcpyAsync(hs->maxc, maxc, sizeof(unsigned long long) * 4,
                                  cudaMemcpyDeviceToHost, stream));
    RUNE_CUDA_TRY(cudaMemcpyAsync(&hs->flags, eng.d_flags, sizeof(unsigned int),
                                  cudaMemcpyDeviceToHost, stream));
    RUNE_CUDA_TRY(cudaStreamSynchronize(stream));
    eng.check_flags(hs->flags, stream);
    for (int which = 0; which < 2; ++which) {
        unsigned long long v = hs->maxc[which];
        int count = (int)(v >> 32);
        int atom = (int)(0xffffffffull - (v & 0xffffffffull));
        int limit = which == 0 ? cfg.max_neighbors_radial : cfg.max_neighbors_angular;
        if (n > 0 && count > limit) {
            throw Error(RUNE_ERR_NEIGHBOR_OVERFLOW,
                        "Neighbor count " + std::to_string(count) + " for atom " +
                            std::to_string(atom) + " exceeds max_neighbors=" +
                            std::to_string(limit) +
                            ". Increase max_neighbors_radial or max_neighbors_angular.");
        }
    }
    int total = hs->total;
    float4* edges = eng.ws.take_n<float4>(total + 1);
    int* shifts = eng.ws.take_n<int>(total + 1);
    if (n > 0 && total > 0) {
        RUNE_KERNEL("k_nbr_fill", stream, k_nbr_fill<<<blocks_for((long long)n * 32, tpb), tpb, 0, stream>>>(n, tv, row_ptr,
                                                                            cnt_short, d_geom,
                                                                            edges, shifts));
        RUNE_LAUNCH_CHECK();
    }
    nd.n_atoms = n;
    nd.total_edges = total;
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
    eng.stats.neighbor_builds++;
    eng.stats.last_edges = total;
    eng.stats.last_radial_edges = (int64_t)hs->maxc[2];
    eng.stats.last_angular_edges = (int64_t)hs->maxc[3];
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
