// Engine-internal types shared by the .cu translation units (not part of the C ABI).
#pragma once

#include <algorithm>
#include <cmath>
#include <map>
#include <string>
#include <vector>

#include "common.cuh"

namespace rune {

// Grow-only device workspace. Each compute call resets the cursor and carves its arrays in
// order; when a call needs more than the current capacity the arena is reallocated before
// the next call (the failing call is retried once by the caller).
struct Arena {
    char* base = nullptr;
    size_t cap = 0;
    size_t off = 0;
    size_t want = 0;  // bytes the current call asked for
    bool overflow = false;
    char* spill = nullptr;  // dummy target used after an overflow until the call restarts

    void reset() {
        off = 0;
        want = 0;
        overflow = false;
    }
    void* take(size_t bytes) {
        size_t aligned = (off + 255) & ~size_t(255);
        want = aligned + bytes;
        if (want > cap) {
            overflow = true;
            throw Error(-1, "workspace");  // caught by the engine, which grows and retries
        }
        off = want;
        return base + aligned;
    }
    template <typename T>
    T* take_n(size_t n) {
        return static_cast<T*>(take(sizeof(T) * (n ? n : 1)));
    }
};

struct StructGeom {
    double cell[9];
    double inv[9];
    int nb[3];
    int reach[3];
    int pbc[3];
    int bin_offset;
};

struct HostSync {
    int total;
    int total2;
    unsigned int flags;
    unsigned int pad;
    unsigned long long maxc[4];
};

// Pinned host staging for the small per-call uploads (cells, structure pointers, reduction
// chunks): copies from pageable memory would synchronise the stream.
struct Staging {
    char* base = nullptr;
    size_t cap = 0;
    size_t off = 0;
};

struct BatchInput {
    int n_atoms, n_structures;
    const int* types;
    const double* positions;
    const double* cells;
    const uint8_t* pbc;
    const int* atom_ptr;
};

struct PaddedInput {
    int n_atoms, n_structures;
    const int* types;
    const float* positions;
    const int64_t* radial_neighbors;
    int radial_width;
    const float* radial_offsets;
    const int64_t* angular_neighbors;
    int angular_width;
    const float* angular_offsets;
    const int* atom_ptr;
};

struct NeighborData {
    int n_atoms = 0;
    int total_edges = 0;
    int total_angular = 0;
    float4* edges = nullptr;
    int* shifts = nullptr;
    const int* cnt_r = nullptr;
    const int* cnt_a = nullptr;
    EdgeList radial, angular;
    // device path only: float64 geometry to re-form pair vectors exactly (ZBL)
    const double* positions64 = nullptr;
    const int* sid = nullptr;
    const StructGeom* geom = nullptr;
    const int* types = nullptr;                 // validated copy of the caller's types
    unsigned long long* summary = nullptr;      // max / sum of counts (device)
    long long capacity = 0;                     // edge buffer size
};

// Device layout of one dense layer y = x W^T + b, kept as W^T [in, out] (forward) and
// W [out, in] (backward) so that every GEMM reads its right operand row-major.
struct Dense {
    int in = 0, out = 0;
    const float* wt = nullptr;  // [in, out]
    const float* w = nullptr;   // [out, in]
    const float* b = nullptr;   // [out] or null
};

// One MP message block (rune/mobius/message.py), device layouts.
struct MpLayerArgs {
    int H, M, G, V, K, T, act;
    float rc, eps;
    const float* pb;    // [T*T][Mp] W_e[:, K:] P[pair] + b_e (zero padded)
    const float* we_k;  // [Mp][K]   W_e basis columns
    const float* wgv;   // [G+V][Mp] group gate rows, then vector gate rows
    const float* bgv;   // [G+V]
    const float* g_msg; // [H]       message_norm weight
    const float* wmix;  // [V][V]
    int Mp = 0;         // edge hidden size padded to a multiple of 4 (pb, we_k, wgv rows)
};

struct MpLayer {
    MpLayerArgs args;
    Dense vs;    // [H -> H+V]: value_projection ; vector_source (input_norm weight folded)
    Dense upd1;  // [H+V -> M]
    Dense upd2;  // [M -> H]
};

// gv: gates * cutoff per edge (read by the neighbour-side pull); sg: the gates before the cutoff
// (read by the centre side of the backward instead of recomputing the edge MLP)
void mp_forward_edges(const MpLayerArgs& L, int n_atoms, const EdgeList& rad, const int* types,
                      const float* vs, float* msg, float* vec, float* gv, float* sg,
                      cudaStream_t stream);
void mp_node_forward(const MpLayerArgs& L, int n_atoms, const float* msg, const float* vec,
                     float* uin, float* rho_m, float* mixed, cudaStream_t stream);
void mp_node_backward(const MpLayerArgs& L, int n_atoms, const float* msg, const float* rho_m,
                      const float* mixed, const float* duin, float* dmsg, float* dvec,
                      cudaStream_t stream);
void mp_backward_edges(const MpLayerArgs& L, int n_atoms, const EdgeList& rad, const int* types,
                       const float* vs, const float* dmsg, const float* dvec, const float* gv,
                       const float* sg, float4* edge_grad, float* dvs, cudaStream_t stream);

// One EQ block (rune/mobius/equivariant.py), device layouts (padded as equivariant.cu expects).
// Padded GEMM dimensions of the EQ edge kernels: reduction (K) dims to a multiple of 16,
// output (N) dims to 32 x nt with nt in {1, 2, 3, 4, 6, 8, 10}.
struct EqTileDims {
    int XK, XN, MK, MN, GK, GN;
    __host__ __device__ static int k16(int n) { return (n + 15) / 16 * 16; }
    // tile widths 32 x {1, 2, 3, 4, 6, 8, 10}: an even count above 4 lets every thread read its
    // weight columns as float2 (an odd count of nine would need scalar shared-memory loads)
    __host__ __device__ static int n32(int n) {
        int t = (n + 31) / 32;
        if (t == 5) t = 6;
        if (t == 7) t = 8;
        if (t == 9) t = 10;
        return 32 * t;
    }
    __host__ __device__ EqTileDims(int x, int m, int g)
        : XK(k16(x)), XN(n32(x)), MK(k16(m)), MN(n32(m)), GK(k16(g)), GN(n32(g)) {}
};

// One EQ edge-GEMM weight matrix W [K][N] (as the edge kernels use it: out[f][e] =
// sum_k W[k][f] x[k][e]) packed for the tensor cores (equivariant.cu): units of 128 output
// features x 32 k, four digit planes each (16 KB), chunk-major; then one exponent per feature.
struct EqTcW {
    const signed char* q = nullptr;
    const int* fexp = nullptr;
    int K = 0, N = 0, steps = 0, chunks = 0;
};

// default bound of the EQ kernels' waits (polls of mbarrier.try_wait)
constexpr unsigned kEqWaitPolls = 1u << 22;

struct EqLayerArgs {
    int H, M, G, Ce, Le, Cl, K, T, act;
    float rc, eps;
    const float* pb;     // [T*T][M]     W_e[:, pair] P[pair] + b_e
    const float* wxT;    // [XK][MN]     basis + probe columns of W_e, transposed, zero padded
    const float* wx;     // [MK][XN]
    const float* wgdT;   // [MK][GN]     [W_g ; W_d]^T
    const float* wgd;    // [GK][MN]
    const float* bgd;    // [GD]
    const float* wmix;   // [Le][Ce][Ce]
    const float* g_msg;  // [H]
    const float* scale;  // [Cl]         orthonormal harmonic scale
    const float* zc;     // z-polynomial table
    // Tile-padded GEMM shapes of the edge kernels (K dims to 16, N dims to 32 x {1,2,3,4,6,8,10}):
    // wxT [XK][MN], wgdT [MK][GN], wgd [GK][MN], wx [MK][XN]
    int XK = 0, XN = 0, MK = 0, MN = 0, GK = 0, GN = 0;
    // tensor-core forms of wxT, wgdT, wgd, wx (tc = false: the SIMT tile GEMM)
    bool tc = false;
    EqTcW tx, tgd, tgdT, txT;
    // polls of a bounded wait on a weight copy or an MMA completion before the block gives up
    // (error flag 32); the drain of the copies still in flight always uses the full bound
    unsigned wait_polls = kEqWaitPolls;
};
// bytes of the packed tensor-core form of W [K][N]; packs it (device arrays, stream order)
size_t eq_tc_bytes(int K, int N);
EqTcW eq_tc_pack(const float* W, int K, int N, void* out, cudaStream_t stream);

struct EqLayer {
    EqLayerArgs args;
    Dense nodes;  // [H -> 2M + H]: W_e,c W_c ; W_e,n W_n ; W_v  (input_norm weight folded)
    Dense upd1;   // [H + Le Ce -> M]
    Dense upd2;   // [M -> H]
};

void eq_mix(const EqLayerArgs& L, int n, const float* D, float* mixed, cudaStream_t stream);
void eq_forward_edges(const EqLayerArgs& L, int n, const EdgeList& rad, const int* types,
                      const float* abv, const float* D, const float* mixed, float* msg,
                      float* dn, float* gva, unsigned* err, cudaStream_t stream);
void eq_node_forward(const EqLayerArgs& L, int n, const float* msg, const float* dn, float* uin,
                     float* rho_m, cudaStream_t stream);
void eq_node_backward(const EqLayerArgs& L, int n, const float* msg, const float* rho_m,
                      const float* dn, const float* duin, const float* ddn_next, float* dmsg,
                      float* ddp, cudaStream_t stream);
// The centre kernel runs over atoms [0, n_centres); the pull over all n atoms, skipping reverse
// edges from atoms >= n_centres (n_centres = n outside domain calls).
void eq_backward_edges(const EqLayerArgs& L, int n, int n_centres, const EdgeList& rad,
                       const int* types, const float* abv, const float* D, const float* mixed, const float* dmsg,
                       const float* ddp, const float* gva, float* dpre, float* dpn,
                       float4* edge_grad, float* dabv, float* ddc, float* dd_prev,
                       unsigned* err, cudaStream_t stream);
void eq_encode(const EqLayerArgs& L, int n, int na, int C, const float* proj, const float* s,
               float* D0, cudaStream_t stream);
void eq_encode_backward(const EqLayerArgs& L, int n, int na, int C, const float* proj,
                        const float* dd0, float* mg, cudaStream_t stream);

// Tensor-core operand of one weight matrix B [K][N] (dense_tc.cu): four planes of signed 7-bit
// digits in units of 32 k x 64 columns, then the columns' exponents.
struct TcMatrix {
    const void* w = nullptr;
    int K = 0, N = 0;
};

struct Engine {
    rune_model_config cfg{};
    int device = 0;
    bool finalized = false;
    std::map<std::string, std::vector<float>> host;

    // derived sizes
    int C = 0, nL = 0, D = 0, n_terms = 0, n_dterms = 0;

    // device weights: one blob
    float* blob = nullptr;
    size_t blob_floats = 0;
    std::map<std::string, size_t> offsets;
    DescParams desc{};

    // NEP
    const float* nep_w1 = nullptr;   // [T][H][Dp], rows padded to a multiple of 4
    const float* nep_w1t = nullptr;  // [T][D][Hp]
    const float* nep_b1 = nullptr;   // [T][H]
    const float* nep_w2 = nullptr;   // [T][H]
    const float* q_scaler = nullptr; // [D]
    float nep_bias = 0.f;

    // Möbius
    Dense input_projection;
    const float* embedding = nullptr;  // [T][H]
    std::vector<Dense> ffn1, ffn2;     // per residual block (norm weight folded into ffn1)
    std::vector<const float*> block_norm;  // [H] norm weights
    const float* out_norm = nullptr;   // [H]
    const float* head_w = nullptr;     // [T][H]
    const float* head_b = nullptr;     // [T]
    std::vector<MpLayer> mp;           // MP message blocks
    std::vector<EqLayer> eq;           // EQ blocks
    const float* eq_proj = nullptr;    // [Le][Ce][na] direction encoder

    // ZBL
    const float* zbl_z = nullptr;       // [T] atomic numbers
    const float* zbl_pairs = nullptr;   // [T(T+1)/2][10] flexible parameters
    const float* zbl_coef = nullptr;    // [4][2] universal coefficients
    double zbl_max_outer = 0.0;         // largest outer cutoff (pairs beyond it skip ZBL)

    // workspace and sync
    Arena ws;
    HostSync* host_sync = nullptr;
    unsigned int* d_flags = nullptr;
    Staging staging;
    size_t staging_want = 0;
    char* d_mirror = nullptr;         // device copy of the staging buffer (same offsets)
    size_t stage_first = ~size_t(0);  // first staged byte not yet copied
    int row_stride = 0;  // edge slots per atom of the device-built lists, raised on overflow
    // halo calls: the sizes of the last rehearsal (atoms, owned atoms, row stride, box) and the
    // workspace bytes it used; a call whose sizes match needs no rehearsal
    std::vector<double> halo_key;
    size_t halo_bytes = 0;
    void* eq_tc_buf = nullptr;  // tensor-core forms of the EQ edge-GEMM weights
    unsigned wait_polls = kEqWaitPolls;  // bound of the EQ kernels' waits
    rune_stats stats{};
    Profiler prof;

    // last neighbour list (for rune_engine_neighbor_pairs)
    NeighborData last;
    bool last_valid = false;

    const float* tensor(const std::string& name) const;
    void check_flags(unsigned int flags, cudaStream_t stream);
    // host -> device copy through pinned staging (no stream synchronisation); staging is reset
    // at the start of every call and grows only outside the static-scratch entry point
    // Per-call host tables: stage_upload copies into the pinned staging buffer and returns the
    // device address the bytes will have; flush_uploads issues one copy for everything staged
    // since the last flush (it must precede the first kernel reading the tables).
    void* stage_upload(const void* src, size_t bytes, cudaStream_t stream);
    void flush_uploads(cudaStream_t stream);
    bool static_call = false;
};

// Per-call structure tables on the device: atom_ptr [B + 1] and chunk_ptr [B + 1] (fixed-size
// atom chunks of each structure, for the deterministic per-structure sums).
struct CallTables {
    const int* atom_ptr = nullptr;
    const int* chunk_ptr = nullptr;
    int n_chunks = 0;
};
CallTables stage_call_tables(Engine& eng, int n_structures, const int* atom_ptr_host,
                             cudaStream_t stream);

// Device neighbour lists. With skin > 0 the rows are candidate lists (all pairs within
// max(rc) + skin, one class) in rows of the stride kept in *stride_state.
void build_neighbors(Engine& eng, const BatchInput& in, const int* d_atom_ptr, NeighborData& nd,
                     cudaStream_t stream, double skin = 0.0, int* stride_state = nullptr);
// The exact radial / angular lists from candidate lists at the current positions (same rows
// and stride as the candidates), as build_neighbors would produce them.
void filter_candidates(Engine& eng, const NeighborData& cand, const double* positions,
                       NeighborData& nd, cudaStream_t stream);
void build_padded(Engine& eng, const PaddedInput& in, NeighborData& nd, cudaStream_t stream);
void build_reverse(Engine& eng, NeighborData& nd, EdgeList& list, int n_edges,
                   cudaStream_t stream);
bool finish_neighbors(Engine& eng, const NeighborData& nd, const HostSync& hs);

// ----------------------------------------------------------------------------- launchers
struct NepHeadArgs {
    int H;
    const float* w1;   // [T][H][Dp] (rows padded to a multiple of 4)
    const float* w1t;  // [T][D][Hp]
    const float* b1;
    const float* w2;
    const float* scaler;
    float bias;
};

struct ForceLaunch {
    int n_atoms;
    DescParams p;
    EdgeList rad, ang, zbl_list;
    const int* types;
    const float4* dqr;  // [N][npr] radial adjoint, channels padded to a multiple of 4
    // [N][T][gkp] radial adjoint contracted with the c-table per neighbour type (NEP with few
    // types), or null
    const float* gtab;
    int gkp;
    const float4* ang_grad;
    int zbl_mode;
    double zbl_rc_inner, zbl_rc_outer;
    const float* zbl_zpow;
    const float* zbl_z;
    const float* zbl_coef;
    const float* zbl_pairs;
    const float4* edge_grad;
    const double* positions64;
    const int* sid;
    const StructGeom* geom;
    const int* shifts;
    double zbl_max_outer;
    int n_owned;  // atoms >= n_owned are ghosts of a domain call (n_atoms otherwise)
    bool descriptor;
    double* e_zbl;
    float* forces;
    double* virial_atom;
};

// Descriptor forward: row layout (q [N, D] with invariants, s [N, na, C]) or, with `tiled`,
// the NEP tiled layout (radial channels and moments in 128-atom tiles).
void launch_desc_forward(const DescParams& p, int n_atoms, const EdgeList& rad,
                         const EdgeList& ang, const int* types, float* q, float* s, bool tiled,
                         cudaStream_t stream);
size_t nep_tiled_floats(int n_atoms, int per_atom);
void launch_nep_atoms(const DescParams& p, int n_atoms, int n_owned, const NepHeadArgs& nep,
                      const int* types, const float* qr_t, const float* s_t, double* e_model,
                      float4* dqr, float* w_t, float* gtab, cudaStream_t stream);
void launch_angular_grad(const DescParams& p, int n_atoms, const EdgeList& ang,
                         const int* types, const float* w_t, float4* ang_grad,
                         cudaStream_t stream);
void launch_desc_backward(const DescParams& p, int n_atoms, const EdgeList& ang,
                          const int* types, const float* dq, const float* s, const float* mg,
                          float4* dqr, float4* ang_grad, cudaStream_t stream);
int channel_bound(const DescParams& p);
void launch_forces(const ForceLaunch& f, cudaStream_t stream);

// Dense per-atom layers (dense.cu)
struct GemmEpilogue {
    const float* row_scale = nullptr;  // [M]       acc *= row_scale[m]
    const float* bias = nullptr;       // [N]       + bias[n]
    const float* emb = nullptr;        // [T][N]    + emb[types[m]][n]
    const int* types = nullptr;
    int act = -1;                      // RUNE_ACT_* or -1
    float* dact = nullptr;             // [M, ldc]  activation derivative output
    const float* mul = nullptr;        // [M, ldc]  elementwise factor (applied last)
    const float* residual = nullptr;   // [M, ldc]  + residual (after activation)
};
size_t tc_packed_bytes(int K, int N);
void tc_pack(const float* B, int K, int N, void* out, cudaStream_t stream);
size_t gemm_tc_smem();
void gemm_tc(int M, int N, int K, const float* A, int lda, const TcMatrix& B, float* C, int ldc,
             const GemmEpilogue& ep, unsigned* err, cudaStream_t stream);
// C [M][N] = A [M][K] B [K][N] (host arrays) by the tensor-core GEMM on device `device`
// (diagnostic of rune_tc_selftest).
void tc_selftest(int M, int N, int K, const float* a_host, const float* b_host, float* c_host,
                 int device);
// C[M, N] = epilogue(A[M, K] @ B[K, N]); all row-major.
// Split-K scratch for the gemm calls of one evaluation on this thread (null: no split-K).
void set_gemm_split_scratch(double* ws, size_t cap);
void gemm(int M, int N, int K, const float* A, int lda, const float* B, int ldb, float* C,
          int ldc, const GemmEpilogue& ep, cudaStream_t stream);
void row_rms(int M, int H, const float* h, int ld, float eps, float* rho, cudaStream_t stream);
void rms_backward_add(int M, int H, const float* h, const float* rho, const float* dup,
                      float* dh, cudaStream_t stream);
void readout(int M, int H, const float* h, const int* types, const float* gamma,
             const float* head_w, const float* head_b, float eps, double* e_model, float* dh,
             cudaStream_t stream);

// One rank's local system in a spatial domain decomposition: atoms ordered owned first, then
// ghost shells by distance from the owned region. Shell k (1 <= k <= message layers) holds the
// ghosts within k radial cutoffs, the last shell those within one more descriptor cutoff.
// Energies count owned atoms only; forces and virial are the derivatives of that energy with
// respect to every local atom (ghost forces belong to the ghosts' owners).
struct DomainCall {
    int n_owned = 0;
    std::vector<int> shell_end;  // cumulative atom counts: shell_end[0] = n_owned, back() = N
    // Halo mode (rune_engine_compute_halo): one ghost shell; every layer's centres are the
    // owned atoms, and the ghost rows of the layer inputs come from their owners through
    // `halo`. A rehearsal attempt runs the same work without exchanges (sizing only).
    rune_halo_fn halo = nullptr;
    void* halo_ctx = nullptr;
    bool rehearsal = false;
    mutable int exchanges = 0;  // exchanges issued by the current attempt
    // Message layer l (of n) needs centres within n - 1 - l cutoffs of the owned region.
    int layer_centres(int l, int n_layers) const {
        if (halo) return n_owned;
        int k = n_layers - 1 - l;
        return shell_end[std::min<size_t>((size_t)k, shell_end.size() - 1)];
    }
};

// Evaluate energies (+ forces / virial) on a prepared neighbour list.
struct Outputs {
    float* energies;
    double* energy;
    float* forces;
    double* virial;
    int flags;
};
void evaluate(Engine& eng, NeighborData& nd, int n_atoms, int n_structures, const int* types,
              const CallTables& ct, const Outputs& out, cudaStream_t stream,
              const DomainCall* dom = nullptr);
// Replaces the workspace with one of at least `want` bytes (geometric growth).
void grow_workspace(Engine& e, size_t want, cudaStream_t stream);

// Velocity-Verlet NVE (md.cu): one structure, state in device memory, updated in place.
struct MdArgs {
    int n_atoms;
    const int* types;      // [N]
    double* positions;     // [N, 3] A (in/out)
    double* velocities;    // [N, 3] A/fs (in/out)
    const double* masses;  // [N] amu
    const double* cell;    // [9] host
    const uint8_t* pbc;    // [3] host
    double dt;             // fs
    int n_steps;
    double skin;           // A
    double* energies;      // host [n_steps + 1][2]: potential, kinetic (eV), or null
    float* forces;         // [N, 3] device, forces at the final positions, or null
    int64_t* rebuilds;     // host: candidate-list builds, or null
};
void md_nve(Engine& e, const MdArgs& a, cudaStream_t stream);

}  // namespace rune
