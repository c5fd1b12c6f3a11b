/*
 * rune_b200 — C ABI of the B200-native energy / force / virial engine for RUNE models
 * (NEP4 and Möbius Local / MP / EQ).
 *
 * All entry points are plain C: integer status codes, plain pointers and sizes, no torch
 * types. Device pointers are CUDA device memory of the engine's device; "host" pointers are
 * ordinary host memory. Every compute call runs on the CUDA stream passed as `stream`
 * (a cudaStream_t; NULL = legacy default stream) and returns after the results are written.
 * rune_engine_compute and rune_engine_compute_domain build the neighbour lists in one pass and
 * synchronise that stream once, at the end, to read the error flags and the neighbour-count
 * summary; the padded entry points synchronise twice (after counting the padded rows, to size
 * the edge arrays, and at the end). A call whose workspace or neighbour-row stride turns out too
 * small grows it and runs again, after one more synchronisation. Calls on one engine handle
 * must not overlap; separate handles are independent.
 *
 * Each entry point names the reference interface it replaces (paths inside Jonsnow-willow/Rune).
 */
#ifndef RUNE_B200_H
#define RUNE_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. The Python layer maps them to the reference's exception classes. */
#define RUNE_OK 0
#define RUNE_ERR_INVALID 1            /* bad argument or model definition  -> ValueError   */
#define RUNE_ERR_CUDA 2               /* CUDA runtime failure              -> RuntimeError */
#define RUNE_ERR_NEIGHBOR_OVERFLOW 3  /* neighbour count > max_neighbors   -> ValueError   */
#define RUNE_ERR_TYPE 4               /* atom type outside the model       -> ValueError   */
#define RUNE_ERR_OOM 5                /* device allocation failed          -> MemoryError  */
#define RUNE_ERR_STATE 6              /* call order (e.g. compute before finalize)         */
#define RUNE_ERR_RETRY 7              /* halo call: repeat it on every rank (rows regrown)  */

/* Model families (rune/mobius/model.py:47 message_mode / message_layers; rune/nep/model.py:48) */
#define RUNE_NEP 0
#define RUNE_MOBIUS_LOCAL 1
#define RUNE_MOBIUS_MP 2
#define RUNE_MOBIUS_EQ 3

/* Activations (rune/mobius/layers.py:11-23) */
#define RUNE_ACT_TANH 0
#define RUNE_ACT_SILU 1
#define RUNE_ACT_GELU 2

/* ZBL modes (rune/mobius/zbl.py:68-90, rune/nep/zbl.py:68-95) */
#define RUNE_ZBL_NONE 0
#define RUNE_ZBL_UNIVERSAL 1
#define RUNE_ZBL_FLEXIBLE 2

/* compute flags (the batch keys compute_forces / compute_virial, rune/mobius/model.py:308) */
#define RUNE_FORCES 1
#define RUNE_VIRIAL 2

typedef struct rune_engine rune_engine;

/* Resolved model hyper-parameters: the `model_params` dictionary of a RUNE checkpoint after
 * rune/mobius/plugin.py:resolve_params (:194) or rune/nep/plugin.py:resolve_params (:35). */
typedef struct {
    int32_t kind;                 /* RUNE_NEP / RUNE_MOBIUS_*                          */
    int32_t n_types;              /* len(elements)                                     */
    double rc_radial, rc_angular; /* rcut_radial, rcut_angular (Angstrom)              */
    int32_t n_desc_radial, n_desc_angular, k_max_radial, k_max_angular, l_max;
    int32_t has_q222, has_q1111, has_q112, has_q123, has_q233, has_q134;
    int32_t max_neighbors_radial, max_neighbors_angular;
    int32_t nep_hidden;           /* NEP hidden_dims[0]                                */
    int32_t hidden_dim, ffn_dim, blocks, activation, message_layers, message_dim, pair_dim;
    int32_t message_groups, vector_channels, equivariant_channels, equivariant_l_max;
    int32_t message_basis_size;
    double message_cutoff, norm_eps;
    int32_t zbl_mode;
    double zbl_rc_inner, zbl_rc_outer;
} rune_model_config;

typedef struct {
    int64_t calls;            /* compute calls                              */
    int64_t neighbor_builds;  /* device neighbour-list builds               */
    int64_t last_edges;       /* directed edges of the last build (max rc)  */
    int64_t last_radial_edges, last_angular_edges;
    int64_t workspace_bytes;  /* device workspace currently held            */
    int64_t workspace_grows;  /* times the workspace had to grow            */
    int64_t kernel_launches;  /* device kernels launched by this engine     */
    int64_t tensor_core_layers; /* EQ layers whose edge products run on tcgen05 */
} rune_stats;

/* Create an engine for one model on CUDA device `device`.
 * Replaces the model construction in rune/mobius/plugin.py:load_model (:125-142) and
 * rune/nep/plugin.py:load_model (:62-81); the weights follow via rune_engine_set_tensor. */
int rune_engine_create(const rune_model_config* config, int device, rune_engine** out);

/* Register one parameter or buffer by its reference state_dict name (e.g.
 * "descriptor.radial.c_table", "residual_blocks.0.ffn.0.weight") with `count` float32 values
 * in the reference layout (host memory, copied). Also takes the derived table
 * "invariant_terms" ([n_terms, 6]: coef, output L, four moment indices, -1 = unused).
 * Replaces Module.load_state_dict in load_model (rune/mobius/plugin.py:140). */
int rune_engine_set_tensor(rune_engine* engine, const char* name, const float* host_data,
                           int64_t count);

/* Validate shapes, derive device layouts, upload. Must precede any compute call. */
int rune_engine_finalize(rune_engine* engine);

/* Energy / forces / virial for a batch of independent periodic structures, neighbour lists
 * built on the device (cell list, integer image shifts, pairs with |r| < max cutoff).
 * Replaces Calculator.calculate -> BatchBuilder.build -> model(batch)
 * (rune/mobius/interface/calculator.py:42-85, interface/batch.py:42-166,
 *  rune/mobius/model.py:307-393; NEP: rune/nep/interface, rune/nep/model.py:87-155).
 *   types_dev      int32 [n_atoms]            type index 0..n_types-1
 *   positions_dev  float64 [n_atoms, 3]       Cartesian, any image (wrapped internally)
 *   cells_host     float64 [n_structures, 9]  rows are the lattice vectors a, b, c
 *   pbc_host       uint8 [n_structures, 3]
 *   atom_ptr_host  int32 [n_structures + 1]   structure s owns atoms atom_ptr[s]..atom_ptr[s+1]-1
 *   energies_dev   float32 [n_atoms]          per-atom energies (may be NULL)
 *   energy_dev     float64 [n_structures]     total energy per structure
 *   forces_dev     float32 [n_atoms, 3]       if flags & RUNE_FORCES (else may be NULL)
 *   virial_dev     float64 [n_structures, 9]  if flags & RUNE_VIRIAL, row-major W_ab = -sum g_a r_b */
int rune_engine_compute(rune_engine* engine, int32_t n_atoms, int32_t n_structures,
                        const int32_t* types_dev, const double* positions_dev,
                        const double* cells_host, const uint8_t* pbc_host,
                        const int32_t* atom_ptr_host, int32_t flags, float* energies_dev,
                        double* energy_dev, float* forces_dev, double* virial_dev,
                        void* stream);

/* One rank's part of a spatial domain decomposition of one large structure (no reference
 * counterpart: the reference evaluates a structure on one device; its native evaluator plugs
 * into GPUMD, rune/mobius/src/mobius.cu:334-402, which owns the decomposition). The local
 * system is non-periodic: owned atoms first, then ghost atoms (periodic images included, as
 * positions) in shells by distance from the owned region: shell k = 1 .. n_shells - 1 holds the
 * ghosts within k radial cutoffs, the last shell those within one more max(radial, angular)
 * cutoff. n_shells = message layers + 1 (1 for NEP and Local Möbius). shell_end_host
 * [n_shells + 1] holds cumulative counts: shell_end[0] = owned atoms, shell_end[n_shells] =
 * n_atoms. cell_host [9] is a box used for binning only (atoms outside it are still found).
 * energy_dev [1] receives the owned atoms' energy; energies_dev [n_atoms] per-atom energies
 * (zero for ghosts); forces_dev [n_atoms, 3] and virial_dev [9] the derivatives of the owned
 * energy with respect to every local atom, so that summing ghost forces into their owners and
 * virials over ranks gives the whole structure's forces and virial. */
int rune_engine_compute_domain(rune_engine* engine, int32_t n_atoms, int32_t n_shells,
                               const int32_t* shell_end_host, const int32_t* types_dev,
                               const double* positions_dev, const double* cell_host,
                               int32_t flags, float* energies_dev, double* energy_dev,
                               float* forces_dev, double* virial_dev, void* stream);

/* Halo exchange hook of rune_engine_compute_halo. `rows` is a float32 device array of
 * [n_atoms, row_floats] in the local order of the call (owned atoms, then ghosts), `stream` the
 * call's stream (work enqueued by the hook must be ordered on it). op RUNE_HALO_FILL: every
 * ghost row receives its owner's row. op RUNE_HALO_REDUCE: every ghost row is added into its
 * owner's row, then the ghost rows are set to zero. Returns 0 on success. The hook is called
 * the same number of times, in the same order, on every rank of a decomposition. */
#define RUNE_HALO_FILL 0
#define RUNE_HALO_REDUCE 1
typedef int (*rune_halo_fn)(void* ctx, int32_t op, float* rows, int32_t row_floats,
                            void* stream);

/* One rank's domain of a spatial decomposition with per-layer halo exchange (no reference
 * counterpart; the reference evaluates a structure on one device). The local system is
 * non-periodic: the n_owned owned atoms, then ghost atoms (periodic images included, as
 * positions) within max(radial, angular) cutoff of the owned region. The descriptor, network
 * and every message layer run over the owned atoms only; the ghost rows of each layer's input
 * node state h and (EQ) direction state come from their owners through `halo` (FILL after the
 * stem and after each layer but the last), and in the backward pass the ghost rows of their
 * adjoints go back to their owners (REDUCE after each layer). Models: Local and EQ Möbius.
 * Outputs as rune_engine_compute_domain: energies of owned atoms, forces [n_atoms, 3] on every
 * local atom (ghost rows: partial forces, for the caller's reverse force halo), virial [9] of
 * this rank's part. A call first repeats itself without exchanges when its sizes changed, so
 * that no workspace regrowth happens between exchanges; a neighbour row overflow found at the
 * end returns RUNE_ERR_RETRY after every exchange (the caller repeats the call on all ranks). */
int rune_engine_compute_halo(rune_engine* engine, int32_t n_atoms, int32_t n_owned,
                             const int32_t* types_dev, const double* positions_dev,
                             const double* cell_host, int32_t flags, rune_halo_fn halo,
                             void* halo_ctx, float* energies_dev, double* energy_dev,
                             float* forces_dev, double* virial_dev, void* stream);

/* Same outputs from the reference's padded batch form (the dict consumed by
 * rune/mobius/model.py:forward :307 and rune/nep/model.py:forward :87): neighbour index rows
 * with -1 padding and per-slot Cartesian offsets already in the model dtype (float32).
 * Lists must be symmetric (each (i, j, off) has its (j, i, -off)), as every RUNE builder
 * produces; RUNE_ERR_INVALID otherwise.
 *   positions_dev          float32 [n_atoms, 3]
 *   radial_neighbors_dev   int64 [n_atoms, radial_width];  radial_offsets_dev float32 [.., 3]
 *   angular_neighbors_dev  int64 [n_atoms, angular_width]; angular_offsets_dev float32 [.., 3] */
int rune_engine_compute_padded(rune_engine* engine, int32_t n_atoms, int32_t n_structures,
                               const int32_t* types_dev, const float* positions_dev,
                               const int64_t* radial_neighbors_dev, int32_t radial_width,
                               const float* radial_offsets_dev,
                               const int64_t* angular_neighbors_dev, int32_t angular_width,
                               const float* angular_offsets_dev, const int32_t* atom_ptr_host,
                               int32_t flags, float* energies_dev, double* energy_dev,
                               float* forces_dev, double* virial_dev, void* stream);

/* rune_engine_compute_padded without any device allocation. No counterpart in the reference.
 * For callers that must not allocate GPU memory while they run: hosts whose memory pool owns
 * the whole device (an MD code or a serving process that reserves HBM up front) and forbids
 * libraries from taking more. Inputs, outputs and their meaning are those of
 * rune_engine_compute_padded, and like it the call synchronises `stream` twice (after the
 * padded row count and at the end). The call's scratch comes from one fixed array of
 * RUNE_STATIC_SCRATCH_BYTES in device memory that the library holds on every GPU where it is
 * loaded, until the process exits. Problems that need more scratch than that are rejected with
 * RUNE_ERR_INVALID and a message giving the bytes needed (roughly 2.7 KB per atom for NEP and
 * 15 KB per atom for Möbius Local, at OAM sizes). The first call on each device looks up the
 * array's device address (cudaGetSymbolAddress, with that device current) and caches it.
 * Every call reuses the same array, so calls that overlap on the GPU — on different
 * streams, engines or threads of one device — race and must be serialised by the caller. */
#define RUNE_STATIC_SCRATCH_BYTES (32ull << 20)
int rune_engine_compute_padded_static(rune_engine* engine, int32_t n_atoms,
                                      int32_t n_structures, const int32_t* types_dev,
                                      const float* positions_dev,
                                      const int64_t* radial_neighbors_dev, int32_t radial_width,
                                      const float* radial_offsets_dev,
                                      const int64_t* angular_neighbors_dev,
                                      int32_t angular_width, const float* angular_offsets_dev,
                                      const int32_t* atom_ptr_host, int32_t flags,
                                      float* energies_dev, double* energy_dev,
                                      float* forces_dev, double* virial_dev, void* stream);

/* Export the directed pair list of the last rune_engine_compute call as host int32 rows
 * (i, j, S0, S1, S2) within cutoff `which` (0 = radial, 1 = angular), in engine order.
 * `capacity` rows are available at `pairs_host`; *count receives the number of pairs.
 * The pair-set contract of rune/mobius/interface/batch.py:42-102 (ASE neighbor_list "ijS"). */
int rune_engine_neighbor_pairs(rune_engine* engine, int32_t which, int32_t* pairs_host,
                               int64_t capacity, int64_t* count);

/* Counters (rune/mobius/src/mobius.cuh:10-14 NeighborStats, kernels.cuh:68-72 ScratchStats). */
int rune_engine_stats(const rune_engine* engine, rune_stats* out);

/* Velocity-Verlet NVE of one structure, entirely on the device: n_steps steps of dt_fs, with a
 * Verlet-skin neighbour cache (candidate pairs within max(rc) + skin, rebuilt when an atom has
 * moved more than skin / 2 since the last build: the cache rule of the reference's native
 * evaluator, rune/mobius/src/mobius.cu:334-402, mobius_neighbor_check.py:24-83, used by the
 * MD engine it plugs into). positions_dev [N,3] (A, float64, unwrapped) and velocities_dev
 * [N,3] (A/fs, float64) are updated in place; masses_dev [N] in amu. energies_host, if not
 * null, receives n_steps + 1 rows (potential, kinetic) in eV, row 0 at the initial state;
 * forces_dev, if not null, the forces (eV/A) at the final positions; rebuilds_host, if not
 * null, the number of candidate-list builds. Synchronises `stream` a few times per step. */
int rune_md_nve(rune_engine* engine, int32_t n_atoms, const int32_t* types_dev,
                double* positions_dev, double* velocities_dev, const double* masses_dev,
                const double* cell_host, const uint8_t* pbc_host, double dt_fs, int32_t n_steps,
                double skin, double* energies_host, float* forces_dev, int64_t* rebuilds_host,
                void* stream);

/* Per-kernel timing (no reference counterpart; the reference only counts scratch and
 * neighbour reuse, rune/mobius/src/kernels.cuh:68-72). When enabled, every kernel launch is
 * bracketed by CUDA events on the launching stream and its device time is accumulated under
 * the kernel's name. rune_engine_kernel_stat returns entry `index` (0-based; RUNE_ERR_INVALID
 * past the end): its name, total milliseconds and launch count. */
int rune_engine_set_profiling(rune_engine* engine, int32_t enabled);
int rune_engine_kernel_stat(const rune_engine* engine, int32_t index, char* name_buf,
                            int32_t name_capacity, double* total_ms, int64_t* launches);
int rune_engine_reset_kernel_stats(rune_engine* engine);

/* Bound of the EQ kernels' in-kernel waits on weight copies and tensor-core completions, in
 * polls of the mbarrier (default RUNE_DEFAULT_WAIT_POLLS, about a second at most). A block whose
 * wait gives up sets an error flag, lets the copies it issued land, skips the rest of its work
 * and returns, and the call fails with RUNE_ERR_CUDA ("A device-side copy did not complete in
 * time") while the CUDA context stays usable. 0 makes every such wait give up at once: the
 * failure path can be exercised on healthy copies. No reference counterpart (its kernels do not
 * wait on copies). Takes effect at the next compute call. */
#define RUNE_DEFAULT_WAIT_POLLS 4194304u
int rune_engine_set_wait_polls(rune_engine* engine, uint32_t polls);

/* Check of the tcgen05 tensor-core GEMM kernel (no reference counterpart; the reference's
 * dense layers are cuBLAS Dgemm calls, rune/mobius/src/network.cu:140-160): c_host [M][N] =
 * a_host [M][K] b_host [K][N] on device `device` by the 128 x 64-tile kernel of dense_tc.cu
 * (exact-integer products: power-of-two row / column scales, four signed 7-bit digits per
 * value, int32 accumulation in TMEM, one rounding of the float64 combination). Host arrays,
 * row-major; 1 <= M <= 65536, 1 <= N <= 4096, 1 <= K <= 4096. */
int rune_tc_selftest(int32_t M, int32_t N, int32_t K, const float* a_host, const float* b_host,
                     float* c_host, int32_t device);

/* Release the engine and its device memory. */
void rune_engine_destroy(rune_engine* engine);

/* Message of the last failing call on this thread (rune/mobius/src/mobius.cu:16-18). */
const char* rune_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* RUNE_B200_H */
