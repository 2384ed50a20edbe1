/*
 * spmvb200.h — C ABI of libspmvb200.so, a CSR sparse matrix-vector product (y = A x) for NVIDIA B200
 * (sm_100a) with compressed column indices.
 *
 * It is a drop-in for the hot path of the spmv-index-compression study (HERMES-TorVerLab/
 * spmv-index-compression): the CSR reader, RCM reordering and characterization of include/csr.hpp,
 * include/rcm.hpp and src/characterize_matrix.cpp, the layout encoders and byte model of
 * src/bench_csr_width.cu:149-285 and :795-960, and the kernels and dispatch of
 * src/bench_csr_width.cu:287-629. Every declaration below names the reference interface it replaces.
 * That program has no library interface of its own; its de facto operator surface is
 * launch<T>(threads_per_row, Configuration, DeviceMatrix<T>) (bench_csr_width.cu:607).
 *
 * Conventions
 *   - Every function returns SPMV_OK (0) or a positive SPMV_ERR_* status; the reference calls exit()
 *     on any CUDA error (include/common.cuh:19-27), this library returns the status instead and keeps
 *     a message for spmv_last_error().
 *   - Layouts: CSR-i32, CSR-i16 (16-bit absolute), CSR-r16 (16-bit offset from the row's first column),
 *     CSR-lp (per-lane bit-packed difference chains), and the 8-bit i8/r8 of the same families.
 *   - threads per row T is in {2, 4, 8, 16, 32}; results are bit-identical to the reference CSR-i32
 *     kernel at the same T (same nonzero order, lane striding and shuffle-reduction order).
 *   - Value types FP64, FP32, FP16; FP16 accumulates in FP32 (include/value_types.cuh:9-13).
 *   - Ownership: the library owns the encoded operator buffers; the caller owns x and y.
 *     An operator may be used from several host threads as long as each call has its own stream
 *     and y; calls on one operator never write to the operator.
 *   - Streams are passed as void* (a cudaStream_t, NULL for the legacy default stream), so this header
 *     needs no CUDA include.
 */
#ifndef SPMVB200_H
#define SPMVB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status ----------------------------------------------------------------------------------- */
#define SPMV_OK 0
#define SPMV_ERR_INVALID_ARGUMENT 1
#define SPMV_ERR_IO 2                /* a file could not be opened, read or written */
#define SPMV_ERR_FORMAT 3            /* malformed Matrix Market or permutation file */
#define SPMV_ERR_NOT_ADMISSIBLE 4    /* the layout cannot represent this matrix exactly */
#define SPMV_ERR_OUT_OF_MEMORY 5     /* host or device allocation failed */
#define SPMV_ERR_CUDA 6              /* a CUDA runtime call failed */
#define SPMV_ERR_UNSUPPORTED 7       /* e.g. no CUDA device, or a library that is missing */
#define SPMV_ERR_NCCL 8              /* an NCCL call failed or NCCL could not be loaded */
#define SPMV_ERR_TIMEOUT 9           /* a bounded device-side wait gave up (see spmv_operator_check) */
#define SPMV_ERR_TOO_LARGE 10        /* a size exceeds a documented limit */

/* ---- enums -------------------------------------------------------------------------------------- */
/* Column layouts (the Configuration of bench_csr_width.cu:88 as column_mode x column_bytes). */
#define SPMV_LAYOUT_I32 0   /* absolute, 4 bytes                              */
#define SPMV_LAYOUT_I16 1   /* absolute, 2 bytes: admissible iff cols <= 2^16  */
#define SPMV_LAYOUT_R16 2   /* row-base, 2-byte offsets: every row spans < 2^16 */
#define SPMV_LAYOUT_LP  3   /* lane-packed difference chains (depends on T)   */
#define SPMV_LAYOUT_I8  4   /* absolute, 1 byte: cols <= 256                   */
#define SPMV_LAYOUT_R8  5   /* row-base, 1-byte offsets: every row spans < 256 */

/* Value types (PrecisionName, include/value_types.cuh:37-40). */
#define SPMV_F64 0
#define SPMV_F32 1
#define SPMV_F16 2

/* ---- library ------------------------------------------------------------------------------------ */
const char* spmv_version(void);
const char* spmv_status_string(int status);
/* Message of the last failing call on this host thread ("" if none). */
const char* spmv_last_error(void);

/* ---- host CSR matrix: CsrMatrix (include/csr.hpp:33) -------------------------------------------- */
typedef struct spmv_csr spmv_csr;

/* MatrixStats (include/csr.hpp:22) plus the shape. */
typedef struct {
  int rows;
  int cols;
  int64_t nnz;
  double nnz_per_row_mean;
  int nnz_per_row_max;
  int nnz_per_row_min;
  double nnz_per_row_std;
  double dynamic_range;
  double norm_inf;
  double max_abs;
  double min_abs;
  int symmetric_expanded;
} spmv_csr_info;

/* read_matrix_market (include/csr.hpp:232): coordinate real/integer/pattern, general/symmetric/
 * skew-symmetric/hermitian, symmetric files expanded, columns sorted within rows, stats computed.
 * Errors: SPMV_ERR_IO (cannot open), SPMV_ERR_FORMAT (not Matrix Market, not coordinate, bad size). */
int spmv_csr_read_matrix_market(const char* path, spmv_csr** out);

/* A CsrMatrix from caller arrays (copied). Columns are sorted within rows as sort_columns_within_rows
 * (include/csr.hpp:162) does and the stats are computed (CsrMatrix::compute_stats, csr.hpp:43).
 * values may be NULL (all 1.0). name may be NULL. nnz = row_ptr[rows] must fit int32, as in the
 * reference. */
int spmv_csr_create(int rows, int cols, const int* row_ptr, const int* col_ind, const double* values,
                    const char* name, spmv_csr** out);
int spmv_csr_get_info(const spmv_csr* matrix, spmv_csr_info* info);
/* Borrowed pointers to the host arrays, valid until spmv_csr_destroy. */
int spmv_csr_get_arrays(const spmv_csr* matrix, const int** row_ptr, const int** col_ind, const double** values);
const char* spmv_csr_name(const spmv_csr* matrix);
int spmv_csr_set_name(spmv_csr* matrix, const char* name);
void spmv_csr_destroy(spmv_csr* matrix);

/* Rows [row_begin, row_end) as a matrix of their own with all columns kept (a row shard). */
int spmv_csr_slice_rows(const spmv_csr* matrix, int row_begin, int row_end, spmv_csr** out);

/* ---- RCM ordering: include/rcm.hpp -------------------------------------------------------------- */
/* reverse_cuthill_mckee (rcm.hpp:199): new_to_old[rows]; square matrices only. */
int spmv_rcm_order(const spmv_csr* matrix, int* new_to_old);
/* apply_symmetric_permutation (rcm.hpp:219): B = P A P^T, columns re-sorted, stats recomputed. */
int spmv_csr_permute(const spmv_csr* matrix, const int* new_to_old, spmv_csr** out);
/* permutation_path_for (rcm.hpp:244): "<stem>.<ordering>.perm". Writes at most cap bytes with the NUL. */
int spmv_permutation_path(const char* matrix_path, const char* ordering, char* out, size_t cap);
/* write_permutation (rcm.hpp:250): magic "RCMPERM1", int64 rows, double seconds, int32 new_to_old;
 * written to "<path>.partial" and renamed. */
int spmv_permutation_write(const char* path, const int* new_to_old, int64_t rows, double seconds);
/* read_permutation (rcm.hpp:274): *found = 0 when the file does not exist; SPMV_ERR_FORMAT when it
 * exists but is not a valid permutation of expected_rows entries. */
int spmv_permutation_read(const char* path, int expected_rows, int* new_to_old, double* seconds, int* found);
/* reorder_with_rcm (rcm.hpp:306): loads <stem>.rcm.perm beside matrix_path, or computes and saves it;
 * returns P A P^T and the seconds the ordering took when it was computed. */
int spmv_csr_reorder_rcm(const char* matrix_path, const spmv_csr* matrix, spmv_csr** out, double* seconds);

/* ---- characterization: src/characterize_matrix.cpp ---------------------------------------------- */
/* The 60-column CSV of write_csv (characterize_matrix.cpp:253), header line and value line, for the
 * FP64 byte model. ordering is "original" or "rcm". *needed receives the bytes required (with NUL);
 * SPMV_ERR_TOO_LARGE if cap is smaller. Requires a square matrix with nnz > 0 (characterize main:314). */
int spmv_characterize(const spmv_csr* matrix, const char* ordering, double ordering_seconds, char* csv,
                      size_t cap, size_t* needed);
/* The same CSV computed on the GPU (device ordinal, -1 = current): the per-row metrics (spans, bandwidth,
 * 8/16-bit fits, lane occupancy, windowed segments, uncached gathers) by one thread per row, the span
 * percentiles by a radix select on the device; the FIFO gather model, sequential by definition, as twelve
 * host threads beside the GPU. Byte for byte spmv_characterize's output. No counterpart in the reference
 * (its tool runs on the host, characterize_matrix.cpp:92-251). */
int spmv_characterize_device(const spmv_csr* matrix, const char* ordering, double ordering_seconds, int device,
                             char* csv, size_t cap, size_t* needed);

/* ---- layouts, admissibility and byte model: src/bench_csr_width.cu:149-285 ------------------------ */
/* MatrixFacts (bench_csr_width.cu:160): widest row span and the CSR-lp word counts by log2(T). */
typedef struct {
  int widest_row_span;
  int64_t lane_packed_words[6];   /* [log2 T], T = 2..32 in slots 1..5, each including the 2 spare words */
} spmv_facts;

/* MemoryBreakdown (bench_csr_width.cu:95): bytes of every stream one product touches. */
typedef struct {
  double values;
  double columns;
  double column_bases;
  double row_pointer;
  double vectors;
  double total;
} spmv_memory;

/* facts_of (bench_csr_width.cu:223). */
int spmv_matrix_facts(const spmv_csr* matrix, spmv_facts* facts);
/* configuration_admissible (bench_csr_width.cu:246); tpr matters for CSR-lp only (0 means 8). */
int spmv_admissible(const spmv_csr* matrix, const spmv_facts* facts, int layout, int tpr, int* admissible);
/* memory_of (bench_csr_width.cu:258); tpr matters for CSR-lp only (0 means 8). */
int spmv_memory_of(const spmv_csr* matrix, const spmv_facts* facts, int layout, int dtype, int tpr, spmv_memory* memory);

/* Host encoders, producing the reference's exact streams.
 * upload_columns<T, I> (bench_csr_width.cu:796): absolute columns narrowed to 2 (i16) or 1 (i8) bytes. */
int spmv_encode_absolute(const spmv_csr* matrix, int column_bytes, void* columns);
/* upload_row_bases (bench_csr_width.cu:807): first column of each row, 0 for an empty row. */
int spmv_encode_row_base(const spmv_csr* matrix, int* row_base);
/* upload_relative_columns<I> (bench_csr_width.cu:820): col - row base in 2 (r16) or 1 (r8) bytes. */
int spmv_encode_relative(const spmv_csr* matrix, int column_bytes, void* offsets);
/* upload_lane_major_offsets (bench_csr_width.cu:838, control builds SPMV_R16_LANE/PAIR): the 16-bit
 * row-relative offsets of every row in lane-major order for tpr, (nnz + 1) / 2 * 2 entries (the last one zero
 * when nnz is odd). column_bytes 4 in spmv_encode_relative gives SPMV_R16_WIDE's 32-bit offsets (:944). */
int spmv_encode_relative_lane(const spmv_csr* matrix, int tpr, uint16_t* offsets);
/* packed_word_count (bench_csr_width.cu:206). */
int spmv_lane_packed_word_count(const spmv_csr* matrix, int tpr, int64_t* word_count);
/* build_packed_deltas (bench_csr_width.cu:861): row_word[rows], row_width[rows], words[word_count]. */
int spmv_encode_lane_packed(const spmv_csr* matrix, int tpr, int64_t word_count, int* row_word, uint8_t* row_width,
                            uint32_t* words);
/* build_packed_deltas (bench_csr_width.cu:861) on the GPU, from device-resident row_ptr (int32[rows+1])
 * and col_ind (int32[nnz], sorted within rows): the same row_word, row_width and words as
 * spmv_encode_lane_packed. Call with words NULL to get word_count (2 spare words included) and the row
 * arrays; call again with words of word_capacity >= word_count to pack. Synchronises the stream. */
int spmv_encode_lane_packed_device(const int* row_ptr, const int* col_ind, int rows, int tpr, int* row_word,
                                   uint8_t* row_width, uint32_t* words, int64_t word_capacity, int64_t* word_count,
                                   void* stream);
/* The same encoding without allocating any device memory, for callers that must not allocate while they
 * encode: a framework whose own caching allocator owns every device byte, code that reserves its memory up
 * front under a fixed budget, loops that cannot stall on cudaMalloc/cudaFree. No counterpart in the
 * reference (its encoder runs on the host). Limits: rows at most 2^26 (SPMV_ERR_TOO_LARGE above); the
 * scratch is a fixed 512 KiB array inside the library, held on every GPU that loads it until the process
 * exits. The first call on a device, and the first after that device's context was reset
 * (cudaDeviceReset), looks up that array's address on the device (make that first call before any stream
 * capture). All calls share the array, so calls that overlap on the GPU (other streams, other host
 * threads) race on it; nothing in it needs clearing between calls. Synchronises the stream. Same
 * arguments, results and two-call use as spmv_encode_lane_packed_device. */
int spmv_encode_lane_packed_device_noalloc(const int* row_ptr, const int* col_ind, int rows, int tpr, int* row_word,
                                           uint8_t* row_width, uint32_t* words, int64_t word_capacity,
                                           int64_t* word_count, void* stream);

/* ---- device operator: DeviceMatrix<T> + Configuration (bench_csr_width.cu:88, :128) ------------- */
typedef struct spmv_operator spmv_operator;

typedef struct {
  int layout;
  int dtype;
  int tpr;                /* T: threads per row of the summation order, 2..32                       */
  int physical_tpr;       /* threads of the kernel per row, dividing T (0 = chosen by the library)  */
  int tile_nnz;           /* nonzeros staged per tile (0 = default)                                  */
  int value_rounding;     /* 0: values (T)(float)val as upload_matrix does (:927); 1: (T)val          */
  int device;             /* CUDA device ordinal (-1 = current device)                               */
  int stages;             /* shared-memory tile buffers per CTA, 1..4 (0 = default)                  */
  int tile_rows;          /* rows a tile holds at most, a multiple of 16 (0 = chosen by the library)  */
  int schedule;           /* SPMV_SCHEDULE_*: how rows are mapped to the kernel (0 = chosen by the library) */
  int accumulate;         /* SPMV_ACCUMULATE_*: the type FP16 values are summed in (0 = FP32)             */
} spmv_operator_config;

/* The type a product sums in. WIDE: FP64 values in FP64, FP32 and FP16 values in FP32 (AccumulatorOf,
 * value_types.cuh:9-13; the reference's campaign build). HALF: FP16 values summed in FP16, one __hfma
 * per entry and one __hadd per step of the lane tree, the reference's SPMV_HALF_ACCUMULATE control
 * build (value_types.cuh:7-33, CMakeLists.txt:32); FP16 operators only. */
enum { SPMV_ACCUMULATE_WIDE = 0, SPMV_ACCUMULATE_HALF = 1 };

/* Row schedules. Tiles: runs of consecutive rows staged in shared memory (rows of similar lengths).
 * Classes: rows grouped by length, each group on its own thread mapping straight from global memory
 * (skewed row lengths, such as power-law graphs). Both give the same results. */
enum { SPMV_SCHEDULE_AUTO = 0, SPMV_SCHEDULE_TILES = 1, SPMV_SCHEDULE_CLASSES = 2 };

/* Fills a config with defaults: physical_tpr 0, tile_nnz 0, value_rounding 0, device -1, stages 0,
 * tile_rows 0, schedule SPMV_SCHEDULE_AUTO, accumulate SPMV_ACCUMULATE_WIDE. */
void spmv_operator_config_init(spmv_operator_config* config, int layout, int dtype, int tpr);

/* upload_matrix + upload_* (bench_csr_width.cu:795-951): encodes the matrix in the layout, converts
 * the values, plans the tiles and uploads everything to the device. SPMV_ERR_NOT_ADMISSIBLE when the
 * layout cannot hold the matrix exactly (reported as "not admissible" by the reference, :1198). */
int spmv_operator_create(const spmv_csr* matrix, const spmv_operator_config* config, spmv_operator** out);

typedef struct {
  int rows;
  int cols;
  int64_t nnz;
  int layout;
  int dtype;
  int tpr;
  int physical_tpr;
  int tile_nnz;
  int64_t tiles;             /* staged tiles of short rows                                   */
  int64_t tile_ctas;         /* persistent CTAs over the tiles                               */
  int stages;                /* shared-memory tile buffers per CTA                           */
  int tile_rows;             /* rows a tile holds at most                                    */
  int64_t long_rows;         /* rows longer than a tile, streamed by the long-row path       */
  int64_t device_bytes;      /* bytes of device memory the operator holds                    */
  spmv_memory memory;        /* memory_of of this layout at this T (algorithmic bytes/product) */
  int schedule;              /* SPMV_SCHEDULE_TILES or SPMV_SCHEDULE_CLASSES                 */
  int64_t listed_rows;       /* classes: rows of more than 8 entries on groups of P threads  */
  int64_t blocks;            /* CTAs of one launch                                           */
  int window_elements;       /* tiles: x elements a tile stages for its gathers (0: none)    */
} spmv_operator_info;
int spmv_operator_get_info(const spmv_operator* op, spmv_operator_info* info);

/* launch<T> (bench_csr_width.cu:607): y = A x on the given stream, x and y device pointers of the
 * operator's value type (x: cols entries, y: rows entries). Asynchronous; launch errors are returned. */
int spmv_operator_run(const spmv_operator* op, const void* x, void* y, void* stream);
/* The same product through host buffers: copies x to the device, multiplies, copies y back and waits
 * (result_at_fixed_tpr, bench_csr_width.cu:779). x_device and y_device are caller scratch on the device. */
int spmv_operator_run_host(const spmv_operator* op, const void* x_host, void* y_host, void* x_device, void* y_device,
                           void* stream);
/* A stream of products through host buffers: y_i = A x_i for i < count, x_i at x_host + i * x_stride bytes and
 * y_i at y_host + i * y_stride (a stride of 0 reuses one buffer). The copy of x_{i+1} to the device, the
 * product of x_i and the copy of y_{i-1} back overlap (the given stream and two internal ones); x_device and
 * y_device are caller scratch for two vectors each, the second at an offset of the first's bytes rounded up
 * to 16. Host buffers must be pinned for the copies to overlap. Returns when every y_i is on the host. */
int spmv_operator_run_host_batch(const spmv_operator* op, const void* x_host, int64_t x_stride, void* y_host,
                                 int64_t y_stride, int count, void* x_device, void* y_device, void* stream);
/* Reads and clears the operator's device status word: SPMV_ERR_TIMEOUT if a bounded device-side wait
 * gave up since the last check. Synchronises the device. */
int spmv_operator_check(const spmv_operator* op);
/* Device pointers of the encoded streams (for callers that launch on their own arrays). */
typedef struct {
  const int* row_ptr;
  const void* columns;
  const int* row_base;
  const int* row_word;
  const uint8_t* row_width;
  const uint32_t* words;
  const void* values;
} spmv_operator_arrays;
int spmv_operator_get_arrays(const spmv_operator* op, spmv_operator_arrays* arrays);
void spmv_operator_destroy(spmv_operator* op);

/* ---- raw launch over caller-owned device arrays ------------------------------------------------- */
/* The DeviceMatrix<T> of bench_csr_width.cu:128 restricted to one layout. */
typedef struct {
  int rows;
  int cols;
  int64_t nnz;
  const int* row_ptr;       /* int32[rows + 1]                                         */
  const void* columns;      /* i32: int32, i16/r16: uint16, i8/r8: uint8 [nnz]; lp: unused */
  const int* row_base;      /* r16/r8/lp: int32[rows]                                  */
  const int* row_word;      /* lp: int32[rows]                                         */
  const uint8_t* row_width; /* lp: uint8[rows]                                         */
  const uint32_t* words;    /* lp: uint32[word_count], with its 2 spare words          */
  const void* values;       /* value type [nnz]                                        */
  const void* x;            /* value type [cols]                                       */
  void* y;                  /* value type [rows]                                       */
} spmv_device_matrix;
/* launch<T> (bench_csr_width.cu:607-629) on caller arrays: one vector of T threads per row, no
 * preprocessing and no workspace. */
int spmv_launch(int layout, int dtype, int tpr, const spmv_device_matrix* matrix, void* stream);

/* The reference's CSR-r16 control builds (bench_csr_width.cu:34-42, :343-432, CMakeLists.txt:36-47), each
 * changing only how the offsets reach its global-memory r16 kernel, on caller arrays like spmv_launch:
 * LANE reads matrix->columns as the lane-major stream for tpr (spmv_encode_relative_lane), PAIR the same
 * stream two offsets to a 32-bit load (4-byte aligned), WIDE as 32-bit offsets (spmv_encode_relative with
 * column_bytes 4), UNROLL16 as the 16-bit offsets with the loop unrolled 16 times at FP16. row_ptr,
 * row_base, values, x and y as for CSR-r16. The results are CSR-i32's bits at the same tpr. */
enum { SPMV_R16_CONTROL_LANE = 1, SPMV_R16_CONTROL_PAIR = 2, SPMV_R16_CONTROL_WIDE = 3, SPMV_R16_CONTROL_UNROLL16 = 4 };
int spmv_launch_r16_control(int control, int dtype, int tpr, const spmv_device_matrix* matrix, void* stream);

/* measure_read_bandwidth (include/roofline.cuh:101): the median bandwidth of a pure streaming read of a
 * `bytes`-byte device buffer (16-byte vector loads, no reuse), over `reps` timed passes after 3 warm-ups,
 * on the current device. The roof of the reference's epsilon. */
int spmv_read_bandwidth(int64_t bytes, int reps, double* gigabytes_per_second);
/* The ceiling of random x gathers: the median rate (elements per second) of reads of single elements of
 * value_bytes (2, 4 or 8) at pseudo-random positions of an array of `elements` elements, with every
 * multiprocessor busy. No counterpart in the reference (its roofline is the streaming read above); it
 * bounds SpMV on matrices whose columns are scattered, where each x element costs a 32-byte sector. */
int spmv_gather_rate(int64_t elements, int value_bytes, int reps, double* elements_per_second);

/* ---- synthetic matrices for the benchmark configurations ---------------------------------------- */
/* 2D 5-point Laplacian on grid x grid (diagonal 4, neighbours -1). */
int spmv_synth_laplacian2d(int grid, spmv_csr** out);
/* n x n band: each row k ~ Poisson(mean) (at least 1) distinct off-diagonal columns uniform in
 * [row - half_bandwidth, row + half_bandwidth], plus the diagonal; values N(0,1). */
int spmv_synth_random_band(int n, int half_bandwidth, double mean, uint64_t seed, spmv_csr** out);
/* 3D 27-point stencil on grid^3 in lexicographic order (diagonal 26, neighbours -1). */
int spmv_synth_stencil27(int grid, spmv_csr** out);
/* n x n power law: row lengths Zipf(alpha) clipped to [1, max_length] and rescaled to the given mean,
 * columns uniform over [0, n) without repeats in a row, values uniform [-1, 1]. */
int spmv_synth_power_law(int n, double alpha, int max_length, double mean, uint64_t seed, spmv_csr** out);
/* Rows [row_begin, row_end) of an n x n block matrix of block x block dense blocks: every block row
 * holds its diagonal block and blocks_per_row - 1 more at distinct block offsets uniform within
 * +-offset_range rows; values N(0,1) and a diagonally dominant diagonal. Any row range can be built on
 * its own (a shard), identical to the same rows of the whole matrix. */
int spmv_synth_block_fem(int n, int block, int blocks_per_row, int offset_range, uint64_t seed, int row_begin,
                         int row_end, spmv_csr** out);
/* count values uniform in [-1, 1] from seed, stored as dtype ((T)(float)u, as the reference casts x,
 * bench_csr_width.cu:928). The same seed gives the same values for every dtype. */
int spmv_fill_uniform(int dtype, int64_t count, uint64_t seed, void* out);
/* The reference's own x: std::mt19937(7), uniform_real_distribution<double>(-1, 1), cast through float
 * (upload_matrix, bench_csr_width.cu:923-928). */
int spmv_fill_reference_x(int dtype, int64_t count, void* out);

/* ---- multi-GPU: nnz-balanced row shards, x replicated, y all-gathered into the next x ------------ */
/* Row boundaries of nshards row blocks balanced by nonzeros: row_begin[0] = 0, row_begin[nshards] = rows. */
int spmv_shard_rows(const spmv_csr* matrix, int nshards, int* row_begin);

/* An NCCL communicator over the ranks of one job (NCCL is loaded at run time). */
typedef struct spmv_comm spmv_comm;
/* 128 bytes (ncclUniqueId) to be broadcast from rank 0 to the others by the caller. */
int spmv_comm_unique_id(void* id128);
int spmv_comm_create(int nranks, int rank, const void* id128, int device, spmv_comm** out);
void spmv_comm_destroy(spmv_comm* comm);

/* Waits until the stream's work is done or a collective failed, for at most timeout_ms. On an NCCL
 * error (SPMV_ERR_NCCL) or the timeout (SPMV_ERR_TIMEOUT) the communicator is marked aborted and
 * spmv_comm_destroy aborts it instead of waiting for the other ranks. */
int spmv_comm_check(spmv_comm* comm, void* stream, int timeout_ms);

/* End-to-end products of a row shard from host memory with x split over the ranks: for each of count
 * vectors (x_host + i * x_stride bytes, cols entries; y_host + i * y_stride bytes, the shard's rows) every
 * rank copies its slice of x (ceil(cols / nranks) entries from rank * that) in from host memory, the
 * slices are all-gathered in place (one ncclAllGather), the shard's product runs, and its rows of y go
 * out to host memory; vectors overlap as in spmv_operator_run_host_batch. x_device: two buffers of
 * nranks * ceil(cols / nranks) entries, each rounded up to 16 bytes; y_device: two of the shard's rows,
 * likewise. Waits for its streams (at most 120 s for the collectives, then SPMV_ERR_TIMEOUT and the
 * communicator is aborted). All ranks call it with the same count. No counterpart in the reference (its
 * benchmark runs on one GPU). */
int spmv_shard_run_host_batch(const spmv_operator* shard_op, spmv_comm* comm, const void* x_host, int64_t x_stride,
                              void* y_host, int64_t y_stride, int count, void* x_device, void* y_device, void* stream);

/* Chained products y -> x over the row shards: each rank holds the operator of its rows
 * (shard_row_begin[rank] .. shard_row_begin[rank+1]) and the full x. Every product computes the rank's y
 * shard into its slice of the next x, then all-gathers the slices over NCCL, products times. x_current
 * and x_next are device buffers of cols entries (the square matrix's n); the result is left in x_current
 * if products is even, else in x_next. All ranks must call it with the same products. */
int spmv_chain_run(const spmv_operator* shard_op, spmv_comm* comm, const int* shard_row_begin, void* x_current,
                   void* x_next, int products, void* stream);

/* Chained products over interleaved row blocks, each block round's all-gather beside the next block's
 * product. The square matrix's n = nranks * blocks_per_rank * block_rows rows are cut into blocks of
 * block_rows; rank r holds block_ops[c] for block c * nranks + r (c = 0 .. blocks_per_rank-1), each an
 * operator of block_rows rows and n columns. Every product runs the rank's blocks in order into their
 * places in the next x; the round of blocks c * nranks .. c * nranks + nranks - 1 is all-gathered in
 * place on a stream of the communicator's own while block c + 1 computes, and the products leave a few
 * multiprocessors to those collectives. Results are those of spmv_chain_run; x_current, x_next, the
 * parity of products and the stream mean the same; after an error both x buffers are undefined (the
 * call returns only once the collectives it queued have finished). No counterpart in the reference (its
 * benchmark is single-GPU). */
int spmv_chain_run_blocks(const spmv_operator* const* block_ops, int blocks_per_rank, int block_rows,
                          spmv_comm* comm, void* x_current, void* x_next, int products, void* stream);

/* ---- chained products over peer memory (the all-gather inside the product) ---------------------------
 * No counterpart in the reference (its benchmark runs on one GPU). A peer group is one rank's share of a
 * job of nranks processes, one GPU each, on one node whose GPUs reach each other's memory (NVLink):
 * every rank allocates two x buffers and a block of barrier flags in one allocation, exports it
 * (spmv_peer_group_handle, 64 bytes), the caller gathers every rank's handle in rank order (e.g. an
 * all-gather over torch.distributed) and every rank maps the others' (spmv_peer_group_open). A chained
 * product on rank r multiplies its row shard into its rows of the next x and stores those rows into
 * every other rank's next x as well (stores over NVLink from the product kernel, no collective library),
 * then waits at a barrier between the ranks' GPUs (flags in peer memory; each wait bounded by
 * timeout_ms, after which the group's status word records the timeout and spmv_peer_group_check returns
 * SPMV_ERR_TIMEOUT). Results equal spmv_chain_run's. Every rank must make the same calls in the same
 * order (products, barriers); destroy a group only once no rank still runs products into it. */
#define SPMV_PEER_HANDLE_BYTES 64
typedef struct spmv_peer_group spmv_peer_group;
/* At most 16 ranks; x_bytes: the bytes of one x (n entries of the operators' value type). The buffers
 * start zeroed. */
int spmv_peer_group_create(int nranks, int rank, int64_t x_bytes, int device, spmv_peer_group** out);
/* This rank's allocation exported for the other ranks: SPMV_PEER_HANDLE_BYTES bytes into handle. */
int spmv_peer_group_handle(const spmv_peer_group* group, void* handle);
/* Maps the other ranks' allocations: handles holds nranks handles in rank order (this rank's is skipped). */
int spmv_peer_group_open(spmv_peer_group* group, const void* handles);
/* Device pointer of this rank's current x (which = 0: the next product's input, and after a run the
 * latest result) or of the other buffer (which = 1). Write x0 into the current x before the first run. */
int spmv_peer_group_x(const spmv_peer_group* group, int which, void** x);
/* Copies bytes from buffer (host or device memory) into this rank's current x (direction 0), or from the
 * current x into buffer (direction 1), on the stream, and waits for the copy. */
int spmv_peer_group_copy_x(spmv_peer_group* group, int direction, void* buffer, int64_t bytes, void* stream);
/* A barrier of the ranks' GPUs on the stream, each wait at most timeout_ms. Before spmv_peer_group_open it
 * only waits (no other rank can be told), so it ends in a timeout on more than one rank. */
int spmv_peer_group_barrier(spmv_peer_group* group, int timeout_ms, void* stream);
/* Synchronises the device and reads the group's status word: SPMV_ERR_TIMEOUT if a barrier gave up (the
 * group then refuses further runs; its buffers are undefined). */
int spmv_peer_group_check(spmv_peer_group* group);
/* Halo mode for this rank's row shard (the spmv_csr of its rows, cols = n): lists the entries of x that other
 * ranks own and these rows read (runs split per owner). Chained products then store nothing into the
 * peers; after each product's barrier this rank pulls just those entries of the next x from their
 * owners' memory. Each rank's x buffers then hold its own rows and the entries its rows read; the other
 * entries are not kept up to date. Call before the first spmv_chain_run_peer of this shard. */
int spmv_peer_group_set_halo(spmv_peer_group* group, const spmv_csr* shard, const int* shard_row_begin);
/* The number of x entries the halo pulls each product (-1 when no halo is set). */
int spmv_peer_group_halo_entries(const spmv_peer_group* group, int64_t* entries);
/* products chained products y -> x over the row shards (shard_row_begin[0..nranks], the rank's operator
 * holding rows shard_row_begin[rank] .. shard_row_begin[rank+1] of the square matrix): one barrier, then
 * per product the fused product and a barrier. The current x advances by products. */
int spmv_chain_run_peer(const spmv_operator* shard_op, spmv_peer_group* group, const int* shard_row_begin, int products,
                        int timeout_ms, void* stream);
void spmv_peer_group_destroy(spmv_peer_group* group);

#ifdef __cplusplus
}
#endif

#endif /* SPMVB200_H */
