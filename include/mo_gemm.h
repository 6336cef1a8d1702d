#ifndef MO_GEMM_H_
#define MO_GEMM_H_
/*
 * C ABI of libmo_gemm.so: the sm_100a BF16 GEMM behind the reference's kernel_api.h, plus
 * the N-sharded multi-GPU driver.  Plain pointers and sizes only, so that ctypes (or any
 * other FFI) can bind it; no C++ or torch types cross this boundary and no exception
 * escapes it.  Every entry point returns 0 on success or a negative MO_ERR_* code;
 * mo_error_string() turns the code into text.
 *
 * Matrices are row-major BF16 stored as raw uint16_t bit patterns, with leading dimensions
 * implied by the shape (lda = k, ldb = n, ldc = n), exactly as in the reference ABI
 * (include/kernel_api.h:9).  Device pointers belong to the caller.  The shapes that take the
 * K split or the stream-K schedule draw a workspace from a pool the library keeps per device
 * (mo_release_workspace returns it); the hero shape allocates nothing.
 */

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  MO_OK = 0,
  MO_ERR_NULL_POINTER = -1,   /* a required pointer is NULL                          */
  MO_ERR_BAD_DIMS = -2,       /* m, n or k is not positive, or a size overflows      */
  MO_ERR_UNSUPPORTED = -3,    /* layout the call cannot take (see each call)          */
  MO_ERR_LAUNCH = -4,         /* the CUDA launch (or a CUDA runtime call) failed      */
  MO_ERR_DEVICE = -5,         /* no sm_100 device, or the device query failed         */
  MO_ERR_BAD_ARGUMENT = -6,   /* any other invalid argument (shard count, slab width) */
  MO_ERR_DEVICE_TIMEOUT = -7, /* a kernel's bounded wait expired (watchdog flag set)  */
  MO_ERR_SCRATCH_LIMIT = -8,  /* too big for mo_launch_bf16_gemm_v1_noalloc's scratch  */
  MO_ERR_NO_MEMORY = -9       /* device memory for mo_gemm_from_host's buffers failed */
};

/* Text for an MO_* code (static storage, never NULL). */
const char* mo_error_string(int code);

/* Library version, major*10000 + minor*100 + patch. */
int mo_version(void);

/*
 * C = A·B on the current device, asynchronously on `stream` (a cudaStream_t, or NULL for
 * the legacy default stream).  Replaces matmul_optimizer::launch_bf16_gemm_v1
 * (reference include/kernel_api.h:10-17, src/kernels/bf16_gemm_v1.cu:2098-2180), which
 * returns bool; this twin returns an MO_* code so a ctypes caller learns why.
 *
 * Every shape with m, n, k > 0 runs on the tensor cores: tails in M, N and K are handled by
 * TMA out-of-bounds zero fill on the loads and a predicated epilogue.  The TMA descriptors
 * need 16-byte row strides and bases.  When k or n is not a multiple of 8, or a pointer is
 * off a 16-byte boundary, the call copies A and B into padded buffers from the library's pool
 * (k and n rounded up to multiples of 8, zero padding), runs the GEMM there and copies C back
 * (the reference takes its scalar fallback kernel for these layouts,
 * src/kernels/bf16_gemm_v1.cu:2173-2177).  Only a pointer at an odd address returns
 * MO_ERR_UNSUPPORTED.
 */
int mo_launch_bf16_gemm_v1(const uint16_t* a_bf16, const uint16_t* b_bf16, uint16_t* c_bf16,
                           int m, int n, int k, void* stream);

/* The same GEMM from HOST buffers: A [m,k], B [k,n] and C [m,n], row-major BF16 bits in host
 * memory (page-locked for the copies to overlap); k and n multiples of 8 (else
 * MO_ERR_UNSUPPORTED).  A is uploaded first.  B then goes up in
 * `slabs` column slabs (0 = the library's choice).  Each slab's GEMM starts when its columns
 * land, and each slab of C comes back while later slabs compute.  The uploads, GEMMs and
 * downloads run on three streams the library owns, so both PCIe directions and the tensor cores
 * work at once.  `stream` waits for the last download.  Device buffers come from the library's
 * pool (see mo_release_workspace).  C is bit-identical to mo_launch_bf16_gemm_v1 on device
 * copies of A and B.  Returns MO_ERR_NO_MEMORY when the device buffers cannot be had.  No
 * reference counterpart: the reference's runner copies A and B up and C down around the launch
 * (src/runner/main.cpp:469-491).  This entry point overlaps those copies. */
int mo_gemm_from_host(const uint16_t* a_host, const uint16_t* b_host, uint16_t* c_host, int m,
                      int n, int k, int slabs, void* stream);

/* mo_gemm_from_host with A already on the device (`a_dev`, 16-byte aligned), for example
 * gathered from the other ranks over NVLink: only B goes up and C comes down over PCIe, with
 * the same slab pipeline.  Work queued on `stream` before the call (the gather of A) completes
 * before the first slab GEMM reads A. */
int mo_gemm_b_from_host(const uint16_t* a_dev, const uint16_t* b_host, uint16_t* c_host, int m,
                        int n, int k, int slabs, void* stream);

/*
 * The same C = A·B, with the same bits as mo_launch_bf16_gemm_v1, for callers that cannot
 * allocate device memory during a call.  Examples: a plugin whose host application owns all
 * device memory through its own pool, where a cudaMalloc from inside the plugin fails or splits
 * that pool; or code that cannot pay for cudaMalloc's implicit synchronisation.  No counterpart
 * in the reference (its kernels need no scratch).
 *
 * It runs the K-split kernel, and keeps the FP32 partial products of the K chunks in one
 * fixed array inside the library.  Layouts that mo_launch_bf16_gemm_v1 runs through padded
 * copies (k or n not a multiple of 8, a pointer off a 16-byte boundary) need memory for the
 * copies, so this call returns MO_ERR_UNSUPPORTED for them.  That array is 32 MiB per GPU and is held from the
 * library's first use on that GPU until the process exits.  The call allocates and frees
 * nothing, neither with cudaMalloc nor with any allocating library routine.
 *
 * Limit: the partials take (number of K chunks) x m x n x 4 bytes.  Larger problems return
 * MO_ERR_SCRATCH_LIMIT without launching.  K up to 1856 is a single chunk; it needs no
 * scratch and runs the unsplit kernel.  The hero shape has 4 chunks, so m x n may reach 2 Mi
 * elements; for example m = 269 with n = 7776.
 *
 * The first call on a device sets up: it looks up the array's device address once, with that
 * device current, and sets kernel attributes.  Make that first call before any stream capture.
 * Every call reuses the same array and leaves its contents behind.  Each call overwrites every
 * partial it reads before reading it, so nothing has to be cleared.  Two calls that overlap
 * on the same GPU, for example on two streams, race on the array: the caller must order them.
 * If a bounded wait in the kernel expires, C may hold a sum over the previous call's partials
 * and still look plausible; mo_read_device_watchdog reports it.
 */
int mo_launch_bf16_gemm_v1_noalloc(const uint16_t* a_bf16, const uint16_t* b_bf16,
                                   uint16_t* c_bf16, int m, int n, int k, void* stream);

/* The launch configuration the library picks for a shape: no reference counterpart (the
 * reference hard-codes its tiles, src/kernels/bf16_gemm_v1.cu:2117-2166); exposed so tests
 * and the benchmark can report which kernel ran. */
typedef struct mo_gemm_plan {
  int block_m;       /* output rows per tile (per CTA pair when cta_group == 2)   */
  int block_n;       /* output columns per tile                                   */
  int block_k;       /* K elements per pipeline stage                             */
  int stages;        /* shared-memory pipeline depth                              */
  int cta_group;     /* 1: one CTA per tile, 2: a CTA pair per tile (cta_group::2)*/
  int num_tiles;     /* tiles covering C                                          */
  int grid;          /* CTAs launched (persistent: at most one per SM)            */
  int smem_bytes;    /* dynamic shared memory per CTA                             */
  int num_chunks;    /* K chunks of the two-level FP32 accumulation               */
  int split;         /* 1: chunks run as separate work units + an ordered reduce  */
  int stream_k;      /* 1: leftover tiles' chunks spread over all clusters         */
} mo_gemm_plan;

/* Pure host computation of the plan for an m×n×k GEMM on a GPU with `num_sms` SMs, after the
 * same overrides the launch honours (MO_GEMM_SPLIT, MO_GEMM_STREAMK, MO_GEMM_VARIANT,
 * MATMUL_FIXED_MAIN_TILE_N; an invalid value returns MO_ERR_BAD_ARGUMENT).  Needs no GPU; the
 * launcher uses the same functions with the device's SM count. */
int mo_gemm_select_plan(int m, int n, int k, int num_sms, mo_gemm_plan* out);

/*
 * N-sharding (no reference counterpart: the reference is single-GPU).  Column slab i of C
 * covers columns [slab_begin[i], slab_begin[i] + slab_n[i]) with
 * w = roundup16(ceil(n / g)), slab_begin[i] = i·w, slab_n[i] = min(w, n - i·w).
 * Writes g entries into each output array.  Pure host math.
 */
int mo_shard_partition(int n, int g, int* slab_begin, int* slab_n);

/*
 * Launches slab i of an N-sharded GEMM on devices[i], stream streams[i]: c_slabs[i][m, slab_n[i]]
 * = a[i][m, k] · b_slabs[i][k, slab_n[i]].  Each GPU reads only its own memory (A replicated,
 * B slab contiguous), so there is no reduction and no peer access.  The K accumulation order
 * is the same as the 1-GPU call, so every slab is bit-identical to the matching columns of
 * mo_launch_bf16_gemm_v1's output.  Restores the caller's current device before returning.
 */
int mo_gemm_nshard(int g, const int* devices, const uint16_t* const* a,
                   const uint16_t* const* b_slabs, uint16_t* const* c_slabs,
                   int m, int k, const int* slab_n, void* const* streams);

/*
 * Re-layout after an all-gather of C slabs (no reference counterpart): `gathered` holds g
 * blocks of `block_elems` elements; block i is a row-major [m, slab_n[i]] slab.  Writes the
 * row-major [m, sum(slab_n)] matrix `c`.  Device pointers on the current device.
 */
int mo_unshard_columns(const uint16_t* gathered, uint16_t* c, int g, int m,
                       const int* slab_n, int64_t block_elems, void* stream);

/* Reads (and when `clear` is nonzero, resets) the device-side watchdog flag of the current
 * device: 0 when no bounded wait of a library kernel has expired since the last clear, else
 * a code naming the wait.  Synchronises the device.  A launch returns before its kernel runs,
 * so an expired wait surfaces only here.  C is not valid after such a launch: a work unit that
 * gave up wrote nothing, and a K-split reduce then sums whatever its scratch held from an
 * earlier call (for mo_launch_bf16_gemm_v1_noalloc, the previous call's partials), which can
 * look plausible.  A caller that must not take a wrong C for a right one reads this flag after
 * synchronising. */
int mo_read_device_watchdog(int clear, int* flag_out);

/* The work units of the plan that mo_launch_bf16_gemm_v1 would run for this shape on a device
 * with `num_sms` SMs (MO_GEMM_SPLIT, MO_GEMM_STREAMK, MO_GEMM_VARIANT and
 * MATMUL_FIXED_MAIN_TILE_N are honoured), listed by the kernel's own schedule code compiled for
 * the host.  Seven ints per unit, in each cluster's execution order: cluster, position in the
 * cluster's sequence, M block, N block, first K chunk, end K chunk (exclusive) and stream-K
 * tile (-1 unless the unit is one piece of a split tile).  Writes the
 * first min(total, cap) units to `units` and the total to `count`.  Needs no GPU.  No reference
 * counterpart: it lets a test check on the host that a schedule covers every K chunk of every tile
 * exactly once. */
int mo_gemm_schedule(int m, int n, int k, int num_sms, int* units, int cap, int* count);

/* Returns to the device the memory that the library's workspace pool of the current device
 * holds, including the stream-K workspaces it keeps per stream; synchronises the device first.
 * The pool keeps what it has mapped between calls, so that a call after a synchronisation does
 * not map its workspace again; it only ever holds the largest workspaces calls have needed
 * (K-split partials, stream-K pieces).  `held_before`
 * (may be NULL) receives the bytes the pool held.  No reference counterpart: the reference's
 * launch allocates nothing (src/kernels/bf16_gemm_v1.cu). */
int mo_release_workspace(int64_t* held_before);

/* Launches a one-CTA self-test kernel whose mbarrier wait nobody completes; with a
 * `timeout_us` limit the wait expires, the kernel records it in the watchdog flag and
 * returns.  Lets a test check the bounded-wait path without faulting or hanging the GPU. */
int mo_selftest_wait_timeout(int timeout_us, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* MO_GEMM_H_ */
