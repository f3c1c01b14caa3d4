/* libtarscuda - the tars_mini golden executor on an NVIDIA B200 (sm_100a), as a C ABI.
 *
 * The reference implements one NPU "device" behind two call surfaces:
 *   - tars_mini/golden.py  Machine(ddr).run_queue(queue_addr, queue_len) -> Status   (golden.py:41-492)
 *   - deploy/kv260/sw/tars_board.py device backends: mem / to_dev(a, n) / from_dev(a, n) /
 *     run(q, n) -> (done, err, op_idx, cycles)  (tars_board.py:1-13, 50-178), whose board
 *     backend loads a tiny C library with ctypes (libtmdrv: tm_open / tm_alloc / tm_wr / tm_rd /
 *     tm_clean / tm_inval, tars_board.py:58-65).
 * This library is that device for a B200: the DDR image lives in HBM, descriptors are checked on
 * the host in the contract's order and executed by CUDA kernels in queue order. Plain C types
 * only; every function returns TC_OK or a negative error (tc_last_error gives the text), except
 * where noted.
 */
#ifndef TARSCUDA_H
#define TARSCUDA_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TC_ABI_VERSION 1
#define TC_OK 0
#define TC_CONTRACT 1      /* an illegal program: golden.py raises ContractError (golden.py:473-479) */
#define TC_ERR_CUDA (-1)
#define TC_ERR_ARG (-2)
#define TC_ERR_TOO_LARGE (-3) /* tc_conv_w8a8_noalloc: the gathered input exceeds its fixed buffer */

typedef struct tc_machine tc_machine;
typedef struct tc_graph tc_graph;

/* golden.py:22-29 Status(done, err_code, op_idx) */
typedef struct { int32_t done, err_code, op_idx; } tc_status;
/* golden.py:32-39 OpStat(opcode, macs, bytes_read, bytes_written) */
typedef struct { uint64_t opcode, macs, bytes_read, bytes_written; } tc_opstat;
/* One set of byte segments [base + i*ld, base + i*ld + nbytes), i < count. kind >= 0: the
 * descriptor's read tensor of that index; -1: its output rows; -2: ROW_QUANT's second output.
 * base = base_hi * 2^64 + base_lo (BASE_ADDR + offset can exceed 64 bits). */
typedef struct { int32_t kind; uint64_t base_lo, base_hi, ld, nbytes, count; } tc_seg;

int tc_version(void);

/* An HBM image of ddr_bytes zero bytes on CUDA device `device`; replaces the board backend's
 * tm_open + tm_alloc (tars_board.py:58-65, tmdrv.c) and golden.Machine's ddr bytearray. */
int tc_open(int device, uint64_t ddr_bytes, tc_machine** out);
int tc_close(tc_machine* m);
const char* tc_last_error(tc_machine* m);
/* The image's device address and CUDA stream (cudaStream_t), for callers that launch work in
 * the same stream order (the decode engine). */
uint64_t tc_device_ptr(tc_machine* m);
void* tc_stream(tc_machine* m);

/* Host <-> image copies; replace tars_board's to_dev(a, n) / from_dev(a, n) (tars_board.py:101-110)
 * and golden.Machine.write / read (golden.py:52-56). */
int tc_upload(tc_machine* m, uint64_t addr, const void* src, uint64_t n);
int tc_download(tc_machine* m, uint64_t addr, void* dst, uint64_t n);
/* Makes the image equal to `host` (n == image size): every 64 KiB block that differs from
 * `shadow` (the caller's copy of what the image held) is uploaded and copied into shadow.
 * The drop-in Machine uses it to honour host writes made between runs (llm.py:793-799). */
int tc_sync_up(tc_machine* m, const void* host, void* shadow, uint64_t n, uint64_t* uploaded);
/* Copies every byte range the last tc_run_queue wrote back into `host` (and `shadow` if given),
 * so the caller's bytearray is mutated in place as golden.Machine mutates its ddr. */
int tc_sync_down(tc_machine* m, void* host, void* shadow);

/* Runs queue_len descriptors at queue_addr strictly in order; replaces golden.Machine.run_queue
 * (golden.py:450-492) and tars_board's dev.run(q, n) (tars_board.py:117-152, 173-178). Returns
 * TC_OK with *st set (done, or the first error code and its descriptor), or TC_CONTRACT with
 * *contract_op = the illegal descriptor's index (earlier descriptors' writes kept), or < 0. */
int tc_run_queue(tc_machine* m, uint64_t queue_addr, uint32_t queue_len, int32_t core_id,
                 int32_t gemv_only, tc_status* st, int32_t* contract_op);
/* The last run's per-descriptor stats (golden.Machine.stats); returns how many there are. */
uint32_t tc_stats(tc_machine* m, tc_opstat* out, uint32_t cap);

/* Checks a queue exactly as tc_run_queue does and captures its kernels as one CUDA graph without
 * running them; *st is the status the run would end with. The board runtime runs one fixed queue
 * per position (tars_board.py:316-329, llm.py:548-571), so a queue is checked once and replayed.
 * timing == 0: the graph of dependency levels (independent descriptors of a level run side by
 * side; decode GEMVs of one kernel class and row ops of a level are batched into one launch each);
 * timing == 1: the descriptors one after another with an event between them (tc_graph_times gives
 * per-descriptor times); timing == 2: the level graph with an event between levels (per-level
 * times). A queue whose descriptors rewrite later descriptors of the same queue is refused
 * (TC_ERR_ARG). */
int tc_queue_capture(tc_machine* m, uint64_t queue_addr, uint32_t queue_len, int32_t core_id,
                     int32_t gemv_only, int32_t timing, tc_status* st, int32_t* contract_op,
                     tc_graph** out);
/* Enqueues the captured queue on `stream` (NULL: the machine's stream); the next tc_sync_down
 * copies back the ranges it writes. */
int tc_graph_launch(tc_graph* g, void* stream);
/* Per-descriptor milliseconds of the last launch of a graph captured with timing; returns the count. */
int tc_graph_times(tc_graph* g, float* ms, uint32_t cap);
int tc_graph_destroy(tc_graph* g);
/* Kernel launches one replay of the graph makes (the capture batches independent GEMVs and row ops
 * of a dependency level into one launch, so this is usually below the descriptor count). No
 * reference counterpart: the reference executes descriptors one at a time. */
int tc_graph_kernels(tc_graph* g);
/* Waits for everything enqueued on the machine's stream. */
int tc_synchronize(tc_machine* m);

/* The W8A8 GEMM kernel choice: GEMMs of at least `rows` token rows (M) whose operands meet the
 * TMA rules (16-byte aligned A, W and row stride, K % 16 == 0) run on the tensor cores (tcgen05,
 * int8 MMA); the others on the CUDA-core GEMV kernels. Both are bit-exact. Values below 2 mean 2.
 * Default 16 (or the environment variable TARSCUDA_MMA_MIN_M). Returns the previous value; it
 * applies to every machine and engine of the process, to launches enqueued afterwards. */
int tc_set_mma_min_rows(int32_t rows);
/* Tracing of the tensor-core GEMM: with enable = n > 0, the n-th tensor-core GEMM launch enqueued
 * (or captured) after this call records per CTA (its first 2048 CTAs) 8 globaltimer stamps in
 * nanoseconds: 0 entry, 1 setup done, 2 first token slice issued, 3 first stage consumed by the
 * MMA thread, 4 last MMA committed, 5 (split-K) the peers' partial rows received, 6 epilogue done,
 * 7 exit (persistent) or the accumulator ready in the epilogue (split-K). Enabling zeroes the
 * stamps; enable = 0 turns tracing off. With out != NULL, waits for the device and copies
 * min(cap, 2048 * 8) stamps; returns that count (or TC_ERR_CUDA). No counterpart in the reference
 * (a diagnostic). */
int tc_mma_trace(int32_t enable, uint64_t* out, uint32_t cap);
/* The device word (one per device: the current device's is read) in which the streaming kernels
 * (tensor-core GEMM, grouped GEMV, streamed W4A16 GEMV) record a bounded wait that gave up instead
 * of hanging: 0 = none, else the code of the first one since the word was last cleared (GEMM 1-5,
 * grouped GEMV 21-22, streamed W4A16 GEMV 11-12, tiled W4A16 GEMV 13-15: weight ring producer,
 * consumer, the hand-over of a tile's partial sums between the quads of a block); a kernel that
 * gave up skipped the rest of its work, so its
 * outputs are incomplete. clear != 0 resets the word. Synchronous; TC_ERR_CUDA if it cannot be
 * read. No counterpart in the reference (its golden model never waits). */
int tc_wait_error(int32_t clear);
/* The number of polls after which the bounded waits for work give up, for launches enqueued from
 * now on (default and maximum 2^22, about a second on a B200; 0 makes every such wait give up at
 * once, which is how the give-up path is tested without a hang or a fault). The waits that let a
 * block's in-flight copies land before it exits keep the full limit. Returns the previous value.
 * No counterpart in the reference. */
uint32_t tc_set_spin_limit(uint32_t polls);

/* Host-only helpers (no device needed). golden.Machine.validate (golden.py:59-169): decodes the
 * 23 fields of contract.py:14-38 into fields[23] (in that table's order) and returns the first
 * failing check (E_OK .. E_ALIGN). */
int tc_validate(const uint8_t* raw64, int32_t core_id, int32_t gemv_only, uint64_t* fields23);
/* golden.Machine.segments / extra_out (golden.py:195-256) as strided sets; *count = how many. */
int tc_footprint(const uint8_t* raw64, tc_seg* out, uint32_t cap, uint32_t* count);

/* No counterpart in the reference: the W8A8 convolution of a conv descriptor (same arithmetic,
 * same bytes) for callers that must not have the library allocate device memory during a call,
 * such as a server that reserved all of HBM for its own pool up front or an embedder whose
 * device footprint must be fixed when the library loads. The window gather uses a fixed 16 MiB
 * array in device memory that every GPU loading the library holds until exit; OH*OW*KH*KW*Cin
 * bytes above that return TC_ERR_TOO_LARGE. All pointers are device pointers of the caller
 * (img: H*W pixel rows of Cin int8 with row stride ld; weights: int8 [N, KH*KW*Cin]; scale: fp32
 * [N] or [1]; bias: fp32 [N] or NULL; y: OH*OW rows with stride ldy in format out: 0 fp32,
 * 1 bf16, 2 int8 via out_scale); work is enqueued on `stream` (a cudaStream_t, NULL = default).
 * The first call on a device looks the array up with that device current; under CUDA's lazy
 * module loading that call also loads the array onto the device, so make it before any stream
 * capture. Calls share the array and it keeps the last call's contents (every byte a call reads it
 * writes first); calls that overlap on the GPU race, so order them on one stream. TC_ERR_ARG for
 * pad >= KH or KW, or more than 2^31 pixels. */
int tc_conv_w8a8_noalloc(const uint8_t* img, uint64_t ld, int32_t H, int32_t W, int32_t Cin, int32_t KH,
                         int32_t KW, int32_t stride, int32_t pad, const uint8_t* weights, const float* scale,
                         int32_t per_channel, const float* bias, uint8_t* y, uint64_t ldy, int32_t N,
                         int32_t act, int32_t out, float out_scale, void* stream);

#ifdef __cplusplus
}
#endif
#endif
