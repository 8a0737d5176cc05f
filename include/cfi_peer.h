/*
 * cfi_peer.h -- the all-gather of row-sharded products over NVLink peer memory.
 *
 * No counterpart in cuda-for-intel (single GPU, "No NCCL", README.md:110-111).  When the rows of
 * every weight matrix are split over the GPUs of one node (one process per GPU), each product's
 * output must reach every rank.  Instead of one collective per product, each rank maps the other
 * ranks' output buffers into its address space (CUDA IPC; NVSwitch gives every GPU full bandwidth
 * to every peer) and the product kernel stores each finished output tile into its own copy and
 * into every peer's copy, at the same offsets: ggml's column-major dst is assembled in place on
 * every rank, with no gather kernel and no collective.  The launch's last CTA then adds 1 to this
 * rank's signal slot on every peer and waits until every peer has signalled as often as this
 * rank has waited so far, so the launch completes only when the gather is (plain loads and
 * stores over NVLink: no multicast, no NVLS).  Every wait is bounded: a peer that never signals
 * sets the library's device error word (cfi_device_error) instead of hanging the GPU.
 *
 * A peer buffer is one cudaMalloc allocation; `handle` is CFI_PEER_HANDLE_BYTES bytes (a
 * cudaIpcMemHandle_t) that the host side exchanges between the ranks (any channel: the handles
 * are plain bytes).  All pointers are device pointers; `stream` is a cudaStream_t; each call
 * returns 0 or a CUDA error code.
 */
#ifndef CFI_PEER_H
#define CFI_PEER_H
#include <stddef.h>
#include <stdint.h>

#ifndef CFI_API
#define CFI_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define CFI_PEER_HANDLE_BYTES 64
#define CFI_PEER_MAX_RANKS 8

/* *ptr = a new zeroed device buffer of `bytes` on the current device, and its IPC handle */
CFI_API int cfi_peer_alloc(size_t bytes, void **ptr, void *handle);
/* *ptr = this process's mapping of another process's peer buffer (peer access enabled) */
CFI_API int cfi_peer_open(const void *handle, void **ptr);
/* unmaps a buffer cfi_peer_open mapped */
CFI_API int cfi_peer_close(void *ptr);
/* frees a buffer cfi_peer_alloc made (after every peer has closed its mapping) */
CFI_API int cfi_peer_free(void *ptr);

/* A rank's view of its group: byte offsets to the other ranks' mappings and their signal slots
 * for this rank, and its own signal and wait counters.  rank < world <= CFI_PEER_MAX_RANKS;
 * delta[r] = (rank r's buffer as mapped here) - (this rank's buffer), 0 for r == rank;
 * sig_remote[r] = rank r's slot for this rank (inside r's buffer, as mapped here); sig_local and
 * expect: `world` zeroed counters each in this rank's memory (peers add to sig_local[their
 * rank]).  Each signalling launch adds 65536 in all to this rank's slot on every peer; the
 * counters wrap modulo 2^32. */
typedef struct CfiPeerSet {
    int rank, world;
    long long delta[CFI_PEER_MAX_RANKS];
    unsigned int *sig_remote[CFI_PEER_MAX_RANKS];
    unsigned int *sig_local;
    unsigned int *expect;
} CfiPeerSet;

/* A barrier of the group on `stream`, after the work queued before it: signals every peer, then
 * waits until sig_local[r] has reached expect[r] + 65536 for every other rank r and sets
 * expect[r] to that.  A peer that has not signalled within 10 s (CFI_PEER_WAIT_MS
 * milliseconds when set) ends the wait with 0x9e0000 | r in the device error word; once that is
 * set (until cfi_device_error reads it), later waits of the group give up at once. */
CFI_API int cfi_peer_barrier(const CfiPeerSet *peers, void *stream);

/* All-gather over the group: dst is the gathered range inside this rank's peer buffer (world *
 * bytes; rank r's copy of it at dst + delta[r]); every rank stores its `bytes` at src (device
 * memory) at dst + rank * bytes of every rank's copy (its own included), then signals and waits
 * as cfi_peer_barrier does, so when it completes this rank's range holds every rank's slice, rank
 * by rank (the layout of an all_gather_into_tensor).  src, dst and bytes multiples of 16; every
 * rank passes the same bytes and the same offset of dst in its buffer.  A few CTAs do the copy
 * (plain 16-byte loads and stores over NVLink), so the kernels running beside it keep the rest of
 * the GPU. */
CFI_API int cfi_peer_all_gather(const void *src, size_t bytes, void *dst, const CfiPeerSet *peers, void *stream);

/* cfi_mmq_skinny_group (cfi_glue.h) as one step of an all-gather over the group: every output
 * value written at address a of dst[i] (inside this rank's peer buffer) is also written at
 * a + delta[r] on every other rank r; after its last store the launch signals every peer and
 * waits for every peer's signal as cfi_peer_barrier does, so when it completes every rank's rows
 * of the same launch are in this rank's outputs. */
CFI_API int cfi_mmq_skinny_group_peers(uint32_t type, int n, const void *const *x, const void *y, float *const *dst,
                                       const uint32_t *nrows, const uint32_t *stride_row_x,
                                       const uint32_t *stride_col_dst, uint32_t K, uint32_t ncols, uint32_t ncols_y,
                                       const CfiPeerSet *peers, void *stream);

#ifdef __cplusplus
}
#endif
#endif
