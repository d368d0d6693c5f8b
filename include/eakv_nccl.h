/* eakv_nccl.h - multi-GPU decode of long contexts over NCCL
 * (libeakv_b200.so).
 *
 * No counterpart in the reference: its decode is one serial loop over the
 * positions of a sequence on one CPU core (reference
 * kernels/fused_k_score_gqa.ea:29, kernels/fused_attention.ea:38-187). Here
 * the positions of every sequence can be split across the GPUs of a group,
 * one process (or host thread) per GPU, each rank holding its own slice in
 * its own caches; NVLink then carries only each rank's per-row record
 * (normalized output and log-sum-exp), gathered by NCCL and merged exactly
 * on every rank. KV-head shards need no exchange and use eakv_decode_attention.
 *
 * NCCL is loaded at run time (EAKV_NCCL_LIB, else a libnccl.so.2 already
 * loaded in the process, else the dynamic linker's search); without it
 * these calls return EAKV_ERR_INVALID and everything else still works.
 * Communicators are ncclComm_t values passed as void*, so this header needs
 * no NCCL header; a caller with its own NCCL may pass its own communicator
 * (it must come from the same NCCL library).
 *
 * Failure handling: a rank that stops calling leaves its peers' collective
 * waiting on the GPU. A host watchdog that sees a peer gone (a heartbeat,
 * a store) calls eakv_nccl_comm_abort on its communicator, which ends the
 * waiting NCCL kernels; the communicator is then unusable.
 */
#ifndef EAKV_NCCL_H
#define EAKV_NCCL_H

#include "eakv_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

#define EAKV_NCCL_ID_BYTES 128

/* NCCL version code of the loaded library (e.g. 22809), or < 0. */
int eakv_nccl_version(void);

/* Writes a new NCCL unique id (EAKV_NCCL_ID_BYTES bytes) to `id`: one rank
 * makes it and sends it to the others out of band. */
int eakv_nccl_unique_id(void *id);

/* Joins the communicator of n_ranks ranks named by `id` as `rank`, on CUDA
 * device `device`. Blocks until every rank has joined. *comm receives the
 * ncclComm_t. */
int eakv_nccl_comm_init(void **comm, int n_ranks, const void *id, int rank, int device);
int eakv_nccl_comm_destroy(void *comm);
/* Ends the communicator's collectives in flight (host-side failure path). */
int eakv_nccl_comm_abort(void *comm);

/* One decode step of a sequence split over the ranks of `comm`: this rank's
 * caches hold its slice of the positions of every sequence (any slices,
 * disjoint across ranks; a rank's slice may be empty). Every rank calls with
 * the same number and shape of caches and the same queries, in the same
 * order of calls; every rank receives in d_output
 * (f32[n_caches][n_layers][n_q_heads][head_dim]) the softmax attention over
 * the union of the slices. Per rank: the partial decode of positions
 * [pos_begin, min(pos_end, seq_len)) of its caches (0, -1: all), an
 * ncclAllGather of the records (n_layers * n_q_heads * (head_dim + 1) floats
 * per cache and rank), and the exact merge. With two or more caches the
 * caches are taken in two halves: the second half decodes on a second
 * stream while the first half's all-gather and merge run on a collective
 * stream of the library, so two all-gathers are issued per call. Everything
 * is ordered after earlier work on `stream` (NULL: the first cache's
 * stream), later work on `stream` sees the output, and nothing synchronizes
 * the host. Workspace comes from the first cache's scratch; the helper
 * streams are shared by the calls of one device. */
int eakv_decode_attention_split(const eakv_cache_t *const *caches, int n_caches,
                                const float *d_queries, int n_q_heads, int pos_begin,
                                int pos_end, float *d_output, void *comm, void *stream);

/* Same step with host buffers (queries / output f32[n_caches][n_layers]
 * [n_q_heads][head_dim]): copies in, runs the step, copies out, and returns
 * when done. From 1 MiB of queries on, the caches are cut into up to four
 * chunks, each its own split step (its own all-gather) on `stream`, whose
 * copies overlap the other chunks' steps; every rank must make the same
 * call, so the chunks and their collectives match. Every chunk keeps the
 * whole batch's split plan. */
int eakv_decode_attention_split_host(const eakv_cache_t *const *caches, int n_caches,
                                     const float *queries, int n_q_heads, float *output,
                                     void *comm, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* EAKV_NCCL_H */
