/*
 * kotflash_b200 — C ABI of the B200 (sm_100a) attention hot path.
 *
 * Every entry point is `extern "C"`, takes plain pointers, sizes and element
 * strides, launches on the caller's CUDA stream, never allocates device
 * memory, never synchronises, and returns a status code (KF_OK == 0).  On a
 * non-zero status `kf_last_error()` returns a thread-local message.
 *
 * Tensors are described by `kf_tensor4`: a [n0, n1, n2, n3] strided view
 * (strides in ELEMENTS, like torch.Tensor.stride()).  Attention tensors use
 * the reference's [batch, heads, sequence, head_dim] layout
 * (kotflash/attention.py:232-236).  Element types are fp16 or bf16
 * (`KF_F16`, `KF_BF16`); LSE, partials and gradient workspaces are fp32.
 *
 * Device-side waits are bounded.  Kernels that give up on a wait write a
 * non-zero code into the caller-supplied `status` word (int32 in device
 * memory) and return; the host reads that word outside the hot path.
 *
 * Device: every entry point that takes device memory makes the GPU owning
 * its first tensor (q, the K cache, o or the partials) current for the call
 * and restores the caller's device before returning, as the reference's
 * extension does with c10::cuda::CUDAGuard (kotflash/csrc/kv_append_cuda.cu:77).
 * The stream must belong to that GPU.  kf_ipc_open_handle maps into the
 * caller's current device.
 */
#ifndef KOTFLASH_B200_H
#define KOTFLASH_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define KF_OK              0
#define KF_ERR_INVALID     1  /* bad argument (shape, stride, alignment)     */
#define KF_ERR_UNSUPPORTED 2  /* valid but outside this build's envelope     */
#define KF_ERR_CUDA        3  /* a CUDA runtime/driver call failed           */
#define KF_ERR_WORKSPACE   4  /* workspace pointer/size too small            */

/* device status word values written by kernels */
#define KF_DEV_OK          0
#define KF_DEV_TIMEOUT     1  /* a bounded mbarrier wait expired             */

#define KF_F16  0
#define KF_BF16 1

typedef struct kf_tensor4 {
  void*   ptr;
  int64_t size[4];
  int64_t stride[4];
} kf_tensor4;

/* ---- version / errors -------------------------------------------------- */
int         kf_version(void);
const char* kf_last_error(void);

/* ---- K4: KV-cache append ------------------------------------------------
 * Replaces the pybind op `append_kv_(k_cache, v_cache, new_k, new_v, start)`
 * (kotflash/csrc/kv_append.cpp:11-14) and its host checks + launch
 * (kotflash/csrc/kv_append_cuda.cu:44-96).  Copies new_k/new_v [B,H,S,D] into
 * k_cache/v_cache [B,H,cap,D] at sequence offset `start`, K and V in ONE
 * launch.  Bit-exact (pure data movement).  Unlike the reference, fp16 and
 * bf16 are accepted and the destination may be any strided view whose last
 * dimension is contiguous. */
int kf_append(const kf_tensor4* k_cache, const kf_tensor4* v_cache,
              const kf_tensor4* new_k, const kf_tensor4* new_v,
              int64_t start, int dtype, void* stream);

/* ---- K1: forward --------------------------------------------------------
 * Replaces `attention_forward(q, k, v, causal, scale) -> (out, lse)`
 * (kotflash/kernels/triton_forward.py:372-456) and the kernel
 * `_attention_fwd_kernel` (triton_forward.py:21-165).  Writes O [B,Hq,Sq,D]
 * (q dtype) and LSE [B,Hq,Sq] fp32 (natural log of the row's softmax
 * denominator over scale*QK^T).  Causal masks are upper-left aligned (key
 * j visible to query i iff j <= i).  Requirements: 16 <= D <= 128, D % 8 == 0,
 * last-dim-contiguous tensors with 16-byte aligned base and strides; O and
 * LSE contiguous. */
int kf_attn_fwd(const kf_tensor4* q, const kf_tensor4* k, const kf_tensor4* v,
                const kf_tensor4* o, float* lse, int dtype, float scale,
                int causal, int32_t* status, void* stream);

/* ---- K2: backward -------------------------------------------------------
 * Replaces `attention_backward(q, k, v, out, lse, grad_out, causal, scale)`
 * (kotflash/kernels/triton_backward.py:335-421) and its kernels
 * `_attention_bwd_dq`, `_attention_bwd_dkv(_split)`, `_attention_bwd_dkv_reduce`
 * (triton_backward.py:18-332).  Writes dq, dk, dv (input dtype) given the
 * forward's O and LSE and the upstream gradient dO.  dK/dV sum over the
 * GQA group of each KV head.  `workspace` must hold
 * kf_attn_bwd_workspace_bytes(...) bytes (fp32 dQ accumulator + row deltas). */
size_t kf_attn_bwd_workspace_bytes(int64_t B, int64_t Hq, int64_t Sq, int64_t D);
/* The same plus fp32 dK/dV accumulators.  With a workspace this large a
 * causal backward whose key blocks give fewer than two CTAs per SM (e.g. one
 * long-sequence (batch, KV head) unit per GPU) splits each key block's query
 * range over several CTAs that add their dK/dV parts into the accumulators,
 * as the reference does with `_attention_bwd_dkv_split` + `_dkv_reduce`
 * (kotflash/kernels/triton_backward.py:199-332); with the smaller size it
 * runs one CTA per key block. */
size_t kf_attn_bwd_workspace_bytes_kv(int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Sk,
                                      int64_t D);
int kf_attn_bwd(const kf_tensor4* q, const kf_tensor4* k, const kf_tensor4* v,
                const kf_tensor4* o, const float* lse, const kf_tensor4* dout,
                const kf_tensor4* dq, const kf_tensor4* dk, const kf_tensor4* dv,
                int dtype, float scale, int causal,
                void* workspace, size_t workspace_bytes,
                int32_t* status, void* stream);

/* ---- K3: split-KV decode ------------------------------------------------
 * Replaces `attention_forward_strided_decode(q, k, v, scale)`
 * (kotflash/kernels/triton_decode.py:412-468; kernels `_strided_decode_split`
 * 17-104 and `_strided_decode_reduce` 242-297), the split-KV branch of
 * `attention_forward` (triton_forward.py:410-445; kernels 170-349), and, when
 * new_k/new_v are non-NULL, the fused one-token append
 * `attention_forward_strided_append` (triton_decode.py:302-386): the new row
 * is written at position `past_len` of the cache and attended in the same
 * pass.  Non-causal, Sq <= 16.  K/V may be strided prefix views of a larger
 * cache (last dim contiguous).  Writes O (q dtype) and, if lse != NULL, the
 * merged LSE.  num_splits == 0 lets the planner choose.
 * `workspace` must hold kf_decode_workspace_bytes(...) bytes. */
int    kf_decode_num_splits(int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq,
                            int64_t Sk, int64_t D, int sm_count);
size_t kf_decode_workspace_bytes(int64_t B, int64_t Hq, int64_t Sq, int64_t D,
                                 int num_splits);
int kf_decode(const kf_tensor4* q, const kf_tensor4* k, const kf_tensor4* v,
              const kf_tensor4* new_k, const kf_tensor4* new_v, int64_t past_len,
              const kf_tensor4* o, float* lse, int dtype, float scale,
              int num_splits, void* workspace, size_t workspace_bytes,
              void* stream);

/* ---- K3, allocation-free variant ---------------------------------------
 * No counterpart in the reference: added for callers that cannot allocate
 * device memory or hand this library a workspace — a host runtime that owns
 * every device allocation itself (an inference server's memory manager, or an
 * FFI embedder with a fixed device-memory budget) and gives plugins no
 * allocator.  Same arguments and results as kf_decode minus the workspace:
 * the split partials go to one file-scope device array of 8 MiB that every
 * GPU loading the library holds until exit.  Each call looks up the array's
 * address on the tensors' device (a host-side query, no allocation); the
 * first call on a device also loads the module there, so make that first
 * call before any stream capture.  num_splits == 0 plans the split
 * count and lowers it until the partials fit in 8 MiB; an explicit
 * num_splits whose partials (num_splits * B*Hq*Sq * (D+1) * 4 bytes) exceed
 * 8 MiB is rejected with KF_ERR_WORKSPACE.  All calls share the array: calls
 * that overlap on the GPU (different streams or threads) race and must be
 * serialised by the caller.  Calls no allocator. */
int kf_decode_noalloc(const kf_tensor4* q, const kf_tensor4* k, const kf_tensor4* v,
                      const kf_tensor4* new_k, const kf_tensor4* new_v, int64_t past_len,
                      const kf_tensor4* o, float* lse, int dtype, float scale,
                      int num_splits, void* stream);

/* ---- K3b: LSE-weighted merge of partial (O, LSE) ------------------------
 * Replaces `_attention_fwd_split_kv_reduce` (triton_forward.py:270-349).
 * part_o: [S, rows, D] fp32, part_lse: [S, rows] fp32, where rows =
 * B*Hq*Sq in [b][h][s] order.  Writes o (rows x D, dtype, contiguous) and,
 * if lse != NULL, the merged LSE.  Empty partials carry LSE = -inf and
 * contribute nothing; a row whose partials are all empty yields O = 0 and
 * LSE = -inf.  1 <= num_splits <= 512 (KF_ERR_UNSUPPORTED above).  Used for
 * the cross-GPU merge after the all-gather. */
int kf_merge_partials(const float* part_o, const float* part_lse, int num_splits,
                      int64_t rows, int64_t D, void* o, float* lse, int dtype,
                      void* stream);

/* ---- cross-GPU exchange of decode partials over NVLink peer memory -----
 * No counterpart in the reference, which has no multi-GPU decode; it
 * replaces the all-gather + merge of a KV-sequence split across the ranks of
 * one box (the split/merge math is triton_forward.py:270-349 applied across
 * ranks).  Each rank owns a mailbox of kf_peer_mailbox_bytes(world, rows, D)
 * bytes of ZERO-FILLED device memory from cudaMalloc (256-byte aligned) and
 * maps every peer's through CUDA IPC: kf_ipc_get_handle gives a 64-byte
 * handle plus the pointer's offset inside its allocation, kf_ipc_open_handle
 * maps a peer's handle in this process, kf_ipc_close_handle unmaps it.
 * mailboxes[r] is rank r's mailbox as mapped here (mailboxes[rank] is the
 * local one).  1 <= world <= 8; D a multiple of 8 in [8, 128].
 *
 * kf_decode_kv_split_peer: split-KV decode of this rank's key chunk (q, k, v
 * as kf_decode, no fused append; rows = B*Hq*Sq) fused with the exchange:
 * the split kernel, a kernel that merges this rank's splits and stores the
 * fp32 result into every mailbox (peer stores, then a system-scope release
 * add on the receiver's arrival counter), and the final merge into o / lse
 * (lse may be null).  num_splits >= 1 (the plan's value); the workspace
 * needs kf_decode_workspace_bytes(B, Hq, Sq, D, max(2, num_splits)) bytes.
 * kf_decode_kv_split_peer_send is its first two kernels alone (nothing
 * waits); kf_decode_peer_merge with rows = B*Hq*Sq then gives the result
 * as a contiguous [rows, D].
 *
 * kf_decode_peer_exchange: the same exchange for a finished partial: o
 * [rows, D] (fp16/bf16, normalised, contiguous) and lse [rows] fp32 (natural
 * log) in, the merge of all ranks' partials out ([rows, D] and [rows]).
 * kf_decode_peer_put / kf_decode_peer_merge are its two halves.  The put
 * never waits; the merge waits for all `world` partials of the current call,
 * so a single process may drive several mailboxes on one GPU (all puts
 * first, then the merges) without kernels that wait on one another.
 *
 * Every wait is bounded (about one second): on expiry *status (device
 * memory, may be null) = KF_DEV_TIMEOUT and the output is NaN.  The exchange
 * is then unusable: the timed-out half's arrival counter is short and a late
 * sender's rows may still land in it, so every rank must stop calling, zero
 * its mailbox (all ranks), and start again from a new set of mailboxes.  Every rank must
 * make the same sequence of calls with the same rows and D; the call count
 * is kept in the mailbox, so the launches may be captured in a CUDA graph
 * and replayed. */
size_t kf_peer_mailbox_bytes(int world, int64_t rows, int64_t D);
int kf_ipc_get_handle(const void* ptr, void* handle64, uint64_t* offset);
int kf_ipc_open_handle(const void* handle64, uint64_t offset, void** ptr);
int kf_ipc_close_handle(void* ptr, uint64_t offset);
int kf_decode_kv_split_peer(const kf_tensor4* q, const kf_tensor4* k, const kf_tensor4* v,
                            const kf_tensor4* o, float* lse, int dtype, float scale, int num_splits,
                            void* workspace, size_t workspace_bytes, void* const* mailboxes,
                            int world, int rank, int32_t* status, void* stream);
int kf_decode_kv_split_peer_send(const kf_tensor4* q, const kf_tensor4* k, const kf_tensor4* v,
                                 int dtype, float scale, int num_splits, void* workspace,
                                 size_t workspace_bytes, void* const* mailboxes, int world, int rank,
                                 void* stream);
int kf_decode_peer_exchange(const void* o, const float* lse, int64_t rows, int64_t D,
                            int dtype, void* const* mailboxes, int world, int rank,
                            void* out, float* out_lse, int32_t* status, void* stream);
int kf_decode_peer_put(const void* o, const float* lse, int64_t rows, int64_t D, int dtype,
                       void* const* mailboxes, int world, int rank, void* stream);
int kf_decode_peer_merge(void* mailbox, int64_t rows, int64_t D, int dtype, int world,
                         void* out, float* out_lse, int32_t* status, void* stream);

/* ---- self-test of the bounded device wait -------------------------------
 * No counterpart in the reference.  Launches one kernel that waits on a
 * barrier nothing completes; after `budget_us` microseconds the wait gives
 * up and writes KF_DEV_TIMEOUT into *status (device memory), the same path
 * every attention kernel takes when a wait expires.  Used by the tests to
 * show that an expired wait is reported and leaves the context usable. */
int kf_selftest_bounded_wait(int32_t* status, int64_t budget_us, void* stream);

/* ---- self-test of the forward kernel's polynomial exponential -------------
 * No counterpart in the reference (its Triton kernels call exp2 only).  The
 * forward kernel computes part of its softmax exponentials on the fp32 pipe
 * as a degree-3 polynomial after a Cody-Waite range split; this evaluates
 * that same device function on n (even) fp32 arguments x (device memory) into
 * y, so tests can bound its error against exp2 over the argument range. */
int kf_selftest_exp2_poly(const float* x, float* y, int64_t n, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* KOTFLASH_B200_H */
