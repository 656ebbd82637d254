/* C ABI of the B200 (sm_100a) BF16 attention-forward library.
 *
 * Drop-in for the reference's public header (include/fav4_bshd.h:1-20 of
 * rocking5566/flash-attention-v4-rocm): same struct layout, same symbol names,
 * same argument meaning and error codes, with cudaStream_t in place of
 * hipStream_t (both are an opaque pointer, so ctypes callers are unchanged).
 */
#ifndef FAV4_BSHD_H_
#define FAV4_BSHD_H_

#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same field order and types as the reference's Fav4Args
 * (include/fav4_bshd.h:4-10): 5 pointers, 4 ints, 1 float. */
struct Fav4Args {
  const void *q, *k, *v;
  void* o;
  float* lse;
  int batch, heads, sq, sk;
  float scale;
};
typedef struct Fav4Args Fav4Args;

/* Contract (reference include/fav4_bshd.h:12-18):
 * Q/K/V/O are contiguous BF16 [batch, sequence, heads, 128], device-resident,
 * 16-byte aligned and non-overlapping. LSE is optional FP32 [batch, heads, sq]
 * in natural-log units. Top-left causal (key c visible to query row r iff
 * c <= r), equal Q/K/V heads, positive finite scale, finite dot products.
 * The stream belongs to the calling device; the call allocates nothing and
 * never synchronises the host, so it can be captured in a CUDA graph.
 * config 0 = Auto: fav4_bshd_select_config's rule, except that config 1 is
 * taken when config 2's work tiles (batch * heads * ceil(sq / 256)) would
 * occupy at most half of the device's SMs, and that dense launches with
 * sk >= 2048 take the wide-step kernel (fav4_bshd_forward_wide) when its
 * 128-row tiles need fewer than 1.84x the waves of config 2's 256-row tiles;
 * 1/2/3 = explicit tilings.
 * Returns 0 on success, cudaErrorInvalidValue (1) on invalid arguments or
 * config, else the launch status (cudaGetLastError).
 *
 * Replaces: fav4_bshd_forward, reference include/fav4_bshd.h:19 and
 * src/bshd.hip:26-38. */
int fav4_bshd_forward(const Fav4Args* args, int causal, int config, cudaStream_t stream);

/* The reference's auto configuration: 1 when sq < 128, else 2 (the Auto of
 * fav4_bshd_forward, _gqa, _host and the one-launch split-KV entries adds the
 * few-tiles rule above; the partial and packed-sequence entries use this rule
 * as it is).
 * Replaces: fav4_bshd_select_config, reference include/fav4_bshd.h:20 and
 * src/bshd.hip:23-25. */
int fav4_bshd_select_config(const Fav4Args* args);

/* Dense forward through the wide-step kernel whatever the shape: one 128-row
 * Q tile per CTA against 256 keys per step (S as a 128x256 MMA, P in TMEM
 * columns of its own, the 256 keys' softmax split over two warpgroups).
 * fav4_bshd_forward's Auto takes it for dense launches whose 256-row tiles
 * would leave the last wave poorly filled (see config 0 above); this entry
 * runs it on any valid dense problem. Same arguments, checks and return codes
 * as fav4_bshd_forward with causal = 0 and config = 0 (no reference
 * counterpart: the reference has one kernel per config, src/bshd.hip:26-38). */
int fav4_bshd_forward_wide(const Fav4Args* args, cudaStream_t stream);

/* Grouped-query attention (no reference counterpart: the reference requires
 * equal Q/K/V heads, include/fav4_bshd.h:15). args->heads is the number of
 * query heads; K and V are BF16 [batch, sk, kv_heads, 128] with kv_heads
 * dividing args->heads, and query head h attends K/V head
 * h / (heads / kv_heads) (kv_heads = 1 is multi-query attention). O and LSE
 * have args->heads heads. kv_heads == heads is fav4_bshd_forward. Other
 * arguments, validation and return codes as fav4_bshd_forward, plus
 * cudaErrorInvalidValue when kv_heads is not a divisor of heads. */
int fav4_bshd_forward_gqa(const Fav4Args* args, int kv_heads, int causal, int config, cudaStream_t stream);

/* Packed variable-length sequences (no reference counterpart). Sequence b has
 * query rows [cu_seqlens_q[b], cu_seqlens_q[b+1]) of q / o and keys
 * [cu_seqlens_k[b], cu_seqlens_k[b+1]) of k / v; the offset arrays are device
 * int32 [batch + 1]. q, o: BF16 [total_q, heads, 128]; k, v: BF16
 * [total_k, kv_heads, 128] (kv_heads divides heads; equal heads for ordinary
 * attention); lse (optional): FP32 [heads, total_q]. max_sq: the longest query
 * sequence (at most total_q; it sizes the launch). Causal masking is
 * top-left within each sequence, as in fav4_bshd_forward. Offsets are read on
 * the device and clamped to [0, total]: malformed offsets give wrong rows,
 * never an access outside the tensors. Returns 0, cudaErrorInvalidValue or the
 * launch status. */
struct Fav4VarlenArgs {
  const void *q, *k, *v;
  void* o;
  float* lse;
  const int* cu_seqlens_q;
  const int* cu_seqlens_k;
  int batch, heads, kv_heads, max_sq, total_q, total_k;
  float scale;
};
typedef struct Fav4VarlenArgs Fav4VarlenArgs;

int fav4_bshd_forward_varlen(const Fav4VarlenArgs* args, int causal, int config, cudaStream_t stream);

/* Split-KV slice (no reference counterpart; needed because Fav4Args carries
 * no key offset). Attends only keys [kv_begin, kv_end) with absolute
 * positions, so top-left causal masking stays correct for any slice. O is the
 * slice-normalised output (BF16, zero for rows that see no key of the slice);
 * LSE is required and is -inf for such rows. Same validation and return codes
 * as fav4_bshd_forward, plus 0 <= kv_begin < kv_end <= sk. */
int fav4_bshd_forward_partial(const Fav4Args* args, int causal, int config, int kv_begin, int kv_end,
                              cudaStream_t stream);

/* LSE-weighted combine of `parts` split-KV slices (no reference counterpart):
 *   LSE = log(sum_g exp(LSE_g)),  O = sum_g exp(LSE_g - LSE) * O_g.
 * o_parts[g] / lse_parts[g] are the outputs of fav4_bshd_forward_partial for
 * the same (batch, heads, sq) and may live on peer GPUs with peer access
 * enabled (read with plain loads). o and lse (lse may be NULL) receive the
 * result; rows whose every slice is empty get O = 0 and LSE = -inf.
 * 1 <= parts <= 16. Returns 0, cudaErrorInvalidValue or the launch status. */
int fav4_bshd_combine(const void* const* o_parts, const float* const* lse_parts, int parts, void* o, float* lse,
                      int batch, int heads, int sq, cudaStream_t stream);

/* Split-KV forward on one GPU that allocates nothing (no counterpart in the
 * reference). Same result as fav4_bshd_forward (within the split-KV
 * tolerance), computed as `splits` key ranges in one launch of the split-KV
 * kernel plus the LSE-weighted combine. It is for callers that cannot call
 * cudaMalloc: plugins whose host application owns every byte of device
 * memory through its own pool (there a cudaMalloc fails, or takes memory the
 * host has promised elsewhere), and latency-critical paths that cannot take
 * cudaMalloc's implicit device synchronisation. The key-range partials live
 * in a fixed 64 MiB device array inside the library instead; every GPU that
 * loads the library holds that array until the process exits.
 *   - 1 <= splits <= 16; splits = 1 is fav4_bshd_forward (no partials).
 *   - Needs fav4_bshd_splitkv_workspace_bytes(args, splits) bytes, i.e.
 *     splits * (batch*sq*heads*256 + batch*heads*sq*4), each part rounded up
 *     to 256 bytes; larger problems return cudaErrorMemoryAllocation (2)
 *     before anything is launched.
 *   - Set-up happens on first use: the first call on a device looks up the
 *     array's device address, and the first call of each (causal, config)
 *     variant sets its kernel's shared-memory limit. Make one call of each
 *     variant you use before any stream capture. The array itself is
 *     reserved when the library's kernels are loaded on a device (with lazy
 *     module loading, at the first launch), so make that call before a host
 *     pool claims the device's memory as well.
 *   - All calls share the one array: calls whose work overlaps on the GPU
 *     (different streams, or different host threads) race and give wrong
 *     results. Serialise them. Every byte a call reads from the array is
 *     written earlier by the same call, so nothing needs clearing and stale
 *     contents never leak.
 * Other arguments and return codes as fav4_bshd_forward. */
int fav4_bshd_forward_splitkv_static(const Fav4Args* args, int causal, int config, int splits,
                                     cudaStream_t stream);

/* Split-KV forward in one launch, for shapes with few query tiles such as
 * decoding (Sq much smaller than Sk; no reference counterpart). The keys are
 * cut into `splits` ranges of whole 128-key tiles; one kernel launch computes
 * every (query tile, key range) pair, writing per-range partial O and LSE to
 * `workspace`, and the LSE-weighted combine kernel (fav4_bshd_combine) merges
 * them into args->o / args->lse. Results equal fav4_bshd_forward within the
 * split-KV tolerance (|dO| <= 2e-2, |dLSE| <= 1e-3).
 *   - splits: 1..32, or 0 for fav4_bshd_splitkv_splits(args, causal, config);
 *     1 is fav4_bshd_forward and needs no workspace.
 *   - workspace: device memory, 256-byte aligned, at least
 *     fav4_bshd_splitkv_workspace_bytes(args, splits) bytes; calls sharing a
 *     workspace must not overlap.
 * Other arguments and return codes as fav4_bshd_forward. */
int fav4_bshd_forward_splitkv(const Fav4Args* args, int causal, int config, int splits, void* workspace,
                              size_t workspace_bytes, cudaStream_t stream);

/* fav4_bshd_forward_partial with the one-launch split: keys [kv_begin, kv_end)
 * (absolute positions) in `splits` (1..32) ranges, combined into the slice's
 * partial O and its LSE (required), as fav4_bshd_forward_partial returns them.
 * For a GPU that holds one key chunk of a multi-GPU decode step. Validation
 * and return codes as fav4_bshd_forward_partial, workspace as
 * fav4_bshd_forward_splitkv. */
int fav4_bshd_forward_partial_splitkv(const Fav4Args* args, int causal, int config, int kv_begin, int kv_end,
                                      int splits, void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* Workspace bytes fav4_bshd_forward_splitkv needs for `splits` (0 for 1 split
 * or invalid arguments). */
size_t fav4_bshd_splitkv_workspace_bytes(const Fav4Args* args, int splits);

/* The automatic number of splits on the current device: enough work tiles to
 * fit one wave over its SMs, at least 4 key tiles (512 keys) per split, at most 32. Returns
 * 1 when the query tiles alone fill the GPU, -1 on invalid arguments or a CUDA
 * error. */
int fav4_bshd_splitkv_splits(const Fav4Args* args, int causal, int config);

/* Backward pass (no reference counterpart: the reference implements the
 * forward only, README.md:24). Tensors BF16 [batch, seq, heads, 128],
 * contiguous, 16-byte aligned: q, k, v and the forward's o; dout = dL/dO; lse
 * = the forward's LSE (FP32 [batch, heads, sq], from fav4_bshd_forward with
 * a non-NULL lse). Writes dq, dk, dv (same layouts as q, k, v). */
struct Fav4BwdArgs {
  const void *q, *k, *v, *o, *dout;
  const float* lse;
  void *dq, *dk, *dv;
  int batch, heads, sq, sk;
  float scale;
};
typedef struct Fav4BwdArgs Fav4BwdArgs;

/* Device workspace fav4_bshd_backward and fav4_bshd_backward_deterministic
 * need: D = rowsum(dO * O) and LSE * log2(e) (FP32 [batch, heads, q tiles *
 * 128] each) and the FP32 dQ accumulator (batch * heads * q tiles * 128 * 128
 * floats), q tiles = ceil(sq / 128); 0 on invalid arguments. */
size_t fav4_bshd_backward_workspace_bytes(const Fav4BwdArgs* args);

/* dQ, dK, dV of O = softmax(Q K^T * scale) V (causal: top-left). On
 * `stream`: D, a zero fill of the dQ accumulator, one fused kernel (work
 * tiles of 128 keys: dK and dV, and each key tile's dQ contribution added
 * into the FP32 accumulator by atomic reductions), then the BF16 conversion
 * of dQ. dK and dV are deterministic; dQ's FP32 summation order is not.
 * Same mask convention as fav4_bshd_forward; keys no query row sees get zero
 * gradients. workspace: device memory, 256-byte aligned,
 * fav4_bshd_backward_workspace_bytes long. Returns 0, cudaErrorInvalidValue
 * (1) on invalid arguments, else the first failing launch status. */
int fav4_bshd_backward(const Fav4BwdArgs* args, int causal, void* workspace, size_t workspace_bytes,
                       cudaStream_t stream);

/* The same gradients with no atomics, bit-reproducible run to run: D, then
 * dK/dV (work tiles of 128 keys), then dQ (work tiles of 128 query rows,
 * recomputing S and dP). Slower than fav4_bshd_backward. Same arguments,
 * workspace and return values. */
int fav4_bshd_backward_deterministic(const Fav4BwdArgs* args, int causal, void* workspace,
                                     size_t workspace_bytes, cudaStream_t stream);

/* Grouped-query backward: k, v, dk and dv are [batch, sk, kv_heads, 128]
 * (kv_heads divides args->heads; query head h uses K/V head
 * h / (heads / kv_heads), as in fav4_bshd_forward_gqa). dK and dV of a K/V
 * head sum over the query heads of its group. deterministic = 0 takes the
 * fused path of fav4_bshd_backward, 1 the path of
 * fav4_bshd_backward_deterministic. Same workspace; kv_heads == heads is
 * fav4_bshd_backward / fav4_bshd_backward_deterministic. */
int fav4_bshd_backward_gqa(const Fav4BwdArgs* args, int kv_heads, int causal, int deterministic,
                           void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* Backward of fav4_bshd_forward_varlen (packed sequences). q, o, dout, dq:
 * [total_q, heads, 128]; k, v, dk, dv: [total_k, kv_heads, 128]; lse: the
 * forward's FP32 [heads, total_q]; cu_seqlens_q / cu_seqlens_k: device int32
 * offsets, batch + 1 of them, as in Fav4VarlenArgs. max_sq / max_sk bound
 * every sequence's length (rows or keys past them are not computed); both
 * size the workspace. The fused path (FP32 dQ reductions); keys no query row
 * of their sequence sees get zero gradients. */
struct Fav4VarlenBwdArgs {
  const void *q, *k, *v, *o, *dout;
  const float* lse;
  void *dq, *dk, *dv;
  const int *cu_seqlens_q, *cu_seqlens_k;
  int batch, heads, kv_heads, max_sq, max_sk, total_q, total_k;
  float scale;
};
typedef struct Fav4VarlenBwdArgs Fav4VarlenBwdArgs;

/* Device workspace fav4_bshd_backward_varlen needs (0 on invalid arguments). */
size_t fav4_bshd_backward_varlen_workspace_bytes(const Fav4VarlenBwdArgs* args);

/* Returns 0, cudaErrorInvalidValue (1) on invalid arguments, else the first
 * failing launch status. */
int fav4_bshd_backward_varlen(const Fav4VarlenBwdArgs* args, int causal, void* workspace, size_t workspace_bytes,
                              cudaStream_t stream);

/* One output of fav4_bshd_forward_host: host buffers for O (BF16
 * [batch, sq, heads, 128]) and optionally LSE (FP32 [batch, heads, sq]), and
 * the mask and config it is computed with. */
struct Fav4HostOut {
  void* o;
  float* lse;
  int causal;
  int config;
};
typedef struct Fav4HostOut Fav4HostOut;

/* Device workspace fav4_bshd_forward_host needs for these arguments, in
 * bytes (0 when the arguments are invalid). */
size_t fav4_bshd_host_workspace_bytes(const Fav4Args* args, const Fav4HostOut* outs, int n_outs, int chunks);

/* Forward from host memory (no reference counterpart: the reference's caller
 * copies to the device itself). args->q/k/v are HOST pointers (page-locked
 * memory is needed for the copies to overlap); args->o and args->lse are
 * ignored. Every output in outs[0..n_outs) (1..8 of them, e.g. a dense and a
 * causal forward of the same inputs) is computed from one upload. The batch
 * is cut into `chunks` pieces staged through two slots of `workspace`
 * (device memory, 256-byte aligned, fav4_bshd_host_workspace_bytes long):
 * the upload of one piece, the forwards of the previous one and the download
 * of the one before that overlap. Work is ordered after what is already on
 * `stream`, and `stream` waits for the last download, so a synchronise of
 * `stream` (or an event recorded on it) means the host outputs are written.
 * Results are bit-identical to fav4_bshd_forward on device copies. Calls that
 * share a workspace must not overlap. Returns 0, cudaErrorInvalidValue, or
 * the first failing CUDA status. */
int fav4_bshd_forward_host(const Fav4Args* args, const Fav4HostOut* outs, int n_outs, int chunks, void* workspace,
                           size_t workspace_bytes, cudaStream_t stream);

/* Failure detection (no reference counterpart): every pipeline wait inside the
 * kernels is bounded in time (default 2000 ms, environment variable
 * FAV4_WAIT_LIMIT_MS). A wait that runs out makes the kernel stop cleanly and
 * ORs a code into a per-device status word: 1 load, 2 mma, 4 softmax,
 * 8 drain, 16 probe. This call synchronises the current device, returns the
 * word (or -1 on a CUDA error) and clears it when `clear` is nonzero. */
int fav4_bshd_pipeline_status(int clear);

#ifdef __cplusplus
}
#endif

#endif /* FAV4_BSHD_H_ */
