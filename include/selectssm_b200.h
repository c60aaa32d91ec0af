/*
 * selectssm_b200 -- C ABI of the B200 (sm_100a) selective-scan hot path.
 *
 * The reference (ihh/selectssm) is JAX/Flax.  Its hot path is a set of Python
 * functions traced under jit; the FFI a JAX maintainer would bind for it is an
 * XLA custom call (jax.ffi) per function.  Each entry point below is the plain
 * C function such a custom-call handler wraps; the tests and the Python host
 * bind the same functions with ctypes:
 *
 *   ssm_fwd        replaces ssm_chunked_scan / ssm_recursive_scan / ssm_scan
 *                  forward (src/selectssm/selectssm.py:37-109,
 *                  src/selectssm/ssmrecscan.py:36-88) together with the
 *                  softplus(dt) of selectssm.py:210, the D skip of :238, the
 *                  reverse/complement unflip of :230-231 and the gate of
 *                  BidirectionalMamba (selectssm.py:335-338).
 *   ssm_bwd        replaces the custom-VJP backward ssm_scan_backward
 *                  (src/selectssm/ssmrecscan.py:111-181) and JAX autodiff of
 *                  the chunked/recursive selectors, the softplus, skip and gate.
 *   ssm_fwd_bidir / ssm_bwd_bidir
 *                  both SelectiveSSM directions of BidirectionalMamba
 *                  (selectssm.py:324-338) in one launch each.
 *   ssm_conv1d_act_fwd / ssm_conv1d_act_bwd
 *                  the flip + causal depthwise nn.Conv + activation preamble
 *                  (selectssm.py:167-187) and its gradient.
 *
 * Conventions
 *   - Layout is the reference's channels-last: activations (batch, seqlen, dim),
 *     B/C (batch, seqlen, dstate), A (dim, dstate), D/delta_bias (dim).
 *   - All pointers are device pointers owned by the caller.  Every call is
 *     asynchronous on the given stream; nothing synchronises the host.
 *   - Errors mirror the reference: shapes it rejects with ValueError return
 *     SSM_ERR_SHAPE.  ssm_strerror() gives a message.
 *   - Scratch memory is caller-provided (ssm_workspace_bytes()).
 */
#ifndef SELECTSSM_B200_H_
#define SELECTSSM_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SSM_API __attribute__((visibility("default")))
#else
#define SSM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* ssm_stream_t; /* == cudaStream_t */

enum ssm_status {
  SSM_OK = 0,
  SSM_ERR_SHAPE = 1,            /* sizes the reference rejects or this build does not support */
  SSM_ERR_DTYPE = 2,            /* unsupported dtype code */
  SSM_ERR_LAUNCH = 3,           /* CUDA launch / driver error */
  SSM_ERR_TIMEOUT = 4,          /* a bounded device-side wait gave up (status word) */
  SSM_ERR_NULL = 5,             /* a required pointer is NULL */
  SSM_ERR_ALIGN = 6,            /* pointer / stride alignment not met (16 bytes) */
  SSM_ERR_WORKSPACE = 7         /* workspace missing or too small */
};

enum ssm_dtype { SSM_F32 = 0, SSM_BF16 = 1 };

enum ssm_flags {
  SSM_DELTA_SOFTPLUS = 1 << 0,  /* dt = softplus(delta + delta_bias)  (selectssm.py:210) */
  SSM_REVERSE = 1 << 1,         /* SelectiveSSM.reverse: output / z / skip in the unflipped frame */
  SSM_COMPLEMENT = 1 << 2,      /* SelectiveSSM.complement: the flip also reverses channels */
  SSM_ALIGNED_SKIP = 1 << 3     /* opt-in: skip term flipped with y (the reference adds the
                                   flipped-frame u unflipped, selectssm.py:231 then :238) */
};

enum ssm_act { SSM_ACT_NONE = 0, SSM_ACT_SILU = 1, SSM_ACT_GELU = 2, SSM_ACT_RELU = 3 };

/* Checkpoint spacing in steps.  The forward writes the state h (fp32, dstate
 * values per channel) after every SSM_CHUNK steps; the backward restarts from
 * those states. */
#define SSM_CHUNK 8

typedef struct ssm_params {
  int32_t batch, seqlen, dim, dstate;   /* B, L, D, N (N must be 16) */
  int32_t dtype;                        /* u, delta, z, out, dout, du, ddelta, dz */
  int32_t bc_dtype;                     /* B, C, dB, dC */
  int32_t flags;                        /* ssm_flags */
  int32_t gate_act;                     /* ssm_act applied to z; ignored when z == NULL */
  /* Row strides in elements between consecutive (b, l) rows; 0 means dense
   * (dim for activations, dstate for B/C).  They let the caller pass slices of a
   * wider buffer (in_proj splits, the concatenated fwd/rev output). */
  int64_t z_stride;                     /* z and dz */
  int64_t out_stride;                   /* out and dout */
  int64_t bc_stride;                    /* B, C, dB, dC */

  /* ---- forward inputs (scan frame unless noted) ---- */
  const void* u;                        /* (B,L,D) scan input x (post-conv activation)   */
  const void* delta;                    /* (B,L,D) dt before bias / softplus             */
  const float* A;                       /* (D,N)   A = -exp(A_log)                        */
  const void* Bm;                       /* (B,L,N)                                       */
  const void* Cm;                       /* (B,L,N)                                       */
  const float* D;                       /* (D)     skip weight, NULL: no skip            */
  const float* delta_bias;              /* (D)     NULL: no bias                         */
  const void* z;                        /* (B,L,D) gate input, output frame; NULL: no gate */
  /* ---- forward outputs ---- */
  void* out;                            /* (B,L,D) output frame                          */
  float* states;                        /* (B, ceil(L/8), D, N) fp32 state after every 8 steps;
                                           written by ssm_fwd, read by ssm_bwd            */
  /* ---- backward ---- */
  const void* dout;                     /* (B,L,D) output frame                          */
  void* du;                             /* (B,L,D)                                       */
  void* ddelta;                         /* (B,L,D) grad w.r.t. delta (pre-bias/softplus) */
  float* dA;                            /* (D,N)                                         */
  void* dB;                             /* (B,L,N)                                       */
  void* dC;                             /* (B,L,N)                                       */
  float* dD;                            /* (D)     required when D != NULL               */
  float* ddelta_bias;                   /* (D)     required when delta_bias != NULL      */
  void* dz;                             /* (B,L,D) required when z != NULL               */
  /* ---- scratch ---- */
  void* workspace;                      /* ssm_workspace_bytes() bytes, 256-byte aligned */
  size_t workspace_bytes;
  int32_t* status;                      /* optional device word: nonzero after a device-side
                                           failure (bounded wait gave up)                 */
} ssm_params_t;

/* Bytes of scratch (p->workspace) that ssm_fwd and ssm_bwd need for these
 * params: the forward uses it when it splits the sequence into segments, the
 * backward always; one buffer of this size serves both calls.  The scratch
 * holds per-call partial sums and the segments' carry flags (reset by the
 * call itself, on its stream), so two calls that may overlap on the GPU need
 * separate workspaces. */
SSM_API size_t ssm_workspace_bytes(const ssm_params_t* p);
/* Bytes of scratch a single-direction backward needs for these params: ssm_bwd
 * (multicast = 0) or ssm_bwd_bc_multicast (multicast = 1, which keeps no dB /
 * dC partials of its own).  Never more than ssm_workspace_bytes(p). */
SSM_API size_t ssm_bwd_workspace_bytes(const ssm_params_t* p, int multicast);
/* Bytes of scratch ssm_fwd needs for these params (0 when it needs none). */
SSM_API size_t ssm_fwd_workspace_bytes(const ssm_params_t* p);
/* Number of floats of p->states: B * ceil(L/8) * D * N. */
SSM_API size_t ssm_states_elems(const ssm_params_t* p);

/* Forward (see top of file).  Writes out and states. */
SSM_API int ssm_fwd(const ssm_params_t* p, ssm_stream_t stream);
/* Backward.  Needs the states written by ssm_fwd on the same inputs.  Writes
 * du, ddelta, dA, dB, dC and, when present, dD, ddelta_bias, dz (overwritten).
 * Every output is bit-reproducible from call to call: sums over channels (dB,
 * dC) and over steps (dA, dD, ddelta_bias) are formed in a fixed order. */
SSM_API int ssm_bwd(const ssm_params_t* p, ssm_stream_t stream);

/* Both directions of a BidirectionalMamba block in one launch each.  fwd and
 * rev are complete parameter sets (rev normally has SSM_REVERSE, and
 * SSM_COMPLEMENT when complement=True); they may share z (tie_gate) and write
 * disjoint channel ranges of one output (concatenate_fwd_rev).  When z is shared,
 * dz must not be: the two directions' dz are separate buffers for the caller to add.
 * Shapes and dtypes of the two sets must match.  Scratch: ssm_fwd_bidir uses
 * each set's own workspace; ssm_bwd_bidir uses fwd->workspace only, which must
 * then hold ssm_workspace_bytes(fwd) + ssm_workspace_bytes(rev).               */
SSM_API int ssm_fwd_bidir(const ssm_params_t* fwd, const ssm_params_t* rev, ssm_stream_t stream);
SSM_API int ssm_bwd_bidir(const ssm_params_t* fwd, const ssm_params_t* rev, ssm_stream_t stream);

/* ---- backward fused with the cross-GPU sum of dB / dC (d_inner sharding) ----
 * With the channels split across GPUs and B, C replicated, dB and dC are sums
 * over every GPU's channels (ssmrecscan.py:158-159); ssm_bwd followed by an
 * all-reduce of dB / dC (parallel.replicated_bc over NCCL) is the unfused form.
 * ssm_bwd_bc_multicast instead adds this GPU's per-tile partial sums with
 * multimem.red to `dbc_mc`, the NVLink multicast address of a float32 buffer
 * that every participating GPU has bound: dense rows [2][batch][seqlen][16], dB
 * rows first.  The NVSwitch applies each add to every GPU's copy.  Each GPU
 * zeroes its own copy and all GPUs pass a cross-GPU barrier before any GPU's
 * call; after every GPU's call and a second barrier, each copy holds the full
 * sums.  p->dB and p->dC are not written (they may be NULL); everything else
 * is as in ssm_bwd.  dbc_mc must be 16-byte aligned.  p->workspace needs
 * ssm_bwd_workspace_bytes(p, 1) bytes.  The order of the cross-GPU adds is
 * not fixed, so these dB / dC may differ in the last bits between calls.   */
SSM_API int ssm_bwd_bc_multicast(const ssm_params_t* p, float* dbc_mc, ssm_stream_t stream);

/* ---- causal depthwise conv1d + activation (selectssm.py:167-187) ----
 * u[b,t,c] = act( sum_{k<K} w[k,c] * xt[b, t+k-(K-1), c] ),
 * xt = x, or x flipped in L (and in channels with SSM_COMPLEMENT) with
 * SSM_REVERSE.  x is (B,L,D) in its own frame; u is in the scan frame.
 * w is Flax's shift_conv kernel (K,1,D) viewed as (K,D), fp32. */
typedef struct ssm_conv_params {
  int32_t batch, seqlen, dim, width;    /* B, L, D, K (1 <= K <= 8) */
  int32_t dtype;                        /* x, u, du, dx */
  int32_t flags;                        /* SSM_REVERSE | SSM_COMPLEMENT */
  int32_t act;                          /* ssm_act */
  int64_t x_stride;                     /* row stride of x and dx in elements, 0 = dim */
  const void* x;
  const float* w;
  void* u;                              /* forward output (B,L,D) dense */
  const void* du;                       /* backward input (B,L,D) dense */
  void* dx;                             /* backward output, x's layout */
  float* dw;                            /* backward output (K,D) */
  void* workspace;
  size_t workspace_bytes;
} ssm_conv_params_t;

SSM_API size_t ssm_conv1d_workspace_bytes(const ssm_conv_params_t* p);
SSM_API int ssm_conv1d_act_fwd(const ssm_conv_params_t* p, ssm_stream_t stream);
SSM_API int ssm_conv1d_act_bwd(const ssm_conv_params_t* p, ssm_stream_t stream);

/* ---- RMSNorm before the block and the residual base after it ----
 * flax.linen.RMSNorm of BidirectionalMamba (selectssm.py:306-313, norm_type
 * "rms"): y = x * rsqrt(mean(x^2) + eps) * scale over the last axis, plus, in
 * the same pass, res_base = x + res_bias (the block's residual, selectssm.py
 * :345-352, with out_proj's bias folded in) so that out_proj can accumulate
 * onto it.  Rows of `dim` contiguous elements; scale, rstd, res_bias and
 * dscale are fp32.  The backward writes dx (+ dres when given, the gradient
 * reaching x through res_base) and dscale (summed in a fixed order). */
typedef struct ssm_norm_params {
  int64_t rows;                         /* number of rows (B * L) */
  int32_t dim;                          /* 1 <= dim <= 1024 */
  int32_t dtype;                        /* x, y, res_base, dy, dres, dx */
  float eps;                            /* flax default 1e-6 */
  const void* x;
  const float* scale;                   /* (dim) */
  void* y;                              /* forward output */
  float* rstd;                          /* (rows) forward output, backward input */
  const float* res_bias;                /* (dim) or NULL */
  void* res_base;                       /* forward output x + res_bias, or NULL */
  const void* dy;                       /* backward input: gradient of y */
  const void* dres;                     /* backward input: gradient of res_base, or NULL */
  void* dx;                             /* backward output */
  float* dscale;                        /* backward output (dim) */
  void* workspace;                      /* backward scratch: ssm_rmsnorm_workspace_bytes() */
  size_t workspace_bytes;
} ssm_norm_params_t;

SSM_API size_t ssm_rmsnorm_workspace_bytes(const ssm_norm_params_t* p);
SSM_API int ssm_rmsnorm_fwd(const ssm_norm_params_t* p, ssm_stream_t stream);
SSM_API int ssm_rmsnorm_bwd(const ssm_norm_params_t* p, ssm_stream_t stream);

/* Failure-path self-test: one tiny kernel waits, with the scan kernels'
 * bounded wait, on an mbarrier that nothing arrives on; after spin_limit polls
 * (1 .. 2^24) it writes SSM_ERR_TIMEOUT to *status (a device int32) and
 * returns, leaving the context usable.  No counterpart in the reference. */
SSM_API int ssm_selftest_wait_timeout(int32_t* status, uint32_t spin_limit, ssm_stream_t stream);

/* Failure-path self-test of the backward's decoupled lookback: runs ssm_bwd
 * on p (which must describe a shape the backward cuts into segments, with
 * p->status set; otherwise SSM_ERR_SHAPE / SSM_ERR_NULL) but leaves out the
 * CTAs of the last segment, so the segment before it waits for a flag that is
 * never set.  Every wait gives up after spin_limit polls (1 .. 2^22), the
 * kernel writes SSM_ERR_TIMEOUT to *p->status and returns, and the context
 * stays usable.  The gradients it writes are undefined.  No counterpart in the
 * reference. */
SSM_API int ssm_selftest_lookback_timeout(const ssm_params_t* p, uint32_t spin_limit, ssm_stream_t stream);

/* Message for a status code (static storage). */
SSM_API const char* ssm_strerror(int status);
/* ---- backward without any device allocation ----
 * Same result as ssm_bwd, for callers that cannot allocate device memory
 * (their framework owns the allocator, or allocation is forbidden on their hot
 * path).  No counterpart in the reference.  The scratch ssm_bwd would take from
 * p->workspace comes from one static device array of SSM_NOALLOC_SCRATCH_BYTES
 * per GPU (held until the process exits); p->workspace is ignored and all
 * inputs and outputs are still the caller's.  Returns SSM_ERR_WORKSPACE when
 * ssm_bwd_workspace_bytes(p, 0) exceeds the array.  The first call on each
 * device looks up the array's device address and keeps it for the life of the
 * process; make that call before any stream capture.  A device reset
 * (cudaDeviceReset, or the primary context destroyed and re-created) makes the
 * kept address stale: do not call this after one.  Calls share the array, so
 * calls that overlap on the GPU (other streams, other host threads, same
 * device) race; the backward re-initialises every scratch byte it reads, so no
 * state leaks between calls.  This covers the backward only: the forward,
 * ssm_fwd, still takes p->workspace when it splits a long sequence into
 * segments or when B / C are bf16 (ssm_fwd_workspace_bytes(p) bytes; 0 means
 * ssm_fwd needs no workspace for these params). */
#define SSM_NOALLOC_SCRATCH_BYTES (8u << 20)
SSM_API int ssm_bwd_noalloc(const ssm_params_t* p, ssm_stream_t stream);

/* Detail (CUDA error string and call site) of the most recent SSM_ERR_LAUNCH
 * returned on the calling host thread; "" if none. */
SSM_API const char* ssm_last_error(void);
/* Number of CUDA kernels this library has launched in this process (all
 * devices, all host threads); a diagnostic for counting launches per call. */
SSM_API unsigned long long ssm_launch_count(void);
/* Library version string. */
SSM_API const char* ssm_version(void);

#ifdef __cplusplus
}
#endif
#endif /* SELECTSSM_B200_H_ */
