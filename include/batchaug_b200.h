/*
 * batchaug_b200.h — C ABI of the B200 (sm_100a) backend for batchaug's hot
 * path: the lazily fused geometric resample and the eager intensity chain.
 *
 * Conventions
 *   - Tensors are contiguous NCDHW arrays named (B, C, H, W, D) as in
 *     batchaug; elements are fp32 or bf16.  All pointers are device pointers
 *     unless a comment says otherwise.
 *   - The caller owns every device buffer, including scratch ("workspace",
 *     sized by the matching *_workspace_bytes query).  The library never
 *     allocates or frees device memory and keeps no device state between
 *     calls.
 *   - Work is enqueued on the caller's stream; no call synchronises the host.
 *   - Every entry point returns a ba_status; ba_last_error() returns a
 *     thread-local message for the last failure on the calling thread.
 *   - Argument errors (shape, dtype, null pointer, alignment, aliasing) are
 *     BA_EINVAL; valid-but-unimplemented requests are BA_EUNSUPPORTED; CUDA
 *     launch failures are BA_ECUDA.  No error is signalled from the device by
 *     a fault or a trap.
 *
 * Reference citations are file:line in halleewong/batchaug.
 */
#ifndef BATCHAUG_B200_H
#define BATCHAUG_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define BA_API __attribute__((visibility("default")))
#else
#define BA_API
#endif

typedef struct CUstream_st* ba_stream_t; /* == cudaStream_t; NULL = legacy default stream */

typedef enum ba_status {
  BA_OK = 0,
  BA_EINVAL = 1,
  BA_EUNSUPPORTED = 2,
  BA_ECUDA = 3,
  BA_ETIMEOUT = 4
} ba_status;

typedef enum ba_dtype { BA_F32 = 0, BA_BF16 = 1 } ba_dtype;

/* grid_sample's mode: "bilinear" (trilinear on 5-D tensors) or "nearest". */
typedef enum ba_interp { BA_BILINEAR = 0, BA_NEAREST = 1 } ba_interp;

/* grid_sample's padding_mode. */
typedef enum ba_padding { BA_PAD_ZEROS = 0, BA_PAD_BORDER = 1, BA_PAD_REFLECTION = 2 } ba_padding;

/* How output voxels map to source coordinates. */
typedef enum ba_xform {
  BA_XFORM_AFFINE = 0, /* MONAI-convention affine (B,4,4); theta derived as
                          monai_affine_to_theta does (affine.py:154-195) */
  BA_XFORM_THETA = 1,  /* affine_grid theta, first 3 rows of (B,rows,4) */
  BA_XFORM_GRID = 2    /* explicit grid_sample grid (B,H,W,D,3), xyz order */
} ba_xform;

#define BA_MAX_KEYS 8

typedef struct ba_resample_key {
  const void* src; /* (B, channels, H, W, D) */
  void* dst;       /* same shape and dtype; must not overlap src */
  int64_t channels;
  int32_t dtype;   /* ba_dtype */
  int32_t mode;    /* ba_interp */
  int32_t padding; /* ba_padding */
  int32_t reserved;
  int32_t* minmax; /* optional (NULL: none): (B, channels, 2) int32 that the call
                      fills with the per-(element, channel) minimum and maximum
                      of this key's output, as statistics for a following
                      RESCALE with BA_RESCALE_GIVEN (ba_op.stats); order-
                      preserving keys, opaque to the caller.  The staged affine
                      kernel folds them as it writes; other paths reduce the
                      output after the resample. */
} ba_resample_key;

/* ba_resample_desc.flags */
#define BA_RESAMPLE_EXACT 0x1 /* trilinear weights and sums rounded as torch's CPU
                                 grid_sample rounds them (bit for bit); without it
                                 the interpolation uses fused multiply-add lerps,
                                 within 1e-5 (fp32) / 2 bf16 ulp of it.  Source
                                 coordinates, and so nearest keys, are exact in
                                 both modes. */
#define BA_RESAMPLE_HOST_PARAMS 0x2 /* xform (AFFINE / THETA maps) and mask are host
                                       pointers, read before the call returns: each
                                       launch of up to 32 elements carries them in its
                                       kernel parameters, so no device copy of them is
                                       needed (xform_stride <= 16; a GRID map's grid
                                       stays a device pointer) */

typedef struct ba_resample_desc {
  int64_t batch, H, W, D;
  int32_t xform_kind;    /* ba_xform */
  int32_t align_corners; /* grid_sample's align_corners */
  int32_t n_keys;        /* 1..BA_MAX_KEYS keys sharing one coordinate map */
  int32_t flags;         /* BA_RESAMPLE_* */
  const float* xform;   /* see ba_xform */
  int64_t xform_stride; /* floats between consecutive elements of an AFFINE or
                           THETA xform (16 for (B,4,4), 12 for (B,3,4)) */
  const uint8_t* mask;  /* (B,) 0/1, NULL = every element transformed */
  ba_resample_key keys[BA_MAX_KEYS];
} ba_resample_desc;

/*
 * One fused resample of up to BA_MAX_KEYS tensors through a shared
 * per-element coordinate map; masked-out elements are copied unchanged.
 * Replaces, per call:
 *   Compose._materialize        batchaug/compose.py:71-110
 *     (F.affine_grid + F.grid_sample(float) + .to(dtype) + torch.where, per key)
 *   RandAffine.apply            batchaug/pytorch/geometric/affine.py:284-317
 *   Rand3DElastic.apply         batchaug/pytorch/geometric/elastic.py:101-125
 *   RandRotate90.apply fallback batchaug/pytorch/geometric/rotate90.py:100-112
 * Coordinates and interpolation reproduce torch's CPU affine_grid and
 * grid_sample bit for bit (same operation order, no contraction).
 */
BA_API ba_status ba_resample3d(const ba_resample_desc* desc, ba_stream_t stream);

/*
 * Elastic field composed with the affine that follows it, as one grid
 * (an extension: the reference resamples twice, Rand3DElastic.apply
 * elastic.py:101-125 and then Compose._materialize compose.py:71-110).
 * field: the elastic grid_sample grid (B,H,W,D,3), align_corners=True, xyz
 * order (Rand3DElastic.sample_params, elastic.py:37-99); theta: affine_grid
 * theta (B,3,4) of the affine applied after it.  For output voxel p, with u
 * the affine's source position in voxels of the elastic output
 * (affine_grid + unnormalise, align_corners=False), uc = u clamped to the
 * volume and half = max((N-1)/2, 1e-6) per axis:
 *   grid(p) = trilinear(field, uc) + (u - uc) / half
 * i.e. the elastic displacement extended by clamping; sampling the input
 * once with grid (align_corners=True) gives I(field(A(p))).  Elements with
 * mask_affine[b] == 0 take grid = field; elements with mask_field[b] == 0
 * use the identity grid for field.  Either mask may be NULL (all set).
 */
BA_API ba_status ba_compose_field(const float* field, const float* theta,
                                  const uint8_t* mask_field, const uint8_t* mask_affine,
                                  int64_t batch, int64_t H, int64_t W, int64_t D, float* grid,
                                  ba_stream_t stream);

/* ---------------------------------------------------------------------- */
/* Intensity chain                                                         */
/* ---------------------------------------------------------------------- */

typedef enum ba_op_kind {
  BA_OP_NOISE = 1,      /* x + dt(noise) * dt(mask)        noise.py:62-66 */
  BA_OP_CONTRAST = 2,   /* gamma, per-element min/max      contrast.py:116-131 */
  BA_OP_SCALE = 3,      /* x * dt(1 + dt(factor))          scale_shift.py:51-56 */
  BA_OP_SHIFT = 4,      /* x + dt(offset) [clamp 0..1]     scale_shift.py:106-113 */
  BA_OP_BIAS_FIELD = 5, /* x * exp(sum c L L L)            bias_field.py:99-112 */
  BA_OP_RESCALE = 6,    /* ScaleIntensity min/max rescale  contrast.py:35-68 */
  BA_OP_RICIAN = 7,     /* sqrt((x+n1)^2 + n2^2)           noise.py:146-164 */
  BA_OP_STD_SHIFT = 8,  /* x + factor * std(x)             scale_shift.py:168-198 */
  BA_OP_FIXED_MEAN = 9  /* mean + (x - mean) * (1+factor)  scale_shift.py:252-274 */
} ba_op_kind;

/* ba_op.flags */
#define BA_NOISE_PHILOX 0x1    /* NOISE: generate N(0,1) in-kernel (Philox4x32-10) */
#define BA_SHIFT_SAFE 0x1      /* SHIFT: clamp to [0,1] */
#define BA_RESCALE_MINV 0x1    /* RESCALE: minv given */
#define BA_RESCALE_MAXV 0x2    /* RESCALE: maxv given */
#define BA_RESCALE_CHANNEL 0x4 /* RESCALE: min/max per (element, channel) */
#define BA_RESCALE_FACTOR 0x8  /* RESCALE: x * (1 + c0) instead of min/max */
#define BA_RESCALE_GIVEN 0x10  /* RESCALE (with BA_RESCALE_CHANNEL): the min/max of its
                                  input are ba_op.stats, as ba_resample3d's minmax
                                  produced them for the tensor the chain reads,
                                  instead of a reduction pass of the chain's own */
#define BA_RICIAN_PHILOX 0x1   /* RICIAN: generate u1, u2 ~ N(0,1) in-kernel */
#define BA_RICIAN_RELATIVE 0x2 /* RICIAN: std * std(x) over the element */
#define BA_STD_NONZERO 0x2     /* STD_SHIFT: std of the nonzero values (if > 1 of them) */
#define BA_STAT_CHANNEL 0x4    /* STD_SHIFT, FIXED_MEAN: statistics per (element, channel) */

#define BA_MAX_OPS 8

typedef struct ba_op {
  int32_t kind;  /* ba_op_kind */
  int32_t flags; /* BA_* flags above */
  const uint8_t* mask; /* (B,) 0/1 or NULL = every element (RESCALE ignores it) */
  const float* param;  /* NOISE: std (B,); CONTRAST: gamma (B,); SCALE: factor (B,);
                          SHIFT: offset (B,); BIAS_FIELD: coeffs (B, n_coeff);
                          RICIAN: noise_std (B,); STD_SHIFT, FIXED_MEAN: factor (B,) */
  const float* param2; /* NOISE: mean (B,); RICIAN without BA_RICIAN_PHILOX:
                          injected u2, fp32 (B,C,H,W,D) */
  const float* noise;  /* NOISE without BA_NOISE_PHILOX: injected noise, fp32
                          (B,C,H,W,D), already scaled by std and shifted by mean;
                          RICIAN without BA_RICIAN_PHILOX: injected u1 */
  uint64_t seed;        /* NOISE / RICIAN with the Philox flag: Philox key */
  uint64_t elem_offset; /* ... and the global index of element 0 */
  int32_t degree;       /* BIAS_FIELD: Legendre degree 1..6 */
  int32_t reserved;
  const int32_t* stats; /* RESCALE with BA_RESCALE_GIVEN: (B, C, 2) statistics from
                           ba_resample_key.minmax */
  double c0, c1; /* RESCALE: minv, maxv (or factor in c0 with BA_RESCALE_FACTOR);
                    RICIAN: the noise mean in c0 */
} ba_op;

typedef struct ba_chain_desc {
  const void* src; /* (B,C,H,W,D) */
  void* dst;       /* same shape/dtype; may equal src (in place), no partial overlap */
  int64_t batch, channels, H, W, D;
  int32_t dtype; /* ba_dtype; every op rounds its result to this dtype, as the
                    reference's op-by-op torch arithmetic does */
  int32_t n_ops; /* 1..BA_MAX_OPS, applied in order */
  ba_op ops[BA_MAX_OPS];
} ba_chain_desc;

/* Scratch bytes ba_intensity_chain needs for desc: the statistics of the
 * intermediate results that CONTRAST and RESCALE (min/max) and STD_SHIFT,
 * FIXED_MEAN and relative RICIAN (mean, std) read. */
BA_API size_t ba_intensity_workspace_bytes(const ba_chain_desc* desc);

/*
 * Applies a chain of intensity transforms in as few HBM passes as the
 * statistics allow.  CONTRAST and RESCALE need min/max, STD_SHIFT,
 * FIXED_MEAN and relative RICIAN need the mean or std of their own input, so
 * the chain is cut before each of them: every segment but the last writes its
 * result to dst and reduces those statistics on the fly.
 * Replaces the eager apply of RandGaussianNoise, RandAdjustContrast,
 * RandScaleIntensity, RandShiftIntensity, RandBiasField, ScaleIntensity,
 * RandRicianNoise, RandStdShiftIntensity and RandScaleIntensityFixedMean
 * (files above) and the Triton kernels batchaug/triton/kernels/
 * elementwise.py:9-110, scale_shift.py:13-241, bias_field.py:9-124,
 * rician_noise.py:21-63.
 * workspace: device scratch of ba_intensity_workspace_bytes(desc) bytes,
 * 16-byte aligned (may be NULL when that is 0).
 */
BA_API ba_status ba_intensity_chain(const ba_chain_desc* desc, void* workspace, size_t workspace_bytes,
                             ba_stream_t stream);

/*
 * ba_intensity_chain for callers that cannot allocate device memory — no
 * counterpart in the reference.  Some hosts of this library (plugin hosts,
 * embedded pipelines) own all device memory through their own pool, or call
 * the chain in a loop where cudaMalloc/cudaFree, which may synchronise the
 * device, is not allowed; they cannot supply the chain's scratch.  This entry
 * point takes it from a static device array of BA_NOALLOC_CHAIN_SCRATCH bytes
 * instead (every GPU that loads the library holds that array until the
 * process exits) and allocates nothing.  Chains needing more scratch than
 * that (see ba_intensity_workspace_bytes) are rejected with BA_EINVAL.
 * The first call on each device looks the array's device address up
 * (cudaGetSymbolAddress) and caches it; make that first call before any
 * stream capture.  All calls share the one array: calls that overlap on the
 * GPU (for example on two streams at once) race on it and must not be
 * issued.  Each call re-initialises the statistics it uses, so contents left
 * by an earlier call are never read.
 */
#define BA_NOALLOC_CHAIN_SCRATCH 262144
BA_API ba_status ba_intensity_chain_noalloc(const ba_chain_desc* desc, ba_stream_t stream);
/* The size of that static array, BA_NOALLOC_CHAIN_SCRATCH, as the library
 * was built with it (for bindings that do not read this header). */
BA_API size_t ba_noalloc_chain_scratch_bytes(void);

/*
 * Per-group min and max of a contiguous (n_groups, group_size) view, fp32
 * results in stats[2*g] (min) and stats[2*g+1] (max); a NaN in a group makes
 * both NaN.  Replaces batched_minmax, batchaug/triton/kernels/reduce.py:51-75
 * (and the min/max of contrast.py:44-51, :122-124).
 */
BA_API ba_status ba_minmax(const void* x, int32_t dtype, int64_t n_groups, int64_t group_size,
                    float* stats, ba_stream_t stream);

/* ---------------------------------------------------------------------- */
/* Gaussian smoothing and the elastic field                                */
/* ---------------------------------------------------------------------- */

/*
 * Per-element 1-D Gaussian taps, gaussian_1d_batch
 * (batchaug/pytorch/intensity/smooth.py:9-34): taps (B, K) with
 * K = 2*int(max(max(sigma)*truncated, 0.5) + 0.5) + 1; the caller passes the
 * batch maximum of sigma (max_sigma) so no device-to-host read is needed,
 * and K = ba_gauss_taps_len(max_sigma, truncated).
 */
BA_API int64_t ba_gauss_taps_len(double max_sigma, double truncated);
BA_API ba_status ba_gauss_taps(const float* sigmas, int64_t batch, int64_t K, float* taps,
                        ba_stream_t stream);

/* Border handling of each 1-D pass: conv3d's implicit zeros (padding_mode
 * None or "constant"), or F.pad's "reflect" / "replicate" before the pass. */
typedef enum ba_smooth_pad {
  BA_SMOOTH_ZEROS = 0,
  BA_SMOOTH_REFLECT = 1,
  BA_SMOOTH_REPLICATE = 2
} ba_smooth_pad;

/*
 * Separable Gaussian smoothing of (B,C,H,W,D) with per-element taps for H, W
 * and D (separable_gaussian_conv3d, smooth.py:37-88; RandGaussianSmooth.apply
 * smooth.py:110-117), fp32 compute, result cast to dtype; masked-out
 * elements are copied.  workspace: fp32 intermediates,
 * ba_smooth_workspace_bytes bytes.
 */
BA_API size_t ba_smooth_workspace_bytes(int64_t batch, int64_t channels, int64_t H, int64_t W,
                                 int64_t D);
BA_API ba_status ba_smooth3d(const void* src, void* dst, int32_t dtype, int64_t batch, int64_t channels,
                      int64_t H, int64_t W, int64_t D, const float* taps_h, int64_t Kh,
                      const float* taps_w, int64_t Kw, const float* taps_d, int64_t Kd,
                      int32_t padding, const uint8_t* mask, void* workspace,
                      size_t workspace_bytes, ba_stream_t stream);

/*
 * Unsharp masking of (B,C,H,W,D) with per-element taps and strength
 * (RandGaussianSharpen.apply, sharpen.py:117-136):
 *   blurred        = smooth(src, taps1)      cast to dtype
 *   double_blurred = smooth(blurred, taps2)  cast to dtype
 *   dst = blurred + alpha * (blurred - double_blurred), one op at a time in
 *         dtype (alpha cast to dtype first); masked-out elements copy src.
 * The combination is computed in the last pass of the second blur, so
 * double_blurred is never stored.  Replaces the Triton path
 * batchaug/triton/intensity/sharpen.py:18-38 (two separable blurs, then the
 * combination in torch).  workspace: ba_sharpen_workspace_bytes bytes, 16-byte
 * aligned; dst must not overlap src.
 */
typedef struct ba_sharpen_desc {
  const void* src;
  void* dst;
  int32_t dtype;
  int32_t padding; /* ba_smooth_pad, for both blurs */
  int64_t batch, channels, H, W, D;
  const float* taps1[3]; /* first blur, (B, K1[i]) for H, W, D */
  int64_t K1[3];
  const float* taps2[3]; /* second blur */
  int64_t K2[3];
  const float* alpha;    /* (B,) */
  const uint8_t* mask;   /* (B,) or NULL = every element */
} ba_sharpen_desc;
BA_API size_t ba_sharpen_workspace_bytes(const ba_sharpen_desc* desc);
BA_API ba_status ba_sharpen3d(const ba_sharpen_desc* desc, void* workspace, size_t workspace_bytes,
                              ba_stream_t stream);

/*
 * RandSimulateLowResolution.apply (resolution.py:74-118): per element a
 * target size t = max(1, rint(float(s) * zoom[b])) per axis, then
 * F.interpolate down to t with down_mode and back to (H, W, D) with up_mode,
 * each result cast to dtype; masked-out elements copy src.  Modes are
 * BA_INTERP_*; align_corners applies to a trilinear step.  Bit-identical to
 * torch's CPU interpolate in fp32 and bf16.  A nearest or nearest-exact
 * downsample is folded into the upsample (one pass, no scratch); trilinear
 * or area downsampling stages each element's small volume in workspace.
 * max_zoom bounds every zoom[b] (zoom values above it are clamped to it) and
 * sizes that scratch.  Replaces the per-target-size F.interpolate loop of
 * the reference (:94-116); the reference has no Triton path for it.
 */
typedef enum ba_interp_mode {
  BA_INTERP_NEAREST = 0,
  BA_INTERP_NEAREST_EXACT = 1,
  BA_INTERP_TRILINEAR = 2,
  BA_INTERP_AREA = 3
} ba_interp_mode;

typedef struct ba_lowres_desc {
  const void* src;
  void* dst; /* must not overlap src */
  int32_t dtype;
  int32_t down_mode, up_mode;
  int32_t align_corners;
  int64_t batch, channels, H, W, D;
  const float* zoom;    /* (B,) fp32 */
  const uint8_t* mask;  /* (B,) or NULL = every element */
  double max_zoom;      /* >= every zoom[b] */
} ba_lowres_desc;
BA_API size_t ba_lowres_workspace_bytes(const ba_lowres_desc* desc);
BA_API ba_status ba_lowres3d(const ba_lowres_desc* desc, void* workspace, size_t workspace_bytes,
                             ba_stream_t stream);

/*
 * Rand3DElastic.sample_params (elastic.py:37-99) from its uniform draw: grid
 * (B,H,W,D,3) = ((smooth(u*2-1) * magnitude) + centred grid) / ((N-1)/2),
 * reordered to grid_sample's xyz.  u is (B,3,H,W,D) fp32 in [0,1); when u is
 * NULL the draw is generated in-kernel with Philox keyed on
 * (seed, elem_offset + b, component, voxel).  workspace: fp32 intermediates,
 * ba_elastic_workspace_bytes bytes.
 */
BA_API size_t ba_elastic_workspace_bytes(int64_t batch, int64_t H, int64_t W, int64_t D);
BA_API ba_status ba_elastic_grid(const float* u, uint64_t seed, uint64_t elem_offset, int64_t batch,
                          int64_t H, int64_t W, int64_t D, const float* taps, int64_t K,
                          const float* magnitude, float* grid, void* workspace,
                          size_t workspace_bytes, ba_stream_t stream);

/* ---------------------------------------------------------------------- */
/* Per-element random parameters                                          */
/* ---------------------------------------------------------------------- */

/*
 * Host-side, no device work: out[e*per_elem + i] = uniform [0,1) number i of
 * global element (elem_offset + e) in parameter stream `stream` (low 16 bits)
 * of key `seed`, from Philox4x32-10.  Replaces the per-element torch.rand(B)
 * draws of every sample_params (e.g. base.py:35, affine.py:119-151,
 * noise.py:36-46, contrast.py:106-114, bias_field.py:91-96): each rank of a
 * batch-sharded run derives the same values for the same global element with
 * no collective, and the host knows them without a device read (the batch
 * maximum of sigma that sizes Gaussian taps, smooth.py:24).
 */
BA_API void ba_host_uniform(uint64_t seed, uint32_t stream, uint64_t elem_offset, int64_t n_elems,
                     int64_t per_elem, float* out);

/*
 * RandAffine's per-element parameters, on the host: replaces the tensor
 * arithmetic of RandAffine.sample_params / to_affine and the builders of
 * batchaug/pytorch/geometric/affine.py:9-151 and :229-282, plus
 * monai_affine_to_theta (affine.py:154-195) for the sampled matrices.
 * u is (batch, u_stride) uniforms: column 0 the mask draw, columns 1..15 the
 * 3 angles, 6 shears, 3 shifts and 3 scales.  Component k is
 * (u[1+k] * range_a[k] + range_b[k]) + range_c[k] when bit k of `present` is
 * set (a sampled range) and range_c[k] otherwise (a fixed value).  Bits of
 * `groups` select the factors of I @ R @ Sh @ T @ Sc that exist (1 rotate,
 * 2 shear, 4 translate, 8 scale).  Writes mask (u < prob) as 0/1 bytes, the
 * (batch, 4, 4) MONAI affines and the (batch, 4, 4) thetas (affine_grid takes
 * the first three rows) for a volume of H x W x D; any output pointer may be
 * NULL.
 */
BA_API void ba_host_rand_affine(const float* u, int64_t batch, int64_t u_stride, float prob,
                                const float* range_a, const float* range_b, const float* range_c,
                                uint32_t present, uint32_t groups, int64_t H, int64_t W, int64_t D,
                                uint8_t* mask, float* affine, float* theta);

/* ---------------------------------------------------------------------- */
/* Library                                                                 */
/* ---------------------------------------------------------------------- */

/* Thread-local description of the last failure on this thread ("" if none). */
BA_API const char* ba_last_error(void);

/* ABI version: (major << 16) | minor. */
BA_API int32_t ba_version(void);

/* Number of CUDA kernels this library has enqueued in this process (a
 * host-side counter, incremented after each successful launch). */
BA_API uint64_t ba_kernel_launches(void);

/* Status of the library's bounded device waits (the mbarrier waits of the
 * TMA-staged resample; each gives up after 2 s).  Synchronises `stream`,
 * then returns BA_ETIMEOUT, and clears the record, if any wait of any
 * earlier launch on this device ran out of time (that launch's output is
 * incomplete), else BA_OK.  The only entry point that synchronises the host.
 * No reference counterpart (library housekeeping). */
BA_API ba_status ba_wait_status(ba_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* BATCHAUG_B200_H */
