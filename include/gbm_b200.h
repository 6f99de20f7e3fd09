/*
 * gbm_b200.h -- C ABI of libgbm_b200.so, the B200 engine behind the
 * reference's HybridHistGBMNumbaV1_0_1 binary-logloss hot path.
 *
 * Plain pointers and sizes only.  Every call returns GBM_OK (0) or an error
 * code; gbm_last_error() gives the message.  No C++ exception crosses this
 * boundary.  The caller owns every host buffer; the context owns all device
 * memory and communicators.  One context per host thread; calls on one
 * context are serialised by the caller.
 *
 * Reference interfaces each entry point replaces (paths inside the
 * reference project, src/bsscl_gbm/estimator_v1_0_1.py = E):
 *   gbm_round           the loop body of _fit_binary, E:2849-2905:
 *                       gradients (E:2861, E:2873-2874), _build_one_tree
 *                       (E:2891 -> E:2397-2459 -> _build_tree_leafwise
 *                       E:517-823 or _build_tree_v25 E:233-508),
 *                       _post_prune_tree_jit (E:827-841),
 *                       _enforce_monotonicity (E:2461-2499), the F update
 *                       (E:2896-2897 -> predict_batch_jit E:843-861) and
 *                       the train logloss (E:2905 -> E:2320-2325).
 *   gbm_predict         predict_all_trees_jit (E:863-884) + the sigmoid of
 *                       predict_proba (E:3318-3336).
 *   gbm_sampler_*       _get_subsample_indices (E:2502-2517) on the
 *                       RandomState(random_state) stream (E:3159).
 *   gbm_bin_edges       _build_bin_edges (E:2073-2141), sample_weight=None.
 *   gbm_bin_features    _bin_features (E:2144-2189).
 */
#ifndef GBM_B200_H
#define GBM_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    GBM_OK = 0,
    GBM_ERR_ARG = 1,      /* invalid argument or size */
    GBM_ERR_ALLOC = 2,    /* host or device allocation failed */
    GBM_ERR_CUDA = 3,     /* a CUDA runtime call or kernel failed */
    GBM_ERR_STATE = 4,    /* call out of order (e.g. round before upload) */
    GBM_ERR_COMM = 5,     /* NCCL communicator error */
    GBM_ERR_TIMEOUT = 6,  /* a bounded wait ran out */
    GBM_ERR_UNSUPPORTED = 7
};

typedef struct gbm_ctx gbm_ctx;
typedef struct gbm_sampler gbm_sampler;

/* Growth and regularisation parameters of one tree (the resolved values of
 * the reference's constructor / adaptive hyper-parameters, E:1925-2029). */
typedef struct {
    double reg_lambda;        /* lambda in -G/(H+lambda) and in the gain */
    double gamma;             /* split selection needs gain > gamma (E:646) */
    double min_child_weight;  /* HL, HR >= mcw to split (E:610) */
    double learning_rate;     /* F += lr * leaf value (E:2897) */
    int32_t min_samples_leaf; /* both children need >= msl rows (E:678) */
    int32_t max_depth;
    int32_t max_leaves;       /* best-first stops after max_leaves-1 splits */
    int32_t grow_policy;      /* 0 = leaf-wise best-first, 1 = depth-wise */
    const int32_t *monotone;  /* NULL, or per-feature -1/0/+1 (E:2461-2499) */
    /* The NaN direction.  0 (the reference, E:602-621, E:668): every split
     * is bin <= threshold -> left, so the NaN bin (bin 0) always goes left.
     * 1: for every feature whose nan_bin_id[j] is 0 (its bin 0 is the NaN
     * bin, E:2113-2127) the split search also evaluates, at every bin t >= 1,
     * the split that sends NaN right (left = bins 1..t) and keeps whichever
     * gains more (NaN-left on a tie); the tree then records the direction
     * per split (gbm_tree_out.nan_right) and every partition, F update and
     * predict honours it.  No reference counterpart: parity mode is 0. */
    int32_t nan_direction;
    const int32_t *nan_bin_id;   /* [p] the reference's _nan_bin_id (0 or -1); needed when nan_direction */
} gbm_params;

/* One tree in the reference's tuple layout (E:528-537):
 * features int32, thresholds int64 (bin ids), values f64, left/right int32
 * (-1 at leaves), split gains f64.  `capacity` entries per array; the
 * leaf-wise builder needs 2*max_leaves+2, the depth-wise one
 * 2^(max_depth+1)-1. */
typedef struct {
    int32_t capacity;
    int32_t *tf;
    int64_t *tt;
    double *tv;
    int32_t *tl;
    int32_t *tr;
    double *sg;
    int32_t n_nodes;          /* out: node_count */
    int32_t *leaf_of_row;     /* optional [n]: leaf node id of every row */
    int32_t *nan_right;       /* optional [capacity]: 1 where the split sends NaN right (nan_direction) */
} gbm_tree_out;

/* A packed ensemble, as _pack_tree_list builds it (E:2192-2216). */
typedef struct {
    const int16_t *features;   /* [total_nodes], -1 at leaves */
    const int64_t *thresholds; /* [total_nodes] bin ids */
    const double *values;      /* [total_nodes] */
    const int32_t *left;       /* [total_nodes] tree-local ids */
    const int32_t *right;      /* [total_nodes] */
    const int32_t *offsets;    /* [n_trees+1] */
    int32_t n_trees;
    const uint8_t *nan_right;  /* optional [total_nodes]: 1 where the split sends the NaN bin right
                                  (a model trained with nan_direction); NULL = the reference's NaN-left */
} gbm_packed;

/* ---- context ---------------------------------------------------------- */

/* Create a context on CUDA device `device`.  Fails with GBM_ERR_CUDA when
 * no such device exists (there is no CPU fallback).  The reference's device
 * switch (E:1852-1856, E:2408-2421) falls back to the CPU instead. */
int gbm_ctx_create(int32_t device, gbm_ctx **out);
/* Frees the context's device memory and communicator (no reference
 * counterpart: the reference holds no device state). */
void gbm_ctx_destroy(gbm_ctx *ctx);
const char *gbm_last_error(const gbm_ctx *ctx);

/* Join an NCCL communicator of `nranks` processes (one per GPU); no reference
 * counterpart (the reference runs on one host).  `uid` is
 * the 128-byte ncclUniqueId made by rank 0 and shared by the caller.
 * Histograms are then summed over ranks (exact int64 words), so every rank
 * builds the identical tree from its own row shard.  `timeout_ms` bounds
 * communicator creation and every collective wait.  Bins uploaded before
 * this call are re-scanned with an all-reduce, so every rank must have
 * uploaded its rows before it, or none. */
int gbm_ctx_init_comm(gbm_ctx *ctx, const void *uid, int32_t nranks, int32_t rank,
                      int32_t timeout_ms);
int gbm_nccl_unique_id(void *uid_out /* 128 bytes */);

/* ---- training --------------------------------------------------------- */

/* Upload this rank's rows of the binned matrix.  `xbin` is row-major
 * uint8 [n][p]; ids >= bin_counts[j] are read as bin_counts[j]-1 (the
 * reference clamps them the same way in its histograms, E:593-594, and no
 * threshold can separate them, E:604).  Rows are stored column-blocked on
 * the device ([ceil(p/16)][n][16] bytes).  bin_counts[j] is 1..257: n_bins
 * 256 (the reference's default, 'auto') gives a feature with NaN up to 257
 * bins (E:2111-2127); such a feature keeps min(id, 255) in its byte and the
 * rows of id 256 as a bit per row (uint8 input cannot hold id 256). */
int gbm_upload_bins(gbm_ctx *ctx, const uint8_t *xbin, int64_t n, int32_t p,
                    const int32_t *bin_counts);

/* The same from the reference's own uint16 bin matrix (bin_features'
 * output dtype, E:2144-2190): the ids are narrowed to uint8 while they are
 * staged and clamped on the device, so the caller needs no conversion
 * pass; the ids of 256 of a 257-bin feature become its row bits. */
int gbm_upload_bins_u16(gbm_ctx *ctx, const uint16_t *xbin, int64_t n, int32_t p,
                        const int32_t *bin_counts);

/* ---- binning on the device --------------------------------------------- */

/* Bin edges of a raw feature matrix, computed on the GPU exactly as
 * _build_bin_edges (E:2073-2141) computes them for sample_weight=None:
 * NaN bin 0 for features with NaN, the sorted distinct values when there
 * are at most n_bins (- 1 with a NaN bin) of them, else np.percentile at
 * linspace(0, 1, k) (NumPy's 'linear' arithmetic) made unique, then the
 * appended e[-1] + 1e-8 in the values' dtype.  X is host row-major [n][p],
 * dtype 0 = float32, 1 = float64.  is_cat: NULL or [p] flags of categorical
 * features (edges arange(-0.5, 64.5), 64 bins, E:2086-2090).  edges_out is
 * [p][stride] float64 with stride >= max(n_bins + 2, 65); each row is padded
 * with its last edge, so edges_out[:, :max_b] is the reference's edges_2d,
 * counts_out its bin_counts, nan_bin_out its _nan_bin_id (0 or -1) and
 * *max_b_out = max(counts) + 1.  n_bins in 2..1023.  The matrix stays on the
 * device for gbm_upload_binned_rows. */
int gbm_bin_edges(gbm_ctx *ctx, const void *X, int64_t n, int32_t p, int32_t dtype, int32_t n_bins,
                  const uint8_t *is_cat, double *edges_out, int32_t stride, int32_t *counts_out,
                  int32_t *nan_bin_out, int32_t *max_b_out);

/* The training matrix from rows [row_lo, row_hi) of the matrix last given to
 * gbm_bin_edges, binned on the GPU with the given edges (_bin_features,
 * E:2144-2189) and stored like gbm_upload_bins stores its rows (bin counts
 * <= 257).  Replaces the host binning + gbm_upload_bins of a raw matrix;
 * frees the matrix kept by gbm_bin_edges. */
int gbm_upload_binned_rows(gbm_ctx *ctx, int64_t row_lo, int64_t row_hi, const double *edges,
                           int32_t stride, const int32_t *counts, const int32_t *nan_bin);

/* The reference's raw bin ids of a host matrix (_bin_features, E:2144-2189),
 * computed on the GPU: out is host uint16 [n][p].  edges/counts/nan_bin as
 * gbm_bin_edges returns them (bin counts <= 1024). */
int gbm_bin_features(gbm_ctx *ctx, const void *X, int64_t n, int32_t p, int32_t dtype,
                     const double *edges, int32_t stride, const int32_t *counts,
                     const int32_t *nan_bin, uint16_t *out);

/* Labels (0/1) of this rank's rows, the two class weights of
 * _compute_class_weights (E:2570-2603) and the base score (E:2829-2835).
 * Resets F to base_score and computes round-0 gradients.  `n_global` is the
 * row count over all ranks (the logloss divisor; 0 = this rank's n). */
int gbm_upload_labels(gbm_ctx *ctx, const uint8_t *y, const double class_w[2],
                      double base_score, int64_t n_global);

/* ---- regression (E:2607-2705) ------------------------------------------ */

/* Float64 targets of this rank's rows, the initial score (the mean of all
 * targets, E:2612) and the loss: 0 = mse (g = F - y), 1 = mae
 * (g = sign(F - y)); h = 1.  Each round's fixed-point grid 2^-S follows the
 * round's largest |g| (the smallest S over ranks), so the integer sums stay
 * exact whatever the targets' scale. */
int gbm_upload_targets(gbm_ctx *ctx, const double *y, double init_score, int32_t loss, int64_t n_global);

/* One regression round (the loop body of _fit_regression, E:2625-2663): the
 * tree from the current gradients, F += lr * value(leaf), the train loss
 * mean((y - F)^2) or mean(|y - F|), then the next round's gradients.
 * gbm_get_grad / gbm_get_F / gbm_scale_bits give the next round's state. */
int gbm_round_reg(gbm_ctx *ctx, const uint8_t *inbag_mask, const int32_t *feat_idx, int32_t nfeat,
                  const gbm_params *params, gbm_tree_out *out, double *train_loss);

/* ---- multi-class softmax (E:2949-3065) --------------------------------- */

/* Labels 0..n_classes-1 (3 <= n_classes <= 64) of this rank's rows and the
 * per-class weights of _compute_class_weights (E:2570-2603).  F starts at 0
 * for every class (E:2959); the first round's gradients are computed here. */
int gbm_upload_labels_mc(gbm_ctx *ctx, const uint8_t *y, int32_t n_classes, const double *class_w,
                         int64_t n_global);

/* One multi-class round: K = n_classes trees on the same in-bag rows and
 * features, tree k from the softmax gradients of class k at the round's
 * start (E:2989-3006; hessians floored at 1e-8), F of class k updated after
 * its tree, then the next round's gradients and the multi-class logloss
 * (E:3008, E:2335-2341).  `outs` [n_classes]. */
int gbm_round_mc(gbm_ctx *ctx, const uint8_t *inbag_mask, const int32_t *feat_idx, int32_t nfeat,
                 const gbm_params *params, gbm_tree_out *outs, double *train_loss);

/* F [n_classes][n] (class-major), and class k's current (g, h) as the engine
 * holds them (each rounded to the 2^-S grid). */
int gbm_get_F_mc(gbm_ctx *ctx, double *F_out);
int gbm_get_grad_mc(gbm_ctx *ctx, int32_t k, double *g_out, double *h_out);

/* One boosting round, the body of _fit_binary's loop (E:2849-2905).
 * `inbag_mask` [n] marks this rank's in-bag rows
 * (the subsample); `feat_idx` [nfeat] the sorted column subsample.  Writes
 * the pruned tree to `out`, updates F on the device and returns the train
 * logloss over all rows of all ranks. */
int gbm_round(gbm_ctx *ctx, const uint8_t *inbag_mask, const int32_t *feat_idx, int32_t nfeat,
              const gbm_params *params, gbm_tree_out *out, double *train_loss);

/* gbm_round with the round's subsample taken from `sampler`
 * (_get_subsample_indices, E:2502-2517) over the
 * global row ids of all ranks): the next draw's row ids are copied to the
 * device and this rank's in-bag mask (rows row_offset .. row_offset+n-1) is
 * built there.  Same results as gbm_round with the equivalent mask. */
int gbm_round_sampled(gbm_ctx *ctx, gbm_sampler *sampler, int64_t row_offset, const gbm_params *params,
                      gbm_tree_out *out, double *train_loss);

/* gbm_round_mc with the round's sample drawn from `sampler` as in
 * gbm_round_sampled (the shuffle applied on the device, E:2502-2517), the
 * loop body of _fit_multiclass (E:2989-3008): the same K trees and loss as
 * gbm_round_mc with the equivalent mask.  Replaces the host's full shuffle
 * of every round (gbm_sampler_next with a mask). */
int gbm_round_mc_sampled(gbm_ctx *ctx, gbm_sampler *sampler, int64_t row_offset, const gbm_params *params,
                         gbm_tree_out *outs, double *train_loss);

/* gbm_round_reg with the round's sample drawn from `sampler` as in
 * gbm_round_sampled, the loop body of _fit_regression (E:2625-2663): the
 * same tree and loss as gbm_round_reg with the equivalent mask. */
int gbm_round_reg_sampled(gbm_ctx *ctx, gbm_sampler *sampler, int64_t row_offset, const gbm_params *params,
                          gbm_tree_out *out, double *train_loss);

/* n_rounds consecutive gbm_round_sampled calls, the fit loop of
 * _fit_binary (E:2849-2905): outs[r] and train_loss[r] get round r's tree
 * and loss, identical to calling gbm_round_sampled n_rounds times.  When
 * the tree is replayed on the device (depth-wise growth, or best-first with
 * max_depth <= 10) the rounds are queued back to back with no host wait in
 * between (up to 4 in flight; with a communicator, each round is replayed
 * from a CUDA graph captured on the first call with these parameters);
 * otherwise, or when any outs[r].leaf_of_row is set, the rounds run one by
 * one. */
int gbm_fit_rounds(gbm_ctx *ctx, gbm_sampler *sampler, int64_t row_offset, const gbm_params *params,
                   int32_t n_rounds, gbm_tree_out *outs, double *train_loss);

/* One tree from caller-supplied float64 gradients and hessians [n] (this
 * rank's rows): the reference's internal seam _build_one_tree(X_bin, grad,
 * hess, sample_idx, feat_idx, n_features) (E:2397-2459), including the
 * post-prune and monotone clipping.  F is not touched; call
 * gbm_upload_labels again before the next gbm_round. */
int gbm_build_tree(gbm_ctx *ctx, const double *grad, const double *hess, const uint8_t *inbag_mask,
                   const int32_t *feat_idx, int32_t nfeat, const gbm_params *params,
                   gbm_tree_out *out);

/* Fixed-point exponent S of the current fit: every g and h is rounded once
 * to the grid 2^-S and all sums are exact integer sums (no reference
 * counterpart: the reference sums float64 in row order, E:582-596). */
int32_t gbm_scale_bits(const gbm_ctx *ctx);

/* Copy device state to the host (for parity checks): F [n] (the reference's
 * F_train, E:2896-2897), and the f64 gradient/hessian of the NEXT round's
 * inputs [n] (E:2861, E:2873-2874). */
int gbm_get_F(gbm_ctx *ctx, double *F_out);
int gbm_get_grad(gbm_ctx *ctx, double *g_out, double *h_out);

/* Failure-detection self test; no reference counterpart.  With several
 * ranks each histogram level waits, on the device and with a time limit, for
 * every peer's signal (the peer exchange of the staging histograms); a wait
 * that runs out is reported as GBM_ERR_TIMEOUT by the round.  This runs that
 * wait on `device` for a signal no rank will send, limited to `timeout_ms`
 * (1..10000), and returns GBM_ERR_TIMEOUT when the wait ran out and said so.
 * One GPU; nothing is left waiting. */
int gbm_test_peer_wait(int32_t device, int32_t timeout_ms);

/* ---- predict ---------------------------------------------------------- */

/* F[i] = base + sum_t lr * values[leaf_t(i)] (predict_all_trees_jit,
 * E:863-884) and proba = sigmoid(clip(F)) (predict_proba, E:3318-3336) for
 * row-major uint8 bins [n][p].  Either output may be NULL. */
int gbm_predict(gbm_ctx *ctx, const uint8_t *xbin, int64_t n, int32_t p,
                const gbm_packed *model, double learning_rate, double base_score,
                double *F_out, double *proba_out);

/* Device-resident predict: upload the ensemble and the bins once, then run
 * on the device copies (outputs stay on the device until fetched).  The
 * same computation as gbm_predict (E:863-884, E:3318-3336), split into its
 * steps. */
int gbm_predict_set_model(gbm_ctx *ctx, const gbm_packed *model, int32_t n_features);

/* The checks gbm_predict_set_model (and so gbm_predict / gbm_predict_raw)
 * applies to a packed ensemble before anything is uploaded, on the host
 * only (no device needed): offsets start at 0 and increase (no empty tree),
 * a tree holds at most 32767 nodes, and every internal node has a feature
 * below n_features, a threshold >= 0 and both children after it inside its
 * tree, so every walk ends.  The reference's predict_all_trees_jit
 * (E:863-884) trusts its arrays; a malformed model there loops or reads out
 * of bounds.  Returns GBM_ERR_ARG / GBM_ERR_UNSUPPORTED with a message in
 * errbuf (optional, errlen bytes). */
int gbm_check_model(const gbm_packed *model, int32_t n_features, char *errbuf, int32_t errlen);
int gbm_predict_upload(gbm_ctx *ctx, const uint8_t *xbin, int64_t n, int32_t p);
/* The predict rows as the reference's uint16 bin ids (E:2144-2190): ids
 * above 255 are read as bin 256 (the top bin of a 257-bin feature; a
 * threshold of 255 sends it right, one above 255 left). */
int gbm_predict_upload_u16(gbm_ctx *ctx, const uint16_t *xbin, int64_t n, int32_t p);
int gbm_predict_run(gbm_ctx *ctx, double learning_rate, double base_score);
int gbm_predict_fetch(gbm_ctx *ctx, double *F_out, double *proba_out);

/* predict_proba from a raw host matrix (E:3274-3336): the rows are binned on
 * the GPU (_bin_features, E:2144-2189) into the predict input, then the
 * ensemble runs as in gbm_predict.  gbm_predict_upload_raw is the upload
 * step of the device-resident sequence above. */
int gbm_predict_upload_raw(gbm_ctx *ctx, const void *X, int64_t n, int32_t p, int32_t dtype,
                           const double *edges, int32_t stride, const int32_t *counts,
                           const int32_t *nan_bin);
int gbm_predict_raw(gbm_ctx *ctx, const void *X, int64_t n, int32_t p, int32_t dtype,
                    const double *edges, int32_t stride, const int32_t *counts,
                    const int32_t *nan_bin, const gbm_packed *model, double learning_rate,
                    double base_score, double *F_out, double *proba_out);

/* Ensemble predict that allocates nothing.  No counterpart in the reference:
 * this entry point exists for callers that cannot allocate device memory --
 * a serving process whose GPU memory is one arena handed out by its own
 * allocator, a framework that owns the whole device, or a latency-bound
 * path where cudaMalloc (which can synchronise the device) is not allowed.
 * Every input and output is a device pointer the caller owns: bins
 * row-major uint8 [n][p] (ids clamped to bin_count-1, as gbm_predict
 * reads them), the packed ensemble of _pack_tree_list (features int16,
 * thresholds int64, values f64, left/right int32 [n_nodes], offsets int32
 * [n_trees+1]), and F and/or proba f64 [n].  The only scratch -- the
 * ensemble rewritten as 8-byte nodes, and the walk's list of tree chunks --
 * lives in one fixed device array inside this library, sized for at most
 * 524,288 nodes and 65,536 trees (about 4.3 MiB); every GPU that loads the
 * library holds that array until the process exits.  Larger ensembles are
 * rejected with GBM_ERR_ARG, as are malformed ones (offsets that do not
 * increase or pass n_nodes, a child that is not after its parent inside its
 * tree, a feature >= p, a threshold outside 0..255).  The first call on a
 * device looks up the array's device address; make that first call before
 * any stream capture.  All calls share the array, so calls that overlap on
 * the GPU race: serialise them (one stream, or wait between calls).  The
 * walk is bounded by each tree's size taken from the caller's own offsets,
 * so an overlapping call can make the outputs wrong but cannot make the
 * walk loop or read outside the arrays.  The call runs on `stream` (a
 * cudaStream_t, NULL = the default stream) of the current device,
 * synchronises that stream and returns when the outputs are written, so
 * it cannot be captured into a CUDA graph.
 * `errbuf` (optional, `errlen` bytes) receives a message. */
int gbm_predict_noalloc(const uint8_t *xbin_dev, int64_t n, int32_t p, const int16_t *features_dev,
                        const int64_t *thresholds_dev, const double *values_dev, const int32_t *left_dev,
                        const int32_t *right_dev, const int32_t *offsets_dev, int32_t n_trees,
                        int32_t n_nodes, double learning_rate, double base_score, double *F_dev,
                        double *proba_dev, void *stream, char *errbuf, int32_t errlen);

/* Synchronise the context's stream; returns the first asynchronous error
 * (no reference counterpart). */
int gbm_sync(gbm_ctx *ctx);

/* ---- instrumentation -------------------------------------------------- */

typedef struct {
    int64_t kernel_launches;   /* every kernel this context launched */
    int64_t hist_launches;     /* histogram kernel launches */
    int64_t hist_rows;         /* rows the histogram kernel read */
    int64_t waves;             /* batched node expansions */
    double hist_ms;            /* summed CUDA-event time of the histogram
                                  launches (only while profiling is on) */
    double hist_alg_bytes;     /* algorithmic bytes of the histograms the
                                  reference builds: rows x (nfeat + 8) of the
                                  root and of the smaller child of every
                                  executed split */
    double host_sample_ms;     /* host time waiting for the sampler's draws */
    double host_sync_ms;       /* host time waiting for the device */
    double host_replay_ms;     /* host time in the best-first replay */
    double flush_ms;           /* device time of the gbm_set_l2_flush writes */
    double hist_updates;       /* histogram cell updates (row x selected feature, skipped bin
                                  excluded) of the reference's histograms; 6 shared-memory
                                  atomic adds each */
    double host_comm_ms;       /* host time in the collective calls (enqueue) */
    double comm_ms;            /* device time of the collectives (profiling), waits for peers included */
    double comm_bytes;         /* bytes this rank all-reduced or pulled from peers */
    double peer_wait_ms;       /* peer exchange: time spent waiting for the peers' signals */
    double sampler_ms;         /* device time of the rounds' sampler-stream work (the row
                                  shuffle, mask, root row list, packed feature blocks), from
                                  the start of each round's work to its end (profiling) */
    double sampler_stall_ms;   /* device time the engine stream waited for that work (profiling) */
} gbm_stats;

/* Instrumentation (no reference counterpart; the reference's times dict,
 * E:3226-3240, holds wall times only). */
int gbm_set_profiling(gbm_ctx *ctx, int32_t on);
int gbm_get_stats(gbm_ctx *ctx, gbm_stats *out);
int gbm_reset_stats(gbm_ctx *ctx);
/* Benchmark aid (no reference counterpart): with bytes > 0, every round
 * starts with a write of `bytes` of device scratch on the context's stream,
 * which evicts the L2 cache between timed rounds; its device time is
 * reported in gbm_stats.flush_ms while profiling is on.  0 turns it off. */
int gbm_set_l2_flush(gbm_ctx *ctx, int64_t bytes);
/* CUDA events on the context's stream (slots 0..15), for timing regions
 * (no reference counterpart; the reference times with perf_counter,
 * E:3226-3240). */
int gbm_event_record(gbm_ctx *ctx, int32_t slot);
int gbm_event_elapsed(gbm_ctx *ctx, int32_t a, int32_t b, float *ms);

/* ---- sampler (host) --------------------------------------------------- */

/* The reference's RandomState(seed) row/feature subsample stream
 * (E:2502-2517): every call reproduces the next round's sample_idx (first
 * n_sub of the cumulatively shuffled arange(n)) and sorted feat_idx.
 * `look_ahead` > 0 keeps that many rounds ready, drawn by two host threads
 * (swap targets / swaps) while the caller trains. */
int gbm_sampler_create(uint32_t seed, int64_t n, int32_t p, int64_t n_sub, int32_t n_feat,
                       int32_t subsample_on, int32_t colsample_on, int32_t look_ahead,
                       gbm_sampler **out);
/* A throughput-mode sampler (no reference counterpart; off the parity
 * paths): the features are drawn as above, but each round's in-bag rows are
 * drawn on the device by the engine -- row i (global id) is in-bag in round
 * r iff a counter-based hash of (seed, r, i) is below subsample * 2^64, so
 * each row is in with probability `subsample` (the in-bag count varies
 * around n * subsample) and every rank draws its own rows with no host work
 * and no exchange, identically at any GPU count.  The reference's sampler
 * (_get_subsample_indices, E:2502-2517) is a cumulative shuffle whose host
 * cost grows with n (~7 ms per round at 10M rows); this one has none.  Only
 * the engine's round calls (gbm_round_sampled, gbm_fit_rounds) accept it;
 * gbm_sampler_next / _next_rows answer GBM_ERR_STATE. */
int gbm_sampler_create_device(uint32_t seed, int64_t n, int32_t p, double subsample, int32_t n_feat,
                              int32_t colsample_on, int32_t look_ahead, gbm_sampler **out);

/* The next round's draw of _get_subsample_indices (E:2502-2517).  Any output
 * may be NULL: sample_idx [n_sub] (reference order), inbag_mask [n] (1 = in
 * bag), feat_idx [n_feat]. */
int gbm_sampler_next(gbm_sampler *s, int64_t *sample_idx, uint8_t *inbag_mask, int32_t *feat_idx);
/* The next round as int32 row ids [n_sub] (reference order) + feat_idx. */
int gbm_sampler_next_rows(gbm_sampler *s, int32_t *sample_rows, int32_t *feat_idx);
/* The sizes the sampler was made with (n_sub = int(n * subsample), n_feat =
 * int(p * colsample_bytree), E:2502-2517), and its destruction. */
int64_t gbm_sampler_n_sub(const gbm_sampler *s);
int32_t gbm_sampler_n_feat(const gbm_sampler *s);
void gbm_sampler_destroy(gbm_sampler *s);

#ifdef __cplusplus
}
#endif

#endif /* GBM_B200_H */
