/*
 * boa_b200.h — C-ABI of libboa_b200.so, the B200 (sm_100a) compress/decompress
 * hot path of BoaConstrictor.
 *
 * Conventions (every entry point):
 *   - returns BOA_OK (0) or a BOA_ERR_* code; boa_last_error() gives a message
 *     for the calling thread;
 *   - pointers named d_* are device pointers on the handle's device, h_* /
 *     host_* are host pointers; sizes are in elements unless named *_bytes;
 *   - `stream` is a cudaStream_t passed as void*; work is stream-ordered and
 *     nothing synchronises the device.  Calls that return host data
 *     (boa_rc_get_*, boa_model_status) and boa_rc_encode_noalloc synchronise
 *     only `stream`; every other call only enqueues work.
 *   - errors found on the device (a bounded wait that timed out, a stream that
 *     outgrew its pitch, a symbol outside the vocabulary) cannot be returned
 *     by the call that enqueued the work: they are recorded on the device and
 *     reported by the next host-returning call on the same object
 *     (boa_rc_get_sizes / boa_rc_get_words for a coder, boa_model_status for
 *     a model).
 *   - no torch or C++ types cross this boundary.
 *
 * Reference interfaces replaced (paths relative to the reference project root):
 *   boa_rc_*      : pybind11 class RangeCoderBatch, gpu_range_coder.py:212-324,
 *                   wrapped by gpu.queue.RangeCoderBatch, gpu_range_coder.py:488-550
 *   boa_model_*   : BoaConstrictor / BoaBytePredictor.step, model.py:5,83-131,
 *                   weights in the order of portability_solved_cpp/convert_boa_weights.py:16-135
 *   boa_codec_*   : the per-byte step loops compress_GPU / decompress_GPU,
 *                   codec.py:11-86 and codec.py:89-151 (model step + softmax +
 *                   coder step per byte), fused into one persistent kernel
 */
#ifndef BOA_B200_H
#define BOA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BOA_API __attribute__((visibility("default")))

#define BOA_ABI_VERSION 1

#define BOA_OK 0
#define BOA_ERR_ARG 1        /* invalid argument / shape (reference: std::runtime_error) */
#define BOA_ERR_CUDA 2       /* a CUDA runtime call failed */
#define BOA_ERR_OVERFLOW 3   /* a compressed stream needed more words than its pitch */
#define BOA_ERR_TIMEOUT 4    /* a bounded device-side wait gave up */
#define BOA_ERR_UNSUPPORTED 5
#define BOA_ERR_RANGE 6      /* a model activation outside the operand kind's range (BOA_WEIGHTS_F16X2) */

/* Frequency-table quantisers. */
#define BOA_QUANT_REF 0  /* fp32 probabilities -> reference build_cdf_fast (gpu_range_coder.py:57-79) */
#define BOA_QUANT_BQ 1   /* fp32 logits -> this build's integer quantiser (no reference counterpart) */

/* Projection weight formats for the model kernel. */
#define BOA_WEIGHTS_TF32 0  /* fp32 weights, tf32 tensor-core products, fp32 accumulation */
#define BOA_WEIGHTS_BF16 1  /* bf16 weights and activations, fp32 accumulation and state */
#define BOA_WEIGHTS_F16 2   /* fp16 weights and activations (tf32-equal mantissa), fp32 accumulation and state */
#define BOA_WEIGHTS_TF32X3 3 /* fp32 weights and activations, each split into tf32 hi + lo halves whose
                                products are summed in fp32 (3xTF32): the fp32-equivalent kind, and the
                                one that matches the reference's fp32 nn.Linear (model.py:47-56,90-95) */
#define BOA_WEIGHTS_F16X2 4  /* fp32 weights and activations, each split into an fp16 hi and an fp16
                                residual scaled by 2^11 (22 significant bits, as 3xTF32) with fp32
                                accumulation: half the weight bytes of BOA_WEIGHTS_TF32X3.  Activations
                                must stay below 65504 in magnitude; otherwise the call reports
                                BOA_ERR_RANGE.  d_model 64 and 256. */

BOA_API const char* boa_last_error(void);
BOA_API int boa_abi_version(void);

/* ------------------------------------------------------------------------ */
/* Batched range coder (gpu_range_coder.py:212-324).                        */
/* ------------------------------------------------------------------------ */
typedef struct boa_rc_batch boa_rc_batch;

/* RangeCoderBatch(int N, int K, int pitch) (gpu_range_coder.py:219-230).
 * precision: 24 reproduces the reference coder bit for bit (with
 * BOA_QUANT_REF); 16 is the north-star table total.  Allocates the per-stream
 * coder state and N*pitch_words output words on `device`. */
BOA_API int boa_rc_create(boa_rc_batch** out, int n_streams, int k_symbols, int pitch_words,
                          int precision, int quantiser, int device);
/* ~RangeCoderBatch (gpu_range_coder.py:231-236). */
BOA_API int boa_rc_destroy(boa_rc_batch* b);
BOA_API int boa_rc_info(const boa_rc_batch* b, int* n_streams, int* k_symbols, int* pitch_words,
                        int* precision, int* quantiser);
/* load_compressed_from_host (gpu_range_coder.py:237-253): host_words is
 * [n_streams, pitch_words] (zero padded), host_sizes[n_streams] in words. */
BOA_API int boa_rc_load(boa_rc_batch* b, const uint32_t* host_words, const int32_t* host_sizes, void* stream);
/* set_sizes_from_host (gpu_range_coder.py:259-264). */
BOA_API int boa_rc_set_sizes(boa_rc_batch* b, const int32_t* host_sizes, void* stream);
/* get_sizes_host (gpu_range_coder.py:254-258); reports BOA_ERR_OVERFLOW if a
 * stream ran past its pitch. */
BOA_API int boa_rc_get_sizes(boa_rc_batch* b, int32_t* host_sizes, void* stream);
/* get_compressed_host (gpu_range_coder.py:278-292), as one [n, pitch] block. */
BOA_API int boa_rc_get_words(boa_rc_batch* b, uint32_t* host_words, void* stream);
/* Device addresses of the [n, pitch] word block and the size vector. */
BOA_API int boa_rc_device_buffers(boa_rc_batch* b, uint32_t** d_words, int32_t** d_sizes);
/* encode_step_from_device (gpu_range_coder.py:265-272): one symbol per active
 * stream.  d_rows is [n, K] fp32: probabilities for BOA_QUANT_REF, logits for
 * BOA_QUANT_BQ.  d_mask (u8, may be NULL) skips streams with mask 0. */
BOA_API int boa_rc_encode_step(boa_rc_batch* b, const int32_t* d_symbols, const float* d_rows,
                               const uint8_t* d_mask, void* stream);
/* finalize (gpu_range_coder.py:273-277). */
BOA_API int boa_rc_finalize(boa_rc_batch* b, void* stream);
/* init_decoder_from_current_bytes (gpu_range_coder.py:293-297). */
BOA_API int boa_rc_init_decoder(boa_rc_batch* b, void* stream);
/* decode_step_to_device (gpu_range_coder.py:298-305). */
BOA_API int boa_rc_decode_step(boa_rc_batch* b, const float* d_rows, int32_t* d_out_symbols,
                               const uint8_t* d_mask, void* stream);

/* Multi-step forms of encode_step / decode_step (no counterpart in the
 * reference, which launches once per symbol, gpu_range_coder.py:265-305):
 * one launch codes n_steps symbols per stream, the coder state held in
 * registers across the steps.  Step t uses slot (t % period) of each per-step
 * array (period <= 0: slot t): rows at d_rows + slot * row_stride ([n, K]
 * fp32 logits), symbols at d_symbols + slot * sym_stride (encode), outputs at
 * d_out_symbols + slot * out_stride (decode), mask bytes at d_mask + slot *
 * mask_stride (NULL: every stream codes every step).  Strides are in
 * elements.  Same bits as n_steps single-step calls.  BOA_QUANT_BQ only. */
BOA_API int boa_rc_encode_steps(boa_rc_batch* b, int n_steps, int period, const int32_t* d_symbols,
                                int64_t sym_stride, const float* d_rows, int64_t row_stride, const uint8_t* d_mask,
                                int64_t mask_stride, void* stream);
BOA_API int boa_rc_decode_steps(boa_rc_batch* b, int n_steps, int period, const float* d_rows, int64_t row_stride,
                                int32_t* d_out_symbols, int64_t out_stride, const uint8_t* d_mask,
                                int64_t mask_stride, void* stream);

/* Allocation-free whole-stream encode (no counterpart in the reference).
 * For callers that cannot allocate device memory while they code: hosts and
 * plugin frameworks that own the device memory pool and forbid allocation
 * after start-up, or real-time services that must not stall on cudaMalloc.
 * Codes n_steps symbols of each of n_streams streams with the BQ quantiser,
 * then finalises, using a static per-device scratch array (2 MiB, held by
 * every GPU that loads the library until exit) for the coder state instead of
 * memory from boa_rc_create.  d_logits is [n_steps][n_streams][K] fp32 (rows
 * 16-byte aligned when K is 256 or 1024), d_symbols [n_steps][n_streams]
 * int32, d_mask [n_steps][n_streams] u8 or NULL; writes d_words
 * [n_streams][pitch_words] and d_sizes[n_streams].  At most 65536 streams
 * (BOA_ERR_ARG beyond).  Calls share the scratch: calls that overlap on the
 * GPU race.  The first call on a device looks up the scratch address.  Each
 * call ends by reading the scratch's error word back, so it synchronises
 * `stream` (and reports BOA_ERR_OVERFLOW / BOA_ERR_ARG found on the device). */
BOA_API int boa_rc_encode_noalloc(int n_streams, int k_symbols, int n_steps, int precision,
                                  const float* d_logits, const int32_t* d_symbols, const uint8_t* d_mask,
                                  uint32_t* d_words, int pitch_words, int32_t* d_sizes, void* stream);

/* ------------------------------------------------------------------------ */
/* BoaConstrictor model (model.py:5-134).                                   */
/* ------------------------------------------------------------------------ */
typedef struct boa_model boa_model;

/* Build the device model from fp32 weights in the flat order written by
 * portability_solved_cpp/convert_boa_weights.py:16-135 (in_proj/out_proj bias
 * slots present and zero).  d_state 16, d_conv 4, expand 2, dt_rank
 * ceil(d_model/16) as in mamba_ssm.Mamba(d_model) (model.py:47). */
BOA_API int boa_model_create(boa_model** out, int d_model, int n_layers, int vocab,
                             const float* host_flat_weights, size_t n_floats, int weight_format,
                             int device);
BOA_API int boa_model_destroy(boa_model* m);
/* Shape of a built model and the projection-weight bytes streamed per byte step. */
BOA_API int boa_model_info(const boa_model* m, int* d_model, int* n_layers, int* vocab, int* weight_format,
                           size_t* tile_bytes_per_step);
/* Bytes of device workspace (recurrent state + bookkeeping) that one
 * boa_codec_* / boa_model_logits call over n_chunks streams needs. */
BOA_API size_t boa_model_workspace_bytes(const boa_model* m, int n_chunks);
/* Positions per kernel step for encode and for logits runs of 4 or more
 * positions.  With 4 or 8 the weights and each chunk's recurrent state are
 * read once per 4 or 8 positions; 1 steps one position at a time, as decode.
 * 0 (the default) lets each launch choose 4 or 8 from its chunk and position
 * counts.  8 applies where the model's chunk tile holds whole blocks of 8
 * (d_model 256 and 512; d_model 64 with the 16-bit kinds) and the run has 8
 * or more positions, else 4.  Outputs are bit for bit the same for every
 * setting.  No reference counterpart: the reference codec (codec.py:56-79)
 * always steps one position at a time. */
BOA_API int boa_model_set_time_block(boa_model* m, int positions);
/* The positions per kernel step (1, 4 or 8) that an encode or logits launch
 * over n_chunks chunks and `positions` positions takes with the model's
 * setting; host-only, nothing is launched. */
BOA_API int boa_model_time_block(const boa_model* m, int n_chunks, int positions, int* positions_per_step);

/* Wait for `stream`, then report (and clear) the device-side errors of the
 * model's calls enqueued so far: BOA_ERR_TIMEOUT, BOA_ERR_OVERFLOW (a coded
 * stream outgrew pitch_words), BOA_ERR_ARG (an encoded symbol outside the
 * vocabulary), BOA_ERR_RANGE (an activation outside a BOA_WEIGHTS_F16X2
 * model's range; that call's outputs are not valid).  The error bits are one word per model, shared by the calls of
 * every stream; call this after the calls whose results you read.  Replaces
 * the unchecked per-launch cudaDeviceSynchronize of the reference coder
 * (gpu_range_coder.py:271,276,296,304). */
BOA_API int boa_model_status(boa_model* m, void* stream);

/* Reference-shaped single step: the streaming state of init_stream/step
 * (model.py:104-117) lives in d_workspace (zero it to start a stream).
 * d_tokens [n] int32 -> d_logits [n, vocab] fp32. */
BOA_API int boa_model_step(boa_model* m, int n, const int32_t* d_tokens, float* d_logits,
                           void* d_workspace, size_t workspace_bytes, void* stream);

/* n streams x n_steps tokens [n, n_steps] (int32), from zero state, all
 * logits out [n, n_steps, vocab] (fp32).  Diagnostic/parity entry point. */
BOA_API int boa_model_logits(boa_model* m, int n, int n_steps, const int32_t* d_tokens,
                             float* d_logits, void* d_workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* Fused codec loops (codec.py:11-86 compress_GPU, codec.py:89-151           */
/* decompress_GPU): model step -> quantiser -> range coder for every byte,   */
/* all chunks of the batch in flight, no host round trip per byte.           */
/* ------------------------------------------------------------------------ */

/* Chunk i holds d_lens[i] >= 1 bytes at d_bytes + i*in_pitch.  Byte 0 is not
 * coded (the container stores it raw, codec.py:38); bytes 1..len-1 are coded
 * with the BQ quantiser at `precision`.  Writes d_words [n, pitch_words] and
 * d_sizes[n] (words).  d_workspace must hold boa_model_workspace_bytes(). */
BOA_API int boa_codec_encode(boa_model* m, int n_chunks, const uint8_t* d_bytes, int64_t in_pitch,
                             const int32_t* d_lens, uint32_t* d_words, int pitch_words, int32_t* d_sizes,
                             int precision, void* d_workspace, size_t workspace_bytes, void* stream);

/* Inverse of boa_codec_encode: d_out [n, out_pitch] receives the chunks
 * (byte 0 from d_first_bytes). */
BOA_API int boa_codec_decode(boa_model* m, int n_chunks, const uint32_t* d_words, int pitch_words,
                             const int32_t* d_sizes, const int32_t* d_lens, const uint8_t* d_first_bytes,
                             uint8_t* d_out, int64_t out_pitch, int precision, void* d_workspace,
                             size_t workspace_bytes, void* stream);

/* Position ranges (no counterpart in the reference, whose loops always run a
 * chunk from its first byte to its last, codec.py:56-79,125-143): code only
 * positions [pos_begin, pos_end) of every chunk (clipped to d_lens), with the
 * model's recurrent state carried in d_workspace from the previous range, so
 * a long chunk can be coded in several bounded launches.  pos_begin = 1
 * starts from zero state; otherwise the workspace must hold the state the
 * call for the range ending at pos_begin left there (same chunks, same
 * workspace).  The probabilities are bit for bit those of one whole-chunk
 * call; the coder is flushed at the end of every range, so each range is its
 * own bitstream (d_words / d_sizes per range).  Byte rows cover positions
 * [pos_begin - 1, pos_end): encode reads the byte before the range from slot
 * 0 of each d_bytes row; decode takes it from d_prev_bytes[i] (the chunk's
 * first byte when pos_begin = 1), writes it to slot 0 of each d_out row and
 * the decoded position p to slot p - pos_begin + 1.  boa_codec_encode /
 * boa_codec_decode are the ranges [1, INT32_MAX). */
BOA_API int boa_codec_encode_range(boa_model* m, int n_chunks, const uint8_t* d_bytes, int64_t in_pitch,
                                   const int32_t* d_lens, int pos_begin, int pos_end, uint32_t* d_words,
                                   int pitch_words, int32_t* d_sizes, int precision, void* d_workspace,
                                   size_t workspace_bytes, void* stream);
BOA_API int boa_codec_decode_range(boa_model* m, int n_chunks, const uint32_t* d_words, int pitch_words,
                                   const int32_t* d_sizes, const int32_t* d_lens, int pos_begin, int pos_end,
                                   const uint8_t* d_prev_bytes, uint8_t* d_out, int64_t out_pitch, int precision,
                                   void* d_workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* Diagnostics (no reference counterpart).                                  */
/* ------------------------------------------------------------------------ */
/* Failure-path check (no reference counterpart): launches one thread that
 * waits on a barrier nothing arrives at, with the same bounded wait every
 * kernel of the library uses.  Returns BOA_ERR_TIMEOUT once budget_cycles SM
 * cycles have passed; the CUDA context stays usable.  Synchronous. */
BOA_API int boa_diag_timeout(int64_t budget_cycles, int device);
/* One CTA of the model kernel's projection pipeline on host data:
 * out[M][16] = W[M][K] . X[16][K]^T with W packed into the kernel's SW128 tiles
 * (weight_format as for boa_model_create).  Synchronous; allocates scratch. */
BOA_API int boa_diag_gemm(int weight_format, int M, int K, const float* h_w, const float* h_x, float* h_out,
                          int device);

#ifdef __cplusplus
}
#endif

#endif /* BOA_B200_H */
