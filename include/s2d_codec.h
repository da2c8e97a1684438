/* s2d_codec.h -- C ABI of the sm_100a codec: RVQ codes -> 44.1 kHz PCM, and
 * reference audio -> prompt codes.
 *
 * The step after the Dual-AR token loop: the codebook-major codes that
 * s2d_generate_codes returns go through the codec's RVQ lookup, its 8-layer
 * post-module transformer, two x2 upsample stages and the convolutional
 * decoder (x512) to mono PCM.  Each entry point replaces the reference
 * function named beside it (crates/fish_s2_infer/src/codec.rs) with the same
 * arguments, result layout and error cases; a Rust host would bind them as an
 * `extern "C"` block next to codec.rs.
 *
 * Layouts: codes [num_codebooks][n_frames] int32 (codebook 0 the semantic
 * code, 0..4095; codebooks 1..9 the residual codes, 0..1023); latents and
 * hidden frame-major [frames][1024] float; samples float in [-1, 1], 512 per
 * latent frame (2,048 per code frame).
 *
 * Status codes are the S2D_* codes of s2d.h.  A handle serves one call at a
 * time (its workspace and stream are shared by every call); open one handle
 * per thread to decode in parallel.
 */
#ifndef S2D_CODEC_H
#define S2D_CODEC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct S2dCodec S2dCodec;

/* Load the decode tensors of a codec GGUF (general.architecture
 * "fish-speech-codec", all F16) onto `device`: the quantizers' codebooks and
 * out_proj, the post module, the upsample stages and the decoder, with the
 * dimension checks of CodecF16Weights / CodecPostModuleF16Weights /
 * CodecUpsampleF16Weights / CodecDecoderF16Weights::from_gguf
 * (codec.rs:2335-2413, 502-540, 686-820, 1626-1679). */
int32_t s2d_codec_open(const char *gguf_path, int32_t device, S2dCodec **out);
void s2d_codec_close(S2dCodec *c);
const char *s2d_codec_last_error(const S2dCodec *c);

/* decode_waveform (codec.rs:1690): codes -> samples.  `samples` holds
 * `capacity` floats; *num_samples receives 2048 * n_frames, *latent_frames
 * 4 * n_frames.  S2D_EINVAL for num_codebooks != 10, n_frames == 0, a
 * negative or out-of-range code, or too small a buffer. */
int32_t s2d_codec_decode_waveform(S2dCodec *c, const int32_t *codes, uint32_t num_codebooks, uint32_t n_frames,
                                  float *samples, size_t capacity, size_t *num_samples, uint32_t *latent_frames);

/* The same decode on device buffers, on `stream` (a cudaStream_t; NULL: the
 * codec's own stream, which does not wait for work on other streams,
 * including the legacy default stream), without host copies or a synchronize: codes_dev
 * [num_codebooks][n_frames] int32, samples_dev 2048 * n_frames floats.  Codes
 * are checked on the device: an out-of-range code sets the codec's error flag,
 * which the next s2d_codec_sync reports as S2D_EDEVICE. */
int32_t s2d_codec_decode_waveform_device(S2dCodec *c, const int32_t *codes_dev, uint32_t num_codebooks,
                                         uint32_t n_frames, float *samples_dev, void *stream);
/* Wait for the codec's work and report its device error flag. */
int32_t s2d_codec_sync(S2dCodec *c);

/* rvq_lookup_codes (codec.rs:2536): latents [n_frames][1024]. */
int32_t s2d_codec_rvq_lookup(S2dCodec *c, const int32_t *codes, uint32_t num_codebooks, uint32_t n_frames,
                             float *latents);
/* rvq_decode_latents (codec.rs:1282): post module + upsample,
 * latents [n_frames][1024] -> hidden [4 n_frames][1024]. */
int32_t s2d_codec_decode_latents(S2dCodec *c, const float *latents, uint32_t n_frames, float *hidden);
/* forward_codec_decoder (codec.rs:1941): hidden [n_frames][hidden_dim = 1024]
 * -> samples [512 n_frames]. */
int32_t s2d_codec_decoder(S2dCodec *c, const float *hidden, uint32_t n_frames, uint32_t hidden_dim, float *samples);

/* Device bytes held by the weights and by the workspaces sized for the
 * largest decode and encode so far. */
int32_t s2d_codec_memory(const S2dCodec *c, size_t *weight_bytes, size_t *workspace_bytes);

/* ---- reference-audio encoder: 44.1 kHz mono PCM -> prompt codes ----
 * Present when the codec file holds the encoder, the quantizer's downsample
 * stages and pre module (a full s2-pro codec GGUF does); 1 if so, else 0. */
int32_t s2d_codec_has_encoder(const S2dCodec *c);

/* encode_reference_audio (codec.rs:1056): audio [n_samples] -> codes
 * [10][quantizer_frames] int32 (codebook-major, the layout decode_waveform
 * takes), quantizer_frames = ceil(n_samples / 2048) (one for no samples).
 * final_residual_l2 (optional) receives quantizer_frames floats. */
int32_t s2d_codec_encode_reference_audio(S2dCodec *c, const float *audio, size_t n_samples, int32_t *codes,
                                         size_t capacity, uint32_t *quantizer_frames, uint32_t *encoder_frames,
                                         uint32_t *padded_samples, float *final_residual_l2);
/* forward_codec_encoder_frontend (codec.rs:1087): audio -> hidden
 * [frames = padded_samples / 512][1024]. */
int32_t s2d_codec_encoder_frontend(S2dCodec *c, const float *audio, size_t n_samples, float *hidden, size_t capacity,
                                   uint32_t *frames, uint32_t *padded_samples);
/* forward_codec_quantizer_encode_stage (codec.rs:1020): hidden [n_frames][1024]
 * -> [n_frames / 4][1024]; n_frames a multiple of 4. */
int32_t s2d_codec_quantizer_encode(S2dCodec *c, const float *hidden, uint32_t n_frames, float *out);
/* rvq_encode_latents_nearest (codec.rs:2598): latents [n_frames][1024] ->
 * codes [10][n_frames], final_residual_l2 [n_frames] (optional). */
int32_t s2d_codec_vq_encode(S2dCodec *c, const float *latents, uint32_t n_frames, int32_t *codes,
                            float *final_residual_l2);

#ifdef __cplusplus
}
#endif

#endif /* S2D_CODEC_H */
