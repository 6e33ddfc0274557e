/* SPDX-License-Identifier: MIT
 *
 * qh_gguf.h -- GGUF v3 files for the device model: the loader the
 * reference's slm_model_load path uses (gguf_open, slm/gguf.c:172-261;
 * slm_load_config, slm/qwen.c:59-159; tensors bound by name as
 * slm_load_weights does, slm/qwen.c:174-252) and a writer for synthetic
 * models, so a qh_blob round-trips through the same file format the
 * reference reads.
 *
 * Only the "qwen35" architecture (the hybrid Gated DeltaNet + attention
 * model) is accepted; tensor types F32, Q8_0, Q4_K, Q5_K, Q6_K.
 */
#ifndef QH_GGUF_H
#define QH_GGUF_H

#include <stdint.h>

#include "qh_slm.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Reads `path`: the config from the qwen35.* keys (defaults as
 * slm_load_config: head_count_kv = head_count, key_length = hidden /
 * heads, rope.freq_base 10000, layer_norm_rms_epsilon 1e-5, ssm group 16,
 * state 128, conv 4, full_attention_interval 4; vocab = the length of
 * tokenizer.ggml.tokens), max_pos = min(context_length (default 2048),
 * max_pos_cap, or 4096 when max_pos_cap <= 0), and every tensor into a new
 * blob (bytes copied). QH_ERR_INVALID for a malformed file,
 * QH_ERR_UNSUPPORTED for another architecture or tensor type. */
int qh_gguf_load(const char *path, int32_t max_pos_cap, qh_slm_config *cfg, qh_blob **out);

/* Special token ids of a GGUF file, as slm_model_load binds them: bos/eos
 * from tokenizer.ggml.bos_token_id / eos_token_id (default 0; slm/qwen.c:
 * 150-155), eot = the id of "<|im_end|>" (-1 if absent) and the stop set =
 * the ids of "<|endoftext|>", "<|im_end|>", "<|fim_pad|>", "<|repo_name|>",
 * "<|file_sep|>" present in tokenizer.ggml.tokens (slm/model.c:1153-1178). */
typedef struct qh_special_tokens {
    int32_t bos_id, eos_id, eot_id;
    int32_t n_stop;
    int32_t stop_ids[8];
} qh_special_tokens;
int qh_gguf_special_tokens(const char *path, qh_special_tokens *out);

/* Writes cfg and every tensor of blob as a GGUF v3 file with
 * general.architecture = "qwen35", the qwen35.* keys above,
 * context_length = cfg->max_pos, a placeholder tokenizer.ggml.tokens
 * array of cfg->vocab entries, and 32-byte aligned tensor data. */
int qh_gguf_write(const char *path, const qh_slm_config *cfg, const qh_blob *blob);

#ifdef __cplusplus
}
#endif

#endif /* QH_GGUF_H */
