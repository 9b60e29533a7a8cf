// C interface of the worker-side request processing in libs1_model.so: the tokenizer and
// the decision request contract of the reference's open_jev worker, for hosts that run the
// prefill through s1_model.h without the Rust worker.
//   s1_tokenizer_*        a Hugging Face tokenizer.json (the Qwen byte-level BPE shape, or a
//                         word-level test shape), encoded as the `tokenizers` crate (=0.22.2)
//                         does for the reference (src/models/open_jev/native/src/processing.rs:49)
//   s1_processor_*        Processor::load / prepare (processing.rs:41-91): the request JSON
//                         compiled into questions and candidate prompts (contract.rs:98-224),
//                         each prompt as chat_prefix + prompt.trim() + chat_suffix tokenized on
//                         host threads, lengths above max_length refused (no truncation)
//   s1_prepared_finish    ResponseContext::finish_with_prefix (processing.rs:93-141): the
//                         calibrated answers (contract.rs:226-289) as the response JSON
// Errors: null / nonzero, with the reason in s1_processing_error() (this thread's last).
#pragma once

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

const char* s1_processing_error(void);

void* s1_tokenizer_load(const char* tokenizer_json_path);
void s1_tokenizer_free(void* tokenizer);
// Token ids of `text` (UTF-8, len bytes), special tokens as written in the text: 0 and
// *count ids written; 1 if cap is too small (*count = the ids needed); -1 on error.
int s1_tokenizer_encode(void* tokenizer, const char* text, size_t len, uint32_t* ids, size_t cap, size_t* count);

// checkpoint: "Open-Jev-27B-v1.1" or "Open-Jev-9B" (or its model_id): the model a request
// may name and the response reports. parallel: tokenize candidates on host threads.
void* s1_processor_create(const char* tokenizer_json_path, const char* checkpoint, const char* chat_prefix,
                          const char* chat_suffix, double temperature, size_t max_length, int parallel);
void s1_processor_free(void* processor);
int s1_processor_set(void* processor, size_t max_length, int parallel);
// A prepared request (null on a refused request), freed with s1_prepared_free.
void* s1_processor_prepare(void* processor, const char* request_json, size_t len);
void s1_prepared_free(void* prepared);
size_t s1_prepared_questions(void* prepared);
size_t s1_prepared_candidates(void* prepared, size_t question);
const uint32_t* s1_prepared_ids(void* prepared, size_t question, size_t candidate, size_t* count);
const char* s1_prepared_prompt(void* prepared, size_t question, size_t candidate);
// logits: one score per candidate in prepared order (question by question). policy, shared,
// across_questions, saved_tokens: the prefix-cache metadata of the run. Returns the
// response JSON (free with s1_string_free), or null.
char* s1_prepared_finish(void* prepared, const float* logits, size_t n, const char* policy, int shared,
                         int across_questions, long long saved_tokens);
// One question's calibrated answer from a full logit row (one per key; a Noul question's
// [false, true]) at the given temperature (contract::answer), as JSON; or null.
char* s1_prepared_answer(void* prepared, size_t question, const float* logits, size_t n, double temperature);
void s1_string_free(char* s);

#ifdef __cplusplus
}
#endif
