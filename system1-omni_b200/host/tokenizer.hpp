// Worker-side byte-level BPE tokenizer (tokenizer.cpp): a Hugging Face tokenizer.json of
// the Qwen family, encoded as the reference's worker does with the `tokenizers` crate.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace s1tok {

class Tokenizer {
public:
    Tokenizer();
    ~Tokenizer();
    Tokenizer(const Tokenizer&) = delete;
    Tokenizer& operator=(const Tokenizer&) = delete;
    // Reads tokenizer.json; false (with the reason) for a shape this tokenizer does not run.
    bool load(const std::string& path, std::string& err);
    // Token ids of `text` (valid UTF-8), special tokens included as written in the text.
    // Safe to call from several threads at once.
    bool encode(const std::string& text, std::vector<uint32_t>& ids, std::string& err) const;

private:
    struct Impl;
    Impl* impl_;
};

// The text without leading and trailing Unicode White_Space (Rust's str::trim).
std::string trim(const std::string& s);

}  // namespace s1tok
