"""Fixtures of the worker-side processing tests (tests/test_processing_cpu.py).

    python tests/golden/make_processing_fixtures.py

Writes into tests/golden/:
  tokenizer_bpe.json       a byte-level BPE tokenizer of the Qwen shape (NFC normalizer,
                           Split on the Qwen2 pattern + ByteLevel, BPE, special tokens
                           <|endoftext|> <|im_start|> <|im_end|>, added <think> </think>, and
                           one normalized added token), trained here with Hugging Face
                           `tokenizers` on a seeded synthetic multilingual corpus: the real
                           Qwen vocabulary is not in this tree, so the tokenizer the
                           reference's worker runs (the `tokenizers` crate, =0.22.2) is pinned
                           through its Python binding of the same version on this vocabulary;
  tokenization_cases.json  texts (the reference's unicode test samples, the contract prompts in
                           the Qwen chat template, seeded mixed-script strings) and their ids
                           from that binding;
  tokenizer_wordlevel.json the word-level tokenizer the reference's processing tests build
                           (tests/open_jev/processing.rs:8-66: WordLevel, WhitespaceSplit, a
                           [BOS] template);
  contract_cases.json      the reference's contract vectors (tests/open_jev/data/contract.json,
                           generated there with Open-Jev's jev.api / jev.metrics): requests,
                           prompts, logits, temperature and calibrated answers, read from the
                           reference tree when it is present.
"""
import json
import os
import random

import tokenizers
from tokenizers import AddedToken, Regex, Tokenizer, decoders, models, normalizers, pre_tokenizers, processors, trainers

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("S1_REFERENCE_ROOT", "/root/reference")
QWEN_PATTERN = (r"(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*|"
                r"\s*[\r\n]+|\s+(?!\S)|\s+")
CHAT_PREFIX = "<|im_start|>user\n"
CHAT_SUFFIX = "<|im_end|>\n<|im_start|>assistant\n<think>\n\n</think>\n\n"

WORDS = ["Context", "Question", "answer", "proposed", "correct", "customer", "charged", "twice", "order",
         "service", "working", "normally", "unauthorized", "access", "billing", "security", "technical",
         "urgent", "routine", "critical", "café", "naïve", "Zürich", "São", "Paulo", "déjà", "vu"]
SCRIPTS = ["中文推理选项甲乙丙丁", "日本語のテキスト", "한글자모음", "العربية", "עברית", "Ελληνικά", "Русский",
           "हिन्दी", "ไทย", "𐀀𝕏𝒜"]
SPICE = ["'s", "'S", "'ll", "'LL", "'Re", "'ve", "'m", "'d", "'t", "'\u017f", "\r\n", "\n\n", "\t", "  ", "   ",
         "\u00a0", "\u3000", "\u2028", "\u200b", "e\u0301", "a\u0323\u0308", "\u1100\u1161\u11a8",
         "\uff11\uff12\uff13", "\U0001F469\U0001F3FD\u200d\U0001F4BB", "\U0001F468\u200d\U0001F469\u200d\U0001F467",
         "\ufffd", "...", "?!", "\u2014", "(x)", "[1,2]", "$5.00", "100%", "\x00", "\x7f"]


def synthetic(rng, n):
    parts = []
    for _ in range(n):
        r = rng.random()
        if r < 0.45:
            parts.append(rng.choice(WORDS))
        elif r < 0.6:
            s = rng.choice(SCRIPTS)
            a = rng.randrange(len(s))
            parts.append(s[a:a + rng.randint(1, 4)])
        elif r < 0.75:
            parts.append(str(rng.randint(0, 99999)))
        else:
            parts.append(rng.choice(SPICE))
        parts.append(rng.choice([" ", " ", " ", "", "\n", ", ", ". "]))
    return "".join(parts)


def bpe_tokenizer():
    rng = random.Random(20261202)
    corpus = [synthetic(rng, rng.randint(5, 40)) for _ in range(4000)]
    tok = Tokenizer(models.BPE(unk_token=None, byte_fallback=False))
    tok.normalizer = normalizers.NFC()
    tok.pre_tokenizer = pre_tokenizers.Sequence([
        pre_tokenizers.Split(Regex(QWEN_PATTERN), behavior="isolated", invert=False),
        pre_tokenizers.ByteLevel(add_prefix_space=False, trim_offsets=False, use_regex=False)])
    tok.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(vocab_size=3000, initial_alphabet=pre_tokenizers.ByteLevel.alphabet(),
                                  special_tokens=["<|endoftext|>", "<|im_start|>", "<|im_end|>"], show_progress=False)
    tok.train_from_iterator(corpus, trainer)
    tok.add_tokens([AddedToken("<think>", normalized=False, special=False),
                    AddedToken("</think>", normalized=False, special=False),
                    AddedToken("Zürich-Nord", normalized=True, special=False)])
    return tok


def wordlevel_tokenizer():
    words = ["[UNK]", "[BOS]", "Context:", "x", "Question:", "Route", "Proposed", "answer:", "billing", "security",
             "technical", "Is", "this", "proposed", "answer", "correct?", "Answer", "Yes", "or", "No.", "Verify",
             "the", "to", "question", "yes?"]
    tok = Tokenizer(models.WordLevel({w: i for i, w in enumerate(words)}, unk_token="[UNK]"))
    tok.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    tok.post_processor = processors.TemplateProcessing(single="[BOS] $A", special_tokens=[("[BOS]", 1)])
    return tok


def main():
    bpe = bpe_tokenizer()
    bpe.save(os.path.join(HERE, "tokenizer_bpe.json"))
    wl = wordlevel_tokenizer()
    wl.save(os.path.join(HERE, "tokenizer_wordlevel.json"))
    texts = []
    samples = ["", "  \u4e2d\u6587\u63a8\u7406\uff1a\u9009\u9879\u7532\u3001\u4e59\u3002  ", "caf\u00e9 cafe\u0301",
               "\U0001F469\U0001F3FD\u200d\U0001F4BB \U0001F468\u200d\U0001F469\u200d\U0001F467\u200d\U0001F466",
               "\u0627\u0644\u0639\u0631\u0628\u064a\u0629 \u05e2\u05d1\u05e8\u05d9\u05ea",
               "\u65e5\u672c\u8a9e \ud55c\uae00", "line1\r\n\tline2\x00end",
               "<|im_start|>assistant\n<|im_end|><|endoftext|>", "\U00010000 \U0001D54F \U0001D49C \ufffd",
               "\u200bx\u00a0y\u3000"]
    for i in range(33):  # the reference's batch-vs-serial samples (tests/open_jev/tokenization.rs)
        prompt = f"{samples[i % len(samples)]} {'x ' * i}"
        texts.append(CHAT_PREFIX + prompt.strip() + CHAT_SUFFIX)
    contract = None
    src = os.path.join(REF, "tests", "open_jev", "data", "contract.json")
    if os.path.exists(src):
        with open(src) as f:
            contract = json.load(f)
        with open(os.path.join(HERE, "contract_cases.json"), "w") as f:
            json.dump(contract, f, ensure_ascii=False, indent=1)
    else:
        with open(os.path.join(HERE, "contract_cases.json")) as f:
            contract = json.load(f)
    for case in contract:
        for prompts in case["prompts"]:
            texts.extend(CHAT_PREFIX + p.strip() + CHAT_SUFFIX for p in prompts)
    rng = random.Random(7)
    texts.extend(synthetic(rng, rng.randint(1, 60)) for _ in range(300))
    texts.extend(["Z\u00fcrich-Nord", "Zu\u0308rich-Nord and Z\u00fcrich-Nord", "don'T 'Ve '\u017f",
                  "a\r\n\r\n  \n b", "   ", "x  y", " \t\n", "\uff11\uff12\uff13\uff14", "'s's'S",
                  "\uac01\u1100\u1161\u11a8 \u1112\u1161\u11ab"])
    cases = [{"text": t, "ids": bpe.encode(t, add_special_tokens=True).ids} for t in texts]
    with open(os.path.join(HERE, "tokenization_cases.json"), "w") as f:
        json.dump({"tokenizers": tokenizers.__version__, "chat_prefix": CHAT_PREFIX, "chat_suffix": CHAT_SUFFIX,
                   "cases": cases}, f, ensure_ascii=False)
    print(len(cases), "tokenization cases;", len(contract), "contract cases; tokenizers", tokenizers.__version__)


if __name__ == "__main__":
    main()
