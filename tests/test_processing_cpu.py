"""Worker-side request processing (include/s1_processing.h), no GPU needed.

* The byte-level BPE tokenizer against Hugging Face `tokenizers` 0.22.2 (the version the
  reference's worker pins, Cargo.toml:14) on a tokenizer.json of the Qwen shape trained on
  a synthetic corpus (the Qwen vocabulary is not in this tree): every id of 359 texts (the
  reference's unicode samples in the chat template, the contract prompts, mixed scripts,
  combining marks, Hangul jamo, whitespace runs, contractions, special and added tokens).
* The request contract against the reference's own vectors (tests/open_jev/contract.rs and
  data/contract.json): prompts, and the calibrated answers within 1e-12; its rejections.
* Processor::prepare / finish against the reference's processing tests
  (tests/open_jev/processing.rs): exact candidate ids with the word-level test tokenizer,
  chat prefix / suffix, serial == parallel, answers in request order, usage and metadata,
  the over-long candidate error, prefix-cache metadata, the loaded checkpoint's names.
"""
import json
import math
import os

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
G = os.path.join(HERE, "golden")
BPE = os.path.join(G, "tokenizer_bpe.json")
WL = os.path.join(G, "tokenizer_wordlevel.json")
REQUEST = (b'{"state":"x","questions":{\n    "z":{"type":"choice","instructions":"Route","criteria":'
           b'{"technical":null,"billing":null}},\n    "a":{"type":"noul","instructions":"Verify"}}}')


def _processor(max_length=4096, **kw):
    from s1omni import Processor
    return Processor(WL, "Open-Jev-27B-v1.1", kw.pop("prefix", ""), kw.pop("suffix", ""), 0.5, max_length, **kw)


def test_bpe_tokenizer_matches_the_tokenizers_library():
    from s1omni import Tokenizer
    data = json.load(open(os.path.join(G, "tokenization_cases.json")))
    assert data["tokenizers"] == "0.22.2"
    tok = Tokenizer(BPE)
    bad = [c["text"] for c in data["cases"] if tok.encode(c["text"]) != c["ids"]]
    assert not bad, bad[:3]


def test_tokenizer_refuses_shapes_it_does_not_run(tmp_path):
    from s1omni import Tokenizer
    j = json.load(open(BPE))
    j["pre_tokenizer"]["pretokenizers"][0]["pattern"]["Regex"] = r"\s+"
    p = tmp_path / "t.json"
    p.write_text(json.dumps(j))
    with pytest.raises(RuntimeError, match="pre-tokenizer"):
        Tokenizer(p)
    with pytest.raises(RuntimeError):
        Tokenizer(tmp_path / "missing.json")


def _close(a, b):
    if isinstance(b, float) or isinstance(a, float):
        assert abs(a - b) < 1e-12, (a, b)
    elif isinstance(b, dict):
        assert len(a) == len(b)
        for k in b:
            _close(a[k], b[k])
    else:
        assert a == b


def test_contract_prompts_and_answers_match_the_reference_vectors():
    from s1omni import Processor
    for case in json.load(open(os.path.join(G, "contract_cases.json"))):
        p = Processor(BPE, "Open-Jev-27B-v1.1", "", "", case["temperature"], 1 << 20)
        r = p.prepare(case["request"])
        assert r.prompts == case["prompts"]
        answers = {}
        ids = list(case["request"]["questions"].keys())
        for q, row in enumerate(case["logits"]):
            answers[ids[q]] = r.answer(q, row, case["temperature"])
        _close({"answers": answers}, case["response"])


@pytest.mark.parametrize("raw", [
    b'{"state":"x","state":"y","questions":{}}',
    b'{"state":NaN,"questions":{}}',
    b'{"state":12,"questions":{"q":{"type":"noul","instructions":"x"}}}',
    b'{"state":"x","questions":{}}',
    b'{"model":"other","state":"x","questions":{"q":{"type":"noul","instructions":"x"}}}',
    b'{"state":"x","questions":{"q":{"type":"generation","instructions":"x"}}}',
    b'{"state":"x","questions":{"q":{"type":"choice","instructions":"x","criteria":{}}}}',
    b'{"state":"x","questions":{"q":{"type":"choice","instructions":"x","criteria":{"a":4}}}}',
    b'{"state":"x","questions":{"q":{"type":"score","instructions":"x","criteria":["one"]}}}',
    b'{"state":"x","questions":{"q":{"type":"noul","instructions":"x","criteria":{"true":"yes"}}}}'])
def test_contract_rejects_malformed_and_unsupported_requests(raw):
    with pytest.raises(ValueError):
        _processor().prepare(raw)


def test_answer_rejects_bad_temperatures_and_logits():
    r = _processor().prepare(b'{"state":"x","questions":{"q":{"type":"noul","instructions":"x"}}}')
    for t in (0.0, -1.0, math.nan, math.inf):
        with pytest.raises(RuntimeError):
            r.answer(0, [0.0, 1.0], t)
    with pytest.raises(RuntimeError):
        r.answer(0, [1.0], 1.0)
    with pytest.raises(RuntimeError):
        r.answer(0, [0.0, math.nan], 1.0)


def test_prepared_candidates_have_exact_ids_and_finished_responses_keep_mapping():
    r = _processor().prepare(REQUEST)
    assert r.ids == [[[1, 2, 3, 4, 5, 6, 7, 10, 11, 12, 13, 14, 15, 16, 17, 18, 19],
                      [1, 2, 3, 4, 5, 6, 7, 8, 11, 12, 13, 14, 15, 16, 17, 18, 19]],
                     [[1, 2, 3, 4, 20, 11, 21, 14, 22, 12, 23, 24, 16, 17, 18, 19]]]
    body = r.finish([[3.0, 3.0], [0.0]])
    assert body["answers"] == {
        "z": {"type": "choice", "choice": "technical", "probabilities": {"technical": 0.5, "billing": 0.5},
              "confidence": 0.0},
        "a": {"type": "noul", "noul": 0.5}}
    assert list(body["answers"].keys()) == ["z", "a"]
    assert body["usage"] == {"input_tokens": 50, "output_tokens": 0}
    m = body["metadata"]
    assert m["candidate_sequences"] == 3 and m["temperature"] == 0.5 and m["max_length"] == 4096
    assert m["method"] == "native_merged_lora_decision_head"
    assert m["base_revision"] == "1d4bf0f2ff6012fd82039f2fa52739d0dd7c60c0"
    assert m["prefix_cache"] == {"policy": "default", "enabled": False, "scope": "none", "saved_tokens": 0}
    assert m["inference_seconds"] >= 0.0
    assert body["model"] == "Qwen/Qwen3.8-27B"


def test_serial_preparation_preserves_tokens_and_question_mapping():
    p = _processor()
    expected = p.prepare(REQUEST).ids
    p.set(4096, parallel=False)
    assert p.prepare(REQUEST).ids == expected


def test_preparation_applies_the_saved_chat_prefix_and_suffix():
    r = _processor(prefix="billing ", suffix=" security").prepare(REQUEST)
    # BOS precedes the saved prefix; the suffix follows the question prompt
    assert r.ids[0][0] == [1, 8, 2, 3, 4, 5, 6, 7, 10, 11, 12, 13, 14, 15, 16, 17, 18, 19, 9]


def test_prefix_metadata_uses_executed_savings_without_changing_answers_or_usage():
    request = {"state": "x " * 768, "questions": {"q": {"type": "choice", "instructions": "Route",
                                                         "criteria": {"billing": None, "security": None,
                                                                      "technical": None}}}}
    rows = [[1.0, 2.0, 3.0]]
    baseline = _processor().prepare(request).finish(rows)
    for saved in (1024, 512, 0):
        got = _processor().prepare(request).finish(rows, shared=saved > 0, saved_tokens=saved)
        assert got["answers"] == baseline["answers"] and got["usage"] == baseline["usage"]
        assert got["metadata"]["candidate_sequences"] == 3
        assert got["metadata"]["prefix_cache"] == {"policy": "default", "enabled": saved > 0,
                                                   "scope": "within_question" if saved > 0 else "none",
                                                   "saved_tokens": saved}


def test_responses_name_the_loaded_checkpoint():
    from s1omni import Processor
    body = Processor(WL, "Open-Jev-9B", "", "", 0.5, 4096).prepare(REQUEST).finish([[3.0, 3.0], [0.0]])
    assert body["model"] == "Qwen/Qwen3.5-9B"
    assert body["metadata"]["base_revision"] == "c202236235762e1c871ad0ccb60c8ee5ba337b9a"


def test_preparation_rejects_later_oversize_candidates_before_execution():
    p = _processor(17)
    p.prepare(REQUEST)
    raw = json.loads(REQUEST)
    raw["questions"]["a"]["instructions"] = "x " * 18
    with pytest.raises(ValueError) as e:
        p.prepare(json.dumps(raw).encode())
    assert str(e.value).startswith("question a: ")
    assert str(e.value).endswith("exceeds max_length=17; no silent truncation")
    with pytest.raises(ValueError) as e:
        p.prepare(b'{"state":"x","questions":{}}')
    assert str(e.value) == "questions must be nonempty and within the server question limit"


def test_parallel_tokenization_keeps_candidate_order_across_chunks_and_questions():
    from s1omni import Processor, Tokenizer
    data = json.load(open(os.path.join(G, "tokenization_cases.json")))
    tok = Tokenizer(BPE)
    prompts = {f"o{i}": None for i in range(40)}
    request = {"state": "x", "questions": {"q1": {"type": "choice", "instructions": "pick", "criteria": prompts},
                                           "q2": {"type": "noul", "instructions": "ok?"}}}
    pre, suf = data["chat_prefix"], data["chat_suffix"]
    for parallel in (True, False):
        r = Processor(BPE, "Open-Jev-27B-v1.1", pre, suf, 1.0, 4096, parallel=parallel).prepare(request)
        want = [[tok.encode(pre + p.strip() + suf) for p in q] for q in r.prompts]
        assert r.ids == want
