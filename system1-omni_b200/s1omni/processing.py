"""Worker-side request processing (libs1_model.so, include/s1_processing.h): the tokenizer
and the decision request contract of the reference's open_jev worker.

    tok = Tokenizer("tokenizer.json"); tok.encode("text") -> [ids]
    p = Processor("tokenizer.json", "Open-Jev-27B-v1.1", chat_prefix, chat_suffix, temperature, max_length)
    r = p.prepare(request_bytes)        # r.ids[question][candidate], r.prompts[question][candidate]
    body = r.finish(scores)             # the response JSON (dict); scores: one per candidate
"""
import ctypes
import json

from .model import _get

P, Z = ctypes.c_void_p, ctypes.c_size_t


def _lib():
    lib = _get()
    if not getattr(lib, "_processing_bound", False):
        lib.s1_processing_error.restype = ctypes.c_char_p
        lib.s1_tokenizer_load.restype = P
        lib.s1_tokenizer_load.argtypes = [ctypes.c_char_p]
        lib.s1_tokenizer_free.argtypes = [P]
        lib.s1_tokenizer_encode.argtypes = [P, ctypes.c_char_p, Z, P, Z, ctypes.POINTER(Z)]
        lib.s1_processor_create.restype = P
        lib.s1_processor_create.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p,
                                            ctypes.c_double, Z, ctypes.c_int]
        lib.s1_processor_free.argtypes = [P]
        lib.s1_processor_set.argtypes = [P, Z, ctypes.c_int]
        lib.s1_processor_prepare.restype = P
        lib.s1_processor_prepare.argtypes = [P, ctypes.c_char_p, Z]
        lib.s1_prepared_free.argtypes = [P]
        lib.s1_prepared_questions.restype = Z
        lib.s1_prepared_questions.argtypes = [P]
        lib.s1_prepared_candidates.restype = Z
        lib.s1_prepared_candidates.argtypes = [P, Z]
        lib.s1_prepared_ids.restype = ctypes.POINTER(ctypes.c_uint32)
        lib.s1_prepared_ids.argtypes = [P, Z, Z, ctypes.POINTER(Z)]
        lib.s1_prepared_prompt.restype = ctypes.c_char_p
        lib.s1_prepared_prompt.argtypes = [P, Z, Z]
        lib.s1_prepared_finish.restype = P
        lib.s1_prepared_finish.argtypes = [P, P, Z, ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_longlong]
        lib.s1_prepared_answer.restype = P
        lib.s1_prepared_answer.argtypes = [P, Z, P, Z, ctypes.c_double]
        lib.s1_string_free.argtypes = [P]
        lib._processing_bound = True
    return lib


def _error(what):
    return RuntimeError(f"{what}: {_lib().s1_processing_error().decode()}")


def _take_string(ptr):
    lib = _lib()
    if not ptr:
        return None
    try:
        return ctypes.string_at(ptr).decode()
    finally:
        lib.s1_string_free(ptr)


class Tokenizer:
    def __init__(self, path):
        self._lib = _lib()
        self._h = self._lib.s1_tokenizer_load(str(path).encode())
        if not self._h:
            raise _error("tokenizer")

    def encode(self, text):
        raw = text.encode() if isinstance(text, str) else bytes(text)
        n = Z()
        cap = max(64, 2 * len(raw) + 16)
        while True:
            buf = (ctypes.c_uint32 * cap)()
            rc = self._lib.s1_tokenizer_encode(self._h, raw, len(raw), buf, cap, ctypes.byref(n))
            if rc == 1:
                cap = n.value
                continue
            if rc != 0:
                raise _error("encode")
            return list(buf[:n.value])

    def close(self):
        if getattr(self, "_h", None):
            self._lib.s1_tokenizer_free(self._h)
            self._h = None

    def __del__(self):
        self.close()


class Prepared:
    def __init__(self, lib, h):
        self._lib, self._h = lib, h
        nq = lib.s1_prepared_questions(h)
        self.ids, self.prompts = [], []
        for q in range(nq):
            ids, prompts = [], []
            for c in range(lib.s1_prepared_candidates(h, q)):
                n = Z()
                p = lib.s1_prepared_ids(h, q, c, ctypes.byref(n))
                ids.append([p[i] for i in range(n.value)])
                prompts.append(lib.s1_prepared_prompt(h, q, c).decode())
            self.ids.append(ids)
            self.prompts.append(prompts)

    def finish(self, scores, policy="default", shared=False, across_questions=False, saved_tokens=0):
        """Response JSON (dict) from one score per candidate, in prepared order."""
        flat = [float(x) for row in scores for x in (row if hasattr(row, "__len__") else [row])]
        arr = (ctypes.c_float * len(flat))(*flat)
        out = _take_string(self._lib.s1_prepared_finish(self._h, arr, len(flat), policy.encode(), int(shared),
                                                        int(across_questions), int(saved_tokens)))
        if out is None:
            raise _error("finish")
        return json.loads(out)

    def answer(self, question, logits, temperature):
        arr = (ctypes.c_float * len(logits))(*[float(x) for x in logits])
        out = _take_string(self._lib.s1_prepared_answer(self._h, question, arr, len(logits), float(temperature)))
        if out is None:
            raise _error("answer")
        return json.loads(out)

    def close(self):
        if getattr(self, "_h", None):
            self._lib.s1_prepared_free(self._h)
            self._h = None

    def __del__(self):
        self.close()


class Processor:
    def __init__(self, tokenizer_json, checkpoint="Open-Jev-27B-v1.1", chat_prefix="", chat_suffix="",
                 temperature=1.0, max_length=4096, parallel=True):
        self._lib = _lib()
        self._h = self._lib.s1_processor_create(str(tokenizer_json).encode(), checkpoint.encode(),
                                                chat_prefix.encode(), chat_suffix.encode(), float(temperature),
                                                int(max_length), int(parallel))
        if not self._h:
            raise _error("processor")

    def set(self, max_length, parallel=True):
        self._lib.s1_processor_set(self._h, int(max_length), int(parallel))

    def prepare(self, request):
        raw = request if isinstance(request, (bytes, bytearray)) else json.dumps(request).encode()
        h = self._lib.s1_processor_prepare(self._h, raw, len(raw))
        if not h:
            raise ValueError(self._lib.s1_processing_error().decode())
        return Prepared(self._lib, h)

    def close(self):
        if getattr(self, "_h", None):
            self._lib.s1_processor_free(self._h)
            self._h = None

    def __del__(self):
        self.close()
