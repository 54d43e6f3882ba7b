"""CPU: the library's tokenizer (vkllm_models_llama2_tokenize, host code) against a restatement of
the reference's algorithm (oracle/tokenizer_ref.py, src/models/vkllm_models_llama2.c:604-816), on
hand-made and seeded random vocabularies: UTF-8 splitting, "▁" for spaces, highest-score merges with
leftmost ties, first-entry lookups for duplicate texts, dropped pieces, and the bos / eos flags.
The reference has no tokenizer test or golden ids, so this parity is pinned to the algorithm only."""
import ctypes as C
import ctypes.util

import numpy as np
import pytest
import tokenizer_ref


class Tok(C.Structure):
    _fields_ = [("text", C.c_char_p), ("score", C.c_float), ("type", C.c_int32)]


class TokArray(C.Structure):
    _fields_ = [("alloc_n", C.c_size_t), ("used_n", C.c_size_t), ("data", C.POINTER(Tok))]


_libc = C.CDLL(ctypes.util.find_library("c"))
_libc.free.argtypes = [C.c_void_p]


def run(vk, vocab, sentence, add_bos=True, add_eos=True):
    toks = (Tok * len(vocab))(*[Tok(t, s, 1) for t, s in vocab])
    arr = TokArray(len(vocab), len(vocab), toks)
    m = vk.Llama2()
    m.meta.tokens = C.cast(C.pointer(arr), C.c_void_p)
    m.meta.add_bos_token, m.meta.add_eos_token = add_bos, add_eos
    m.meta.bos_token_id, m.meta.eos_token_id = 1, 2
    out = C.POINTER(vk.TokenIdArray)()
    vk.check(vk.lib().vkllm_models_llama2_tokenize(C.byref(m), sentence, C.byref(out)), "tokenize")
    ids = [out.contents.data[i] for i in range(out.contents.used_n)]
    _libc.free(C.cast(out.contents.data, C.c_void_p))
    _libc.free(C.cast(out, C.c_void_p))
    return ids


S = "▁"
HAND = [(b"<unk>", 0.0), (b"<s>", 0.0), (b"</s>", 0.0)] + [(t.encode(), s) for t, s in [
    (S, -1.0), ("a", -2.0), ("b", -2.0), ("c", -2.0), ("é", -2.0), ("日", -2.0), ("本", -2.0),
    ("ab", -1.5), ("bc", -1.5), ("abc", -1.0), (S + "a", -1.2), (S + "ab", -0.8), (S + "abc", -0.5),
    ("日本", -0.7), (S + "日本", -0.6), ("éa", -1.5), ("ca", -1.5),
    ("ab", 5.0),  # a later duplicate: the first entry (id and score) is the one that counts
]]


@pytest.mark.parametrize("sentence", ["abc", "abc abc", " a", "a  b", "cab", "éab", "日本 日本", "ab c é", "zzz",
                                      "a", "", "éé é"])
def test_hand_vocabulary(vk, sentence):
    b = sentence.encode()
    assert run(vk, HAND, b) == tokenizer_ref.tokenize(HAND, b), sentence


@pytest.mark.parametrize("bos,eos", [(False, False), (True, False), (False, True)])
def test_bos_eos_flags(vk, bos, eos):
    b = "abc ab".encode()
    assert run(vk, HAND, b, bos, eos) == tokenizer_ref.tokenize(HAND, b, bos, eos)


def random_vocab(rng, n):
    alphabet = ["a", "b", "c", "d", S, "é", "ß", "日", "😀"]
    vocab = [(b"<unk>", 0.0), (b"<s>", 0.0), (b"</s>", 0.0)] + [(ch.encode(), -5.0) for ch in alphabet]
    for _ in range(n):
        k = int(rng.integers(2, 5))
        text = "".join(alphabet[int(i)] for i in rng.integers(0, len(alphabet), size=k))
        score = float(np.float32(rng.integers(-8, 8) / 2.0))  # coarse scores: many ties
        vocab.append((text.encode(), score))
    return vocab, alphabet


@pytest.mark.parametrize("seed", range(6))
def test_random_vocabularies(vk, seed):
    rng = np.random.default_rng(seed)
    vocab, alphabet = random_vocab(rng, 400)
    chars = [a for a in alphabet if a != S] + [" "]
    for _ in range(40):
        k = int(rng.integers(1, 24))
        b = "".join(chars[int(i)] for i in rng.integers(0, len(chars), size=k)).encode()
        assert run(vk, vocab, b) == tokenizer_ref.tokenize(vocab, b), (seed, b)
