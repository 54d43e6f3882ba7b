"""TEST INFRASTRUCTURE ONLY: a restatement of the reference tokenizer's algorithm
(src/models/vkllm_models_llama2.c:604-816, `vkllm_models_llama2_tokenize`), used by tests/ as the
checker of the library's tokenizer. The product never imports it.

Steps, as the reference takes them:
* :666-684  "▁" (U+2581) in front, and "▁" for every space byte;
* :702-740  split into UTF-8 characters by lead byte (0xC0/0xE0/0xF0 classes; any other byte,
  continuation bytes included, is a piece of its own);
* :742-771  while more than one piece: among adjacent pairs whose concatenation is a vocabulary
  text, merge the one with the highest score of its first vocabulary entry (`find_token_by_text`,
  :604-614, is a first-match scan); ties go to the leftmost pair (strict >, :637);
* :773-789  output [bos if add_bos] + the first vocabulary id of every piece that has one (pieces
  without one are dropped) + [eos if add_eos]; an empty sentence gives an empty list (:658-662).

One deliberate difference: a multi-byte lead byte in the last 1-3 bytes of the text makes the
reference copy bytes past the end of its buffer (:717); here the piece stops at the end of the text.
"""

SPACE = "▁".encode()


def first_ids(vocab):
    """text (bytes) -> first index with that text, as the reference's linear scan finds it."""
    out = {}
    for i, (text, _score) in enumerate(vocab):
        out.setdefault(text, i)
    return out


def split_utf8(b):
    pieces, i = [], 0
    while i < len(b):
        c = b[i]
        n = 1
        if c >= 0x80:
            if c & 0xE0 == 0xC0:
                n = 2
            elif c & 0xF0 == 0xE0:
                n = 3
            elif c & 0xF8 == 0xF0:
                n = 4
        pieces.append(b[i:i + n])
        i += n
    return pieces


def tokenize(vocab, sentence, add_bos=True, add_eos=True, bos=1, eos=2):
    """vocab: list of (text bytes, score float); sentence: bytes. Returns the token ids."""
    if len(sentence) == 0:
        return []
    ids = first_ids(vocab)
    text = SPACE + b"".join(SPACE if ch == 0x20 else bytes([ch]) for ch in sentence)
    pieces = split_utf8(text)
    while len(pieces) > 1:
        best, at = float("-inf"), -1
        for i in range(len(pieces) - 1):
            j = ids.get(pieces[i] + pieces[i + 1])
            if j is not None and vocab[j][1] > best:
                best, at = vocab[j][1], i
        if at < 0:
            break
        pieces[at:at + 2] = [pieces[at] + pieces[at + 1]]
    out = [bos] if add_bos else []
    out += [ids[p] for p in pieces if p in ids]
    if add_eos:
        out.append(eos)
    return out
