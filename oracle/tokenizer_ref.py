"""CPU restatement of tokenizer.lisp -- test infrastructure only (the
checker of libembedcuda.so's tokenizer; never part of the product path).

Follows tokenizer.lisp function by function:
  whitespace-p / punctuation-p (:30-43), split-spaces (:60-67),
  bytes_to_unicode (:74-93), make-tokenizer (:119-197),
  tk-encode (:201-244), tk-decode (:246-252), pretokenize-wordpiece
  (:258-270), pretokenize-gpt2 (:280-327), pretokenize-llama3 (:329-377),
  pretokenize-metaspace (:386-391), wordpiece-tokenize-word (:395-415),
  bpe-merge (:417-434), unigram-viterbi (:436-458), json-specials
  (:465-498), pretok-mode (:500-513), make-tokenizer-from-json (:515-552).

SBCL's character predicates are taken as: alpha-char-p = Unicode general
category L*, digit-char-p = Nd, sb-unicode:lowercase = the full per-character
lowercase mapping with final sigma (a capital sigma after a letter and not
before one lowers to the final form).  These come from Python's unicodedata
here; SBCL's own Unicode tables are not available, so parity on non-ASCII
letters, digits and case is unpinned.
"""
from __future__ import annotations

import json
import unicodedata

WS = (" ", "\t", "\n", "\r", "\x0c")


def whitespace_p(c):
    return c in WS


def punctuation_p(c):
    cp = ord(c)
    return (33 <= cp <= 47 or 58 <= cp <= 64 or 91 <= cp <= 96 or 123 <= cp <= 126
            or 0x2000 <= cp <= 0x206F or 0x3000 <= cp <= 0x303F)


def alpha_p(c):
    return unicodedata.category(c).startswith("L")


def digit_p(c):
    return unicodedata.category(c) == "Nd"


def lowercase(s):
    out = []
    for i, c in enumerate(s):
        if c == "Σ":
            prev_letter = i > 0 and alpha_p(s[i - 1])
            next_letter = i + 1 < len(s) and alpha_p(s[i + 1])
            out.append("ς" if prev_letter and not next_letter else "σ")
        else:
            out.append(c.lower())
    return "".join(out)


def split_spaces(s):
    out, start = [], 0
    for i, c in enumerate(s):
        if whitespace_p(c):
            if i > start:
                out.append(s[start:i])
            start = i + 1
    if len(s) > start:
        out.append(s[start:])
    return out


def _byte_map():
    table, n = [], 0
    for b in range(256):
        if (33 <= b <= 126 and b != 92) or 161 <= b <= 172 or 174 <= b <= 255:
            table.append(chr(b))
        else:
            table.append(chr(256 + n))
            n += 1
    return table


BYTE2CHR = _byte_map()


def bytes_to_unicode_str(b: bytes):
    return "".join(BYTE2CHR[x] for x in b)


def pretokenize_wordpiece(s):
    out = []
    for w in split_spaces(s):
        start = 0
        for i, c in enumerate(w):
            if punctuation_p(c):
                if i > start:
                    out.append(w[start:i])
                out.append(c)
                start = i + 1
        if start < len(w):
            out.append(w[start:])
    return out


CONTRACTIONS = ("s", "t", "m", "d", "re", "ve", "ll")


def _scan(s, llama3):
    out, i, n = [], 0, len(s)

    def alpha_at(j):
        return j < n and alpha_p(s[j])

    def digit_at(j):
        return j < n and digit_p(s[j])

    def punct_at(j):
        return j < n and not whitespace_p(s[j]) and not alpha_p(s[j]) and not digit_p(s[j])

    def run(j, pred):
        while pred(j):
            j += 1
        return j

    while i < n:
        c = s[i]
        if c == "'" and i + 1 < n:
            rest = s[i + 1:min(n, i + 3)]
            m = next((x for x in CONTRACTIONS if len(x) <= len(rest) and rest.startswith(x)), None)
            if m:
                out.append(s[i:i + 1 + len(m)])
                i += 1 + len(m)
            else:
                out.append("'")
                i += 1
        elif not llama3 and (alpha_at(i) or (c == " " and alpha_at(i + 1))):
            k = run(i + 1 if c == " " else i, alpha_at)
            out.append(s[i:k])
            i = k
        elif llama3 and (alpha_at(i) or (c not in ("\r", "\n") and not digit_at(i)
                                          and alpha_at(i + 1))):
            k = run(i if alpha_at(i) else i + 1, alpha_at)
            out.append(s[i:k])
            i = k
        elif not llama3 and (digit_at(i) or (c == " " and digit_at(i + 1))):
            k = run(i + 1 if c == " " else i, digit_at)
            out.append(s[i:k])
            i = k
        elif llama3 and digit_at(i):
            out.append(s[i])
            i += 1
        elif punct_at(i) or (c == " " and punct_at(i + 1)):
            k = run(i + 1 if c == " " else i, punct_at)
            out.append(s[i:k])
            i = k
        else:
            k = i
            while k < n and whitespace_p(s[k]):
                k += 1
            out.append(s[i:k])
            i = k
    return out


def pretokenize_gpt2(s):
    return _scan(s, False)


def pretokenize_llama3(s):
    return _scan(s, True)


def pretokenize_metaspace(s):
    return [w if i == 0 else " " + w for i, w in enumerate(split_spaces(s))]


class Tokenizer:
    def __init__(self, kind, vocab, inv, *, merges=None, scores=None, lowercase=True,
                 max_len=512, cls="[CLS]", sep="[SEP]", unk="[UNK]", byte_level=False,
                 pretok="gpt2", bos=None, eos=None):
        self.kind, self.vocab, self.inv = kind, vocab, inv
        self.merges, self.scores = merges or {}, scores or {}
        self.lowercase, self.max_len = lowercase, max_len
        self.cls, self.sep, self.unk = cls, sep, unk
        self.byte_level, self.pretok, self.bos, self.eos = byte_level, pretok, bos, eos
        self.lisp_advance = True

    # models
    def wordpiece_word(self, w):
        if len(w) > 100:
            return [self.unk]
        pieces, start = [], 0
        while start < len(w):
            end, found = len(w), None
            while end > start:
                sub = w[start:end] if start == 0 else "##" + w[start:end]
                if sub in self.vocab:
                    found = sub
                    break
                end -= 1
            if found:
                pieces.append(found)
                # the Lisp advances by (length found), "##" included; with
                # lisp_advance off the advance is the matched characters only
                # (the usual WordPiece, used to pin the rest against HF)
                start += len(found) if self.lisp_advance or start == 0 else len(found) - 2
            else:
                pieces.append(self.unk)
                start = len(w)
        return pieces

    def bpe(self, word):
        parts = list(word)
        while True:
            best, idx = None, -1
            for i in range(len(parts) - 1):
                r = self.merges.get((parts[i], parts[i + 1]))
                if r is not None and (best is None or r < best):
                    best, idx = r, i
            if idx < 0:
                return parts
            parts = parts[:idx] + [parts[idx] + parts[idx + 1]] + parts[idx + 2:]

    def unigram(self, s):
        n = len(s)
        best = [float("-inf")] * (n + 1)
        back = [-1] * (n + 1)
        best[0] = 0.0
        for i in range(n):
            for j in range(i + 1, min(n, i + 20) + 1):
                sc = self.scores.get(s[i:j])
                if sc is not None and best[i] + sc > best[j]:
                    best[j] = best[i] + sc
                    back[j] = i
        ids, j = [], n
        while j > 0:
            i = back[j]
            if i < 0:   # no segmentation: the Lisp's (subseq s -1 j) signals
                raise ValueError("no unigram segmentation")
            ids.insert(0, self.vocab.get(s[i:j]))
            j = i
        return ids

    def encode(self, text):
        s = lowercase(text) if self.lowercase else text
        if self.kind == "wordpiece":
            words = pretokenize_wordpiece(s)
        elif self.kind == "bpe":
            words = pretokenize_llama3(s) if self.pretok == "llama3" else pretokenize_gpt2(s)
        else:
            words = pretokenize_metaspace(s)
        toks = []
        for w in words:
            if self.kind == "wordpiece":
                toks += self.wordpiece_word(w)
            elif self.kind == "bpe":
                toks += self.bpe(bytes_to_unicode_str(w.encode("utf-8")) if self.byte_level
                                 else w)
            else:
                toks += self.unigram(w)
        body = toks[:min(len(toks), self.max_len - 2)]
        unk = self.vocab.get(self.unk)
        cls = self.vocab.get(self.cls)
        sep = self.vocab.get(self.sep)
        # tk-encode looks every body element up in the string-keyed vocab
        # (tokenizer.lisp:228); unigram-viterbi's elements are already ids, so
        # they are not found and become the unknown token
        ids = [self.vocab.get(t, unk) if isinstance(t, str) else unk for t in body]
        if any(i is None for i in ids):
            raise KeyError("token outside the vocabulary and no unknown token")
        out = ([self.bos] if self.bos is not None else []) + ([cls] if cls is not None else [])
        out += ids
        out += ([sep] if sep is not None else []) + ([self.eos] if self.eos is not None else [])
        return out

    def decode(self, ids):
        return "".join(self.inv[i] for i in ids if 0 <= i < len(self.inv) and self.inv[i])


def json_specials(tj):
    by_name = {a["content"]: a["id"] for a in tj.get("added_tokens") or []}
    bos = eos = None
    pp = tj.get("post_processor")
    pp = pp if isinstance(pp, dict) else None
    ptype = pp.get("type") if pp else None
    if ptype in ("RobertaProcessing", "BertProcessing"):
        cls, sep = pp.get("cls"), pp.get("sep")
        bos = cls[1] if cls else None
        eos = sep[1] if sep else None
    else:
        procs = pp.get("processors") if pp else None
        procs = procs if isinstance(procs, list) else None
        tp = next((p for p in procs or [] if p.get("type") == "TemplateProcessing"), None)
        if tp:
            seen_seq = False
            for item in tp.get("single") or []:
                tok = item.get("SpecialToken")
                if tok:
                    idv = by_name.get(tok.get("id"))
                    if seen_seq:
                        eos = idv
                    else:
                        bos = idv
                if item.get("Sequence"):
                    seen_seq = True
    return bos, eos


def pretok_mode(tj):
    pre = tj.get("pre_tokenizer")
    pre = pre if isinstance(pre, dict) else None
    procs = pre.get("pretokenizers") if pre else None
    pat = None
    for p in procs or [pre]:
        if not p:
            continue
        split = p.get("pattern")
        if split:
            rx = split.get("Regex") if isinstance(split, dict) else None
            if rx:
                pat = rx
    return "llama3" if pat and "\\r\\n" in pat else "gpt2"


def from_json(path):
    with open(path, encoding="utf-8") as f:
        tj = json.load(f)
    model = tj["model"]
    mtype, vocab = model["type"], model["vocab"]
    norm = tj.get("normalizer")
    lower = bool(norm.get("lowercase")) if isinstance(norm, dict) else False
    inv = [""] * (max(vocab.values()) + 1)
    for t, i in vocab.items():
        inv[i] = t
    bos, eos = json_specials(tj)
    if mtype == "WordPiece":
        return Tokenizer("wordpiece", vocab, inv, lowercase=lower,
                         cls="" if bos is not None else "[CLS]",
                         sep="" if eos is not None else "[SEP]", unk="[UNK]", bos=bos, eos=eos)
    if mtype == "BPE":
        merges, rank = {}, 0
        for m in model.get("merges") or []:
            if isinstance(m, list):
                pair = (m[0], m[1])
            else:
                sp = m.find(" ")
                pair = (m[:sp], m[sp + 1:]) if sp >= 0 else None
            if pair:
                merges[pair] = rank   # a repeated pair keeps its later rank
                rank += 1
        return Tokenizer("bpe", vocab, inv, merges=merges, lowercase=False, cls="", sep="",
                         unk="<unk>", byte_level=True, pretok=pretok_mode(tj), bos=bos, eos=eos)
    raise ValueError(f"unsupported tokenizer.json model type {mtype}")


def _lines(path):
    """read-line over the file: split at newlines; a final line without one
    still counts, a trailing newline adds no empty line."""
    with open(path, encoding="utf-8", newline="") as f:
        lines = f.read().split("\n")
    if lines and lines[-1] == "":
        lines = lines[:-1]
    return lines


def from_vocab_txt(path, lowercase=True):
    """make-tokenizer :wordpiece (tokenizer.lisp:126-140): id = line number,
    each line trimmed of carriage returns and spaces."""
    vocab, inv = {}, []
    for line in _lines(path):
        tok = line.strip("\r ")
        vocab[tok] = len(inv)
        inv.append(tok)
    return Tokenizer("wordpiece", vocab, inv, lowercase=lowercase)


def from_vocab_merges(vocab_json, merges_txt, lowercase=True, byte_level=False, pretok="gpt2",
                      cls="[CLS]", sep="[SEP]", unk="[UNK]", bos=None, eos=None):
    """make-tokenizer :bpe (tokenizer.lisp:141-173): vocab.json token -> id;
    merges.txt ranked from the second line, '#' lines skipped, split at the
    first space."""
    with open(vocab_json, encoding="utf-8") as f:
        vocab = json.load(f)
    inv = [""] * (max(vocab.values()) + 1)
    for t, i in vocab.items():
        inv[i] = t
    merges, rank = {}, 0
    for n, line in enumerate(_lines(merges_txt)):
        if n == 0 or not line or line[0] == "#":
            continue
        sp = line.find(" ")
        if sp >= 0:
            merges[(line[:sp], line[sp + 1:])] = rank
            rank += 1
    return Tokenizer("bpe", vocab, inv, merges=merges, lowercase=lowercase, byte_level=byte_level,
                     pretok=pretok, cls=cls, sep=sep, unk=unk, bos=bos, eos=eos)


def from_unigram_scores(scores_json, lowercase=True):
    """make-tokenizer :unigram (tokenizer.lisp:174-197): {token: log score},
    ids in the file's key order."""
    with open(scores_json, encoding="utf-8") as f:
        sc = json.load(f)
    vocab, inv, scores = {}, [], {}
    for t, v in sc.items():
        vocab[t] = len(inv)
        inv.append(t)
        scores[t] = float(v)
    return Tokenizer("unigram", vocab, inv, scores=scores, lowercase=lowercase)
