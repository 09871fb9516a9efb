"""Tokenizer fixtures for the tokenizer.lisp parity tests (run from the repo
root: python tests/golden/make_tokenizers.py).

Trains small tokenizers with Hugging Face `tokenizers` on a seeded synthetic
corpus and writes them in the formats tokenizer.lisp reads:
  wordpiece.json (WordPiece, BertNormalizer lowercase, TemplateProcessing
  [CLS] $A [SEP]), vocab.txt (the same vocabulary);
  bpe_gpt2.json (byte-level BPE, GPT-2 regex, a Sequence post-processor whose
  TemplateProcessing adds <s> ... </s>), vocab.json + merges.txt;
  bpe_llama3.json (byte-level BPE behind a Llama-3 style Split regex);
  unigram.json ({piece: log score}, make-tokenizer :unigram's input).
Then encodes texts.json with the Python restatement (oracle/tokenizer_ref.py)
into expected.json, and checks the restatement against `tokenizers` itself
on the texts where tokenizer.lisp and HF do the same thing (ASCII, single
spaces, no contractions)."""
import json
import os
import random
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from tokenizers import Tokenizer, decoders, models, normalizers, pre_tokenizers  # noqa: E402
from tokenizers import processors, trainers  # noqa: E402

from oracle import tokenizer_ref as ref  # noqa: E402

OUT = os.path.join(HERE, "tok")
SYL = ["ka", "to", "ri", "na", "mo", "se", "lu", "pe", "di", "ga", "vo", "qui", "stra", "ble",
       "ing", "tion", "er", "ed", "ly", "pre", "un", "re", "ment", "ness"]


def word(rng):
    return "".join(rng.choice(SYL) for _ in range(rng.randint(1, 4)))


def sentence(rng, unicode_ok):
    parts = []
    for _ in range(rng.randint(3, 14)):
        r = rng.random()
        if r < 0.62:
            w = word(rng)
            parts.append(w.capitalize() if rng.random() < 0.2 else w)
        elif r < 0.72:
            parts.append(str(rng.randint(0, 99999)))
        elif r < 0.80:
            parts.append(rng.choice([",", ".", "!", "?", ";", ":", "(", ")", "-", "\"", "...", "&"]))
        elif r < 0.87:
            parts.append(word(rng) + rng.choice(["'s", "'t", "'re", "'ve", "'ll", "'d", "'m", "'x"]))
        elif unicode_ok:
            parts.append(rng.choice(["café", "naïve", "Ärger", "ΣΟΦΙΑΣ", "λόγος", "日本語", "東京",
                                     "İstanbul", "straße", "emoji😀ok", "x y", "١٢٣",
                                     "Ωmega", "fi", "ǅemal"]))
        else:
            parts.append(word(rng))
    seps = [" "] * (len(parts) - 1)
    if unicode_ok:
        seps = [rng.choice([" ", " ", " ", "  ", "\t", "\n", " \n "]) for _ in seps]
    s = parts[0]
    for sp, p in zip(seps, parts[1:]):
        s += sp + p
    return s


def main():
    os.makedirs(OUT, exist_ok=True)
    rng = random.Random(20261202)
    corpus = [sentence(rng, True) for _ in range(4000)]
    trng = random.Random(7)
    texts = [sentence(trng, True) for _ in range(160)] + [sentence(trng, False) for _ in range(80)]
    texts += ["", "   ", "a", "x" * 150, "hello", "It's", "'", "don't'", "A'S", "Σ", "ΑΣ Σα",
              "  leading and trailing  ", "tab\there", "line\nbreak\r\nwin", "((nested))!!",
              "9999999999", "ab" * 300 + " tail", " ".join(word(trng) for _ in range(700))]

    # WordPiece
    wp = Tokenizer(models.WordPiece(unk_token="[UNK]", max_input_chars_per_word=100))
    wp.normalizer = normalizers.BertNormalizer(clean_text=False, handle_chinese_chars=False,
                                               strip_accents=False, lowercase=True)
    wp.pre_tokenizer = pre_tokenizers.BertPreTokenizer()
    wp.train_from_iterator(corpus, trainers.WordPieceTrainer(
        vocab_size=700, special_tokens=["[PAD]", "[UNK]", "[CLS]", "[SEP]", "[MASK]"]))
    wp.post_processor = processors.TemplateProcessing(
        single="[CLS] $A [SEP]", special_tokens=[("[CLS]", wp.token_to_id("[CLS]")),
                                                 ("[SEP]", wp.token_to_id("[SEP]"))])
    wp.save(os.path.join(OUT, "wordpiece.json"))
    vocab = wp.get_vocab()
    with open(os.path.join(OUT, "vocab.txt"), "w", encoding="utf-8") as f:
        for t, _ in sorted(vocab.items(), key=lambda kv: kv[1]):
            f.write(t + "\n")

    # byte-level BPE, GPT-2 regex, specials through a Sequence post-processor
    bpe = Tokenizer(models.BPE())
    bpe.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    bpe.decoder = decoders.ByteLevel()
    bpe.train_from_iterator(corpus, trainers.BpeTrainer(
        vocab_size=900, special_tokens=["<s>", "</s>", "<unk>"],
        initial_alphabet=pre_tokenizers.ByteLevel.alphabet()))
    bos, eos = bpe.token_to_id("<s>"), bpe.token_to_id("</s>")
    bpe.post_processor = processors.Sequence([
        processors.ByteLevel(trim_offsets=False),
        processors.TemplateProcessing(single="<s> $A </s>",
                                      special_tokens=[("<s>", bos), ("</s>", eos)])])
    bpe.save(os.path.join(OUT, "bpe_gpt2.json"))
    bpe.model.save(OUT)  # vocab.json + merges.txt

    # byte-level BPE behind a Llama-3 style split
    l3 = Tokenizer(models.BPE())
    pat = (r"(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+"
           r"[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+")
    l3.pre_tokenizer = pre_tokenizers.Sequence([
        pre_tokenizers.Split(pattern=__import__("tokenizers").Regex(pat), behavior="isolated"),
        pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)])
    l3.decoder = decoders.ByteLevel()
    l3.train_from_iterator(corpus, trainers.BpeTrainer(
        vocab_size=900, special_tokens=["<|begin|>", "<|end|>"],
        initial_alphabet=pre_tokenizers.ByteLevel.alphabet()))
    l3.save(os.path.join(OUT, "bpe_llama3.json"))

    # unigram scores: {piece: log score} over frequent substrings
    cnt = {}
    for s in corpus[:1500]:
        for w in s.lower().split():
            for i in range(len(w)):
                for j in range(i + 1, min(len(w), i + 6) + 1):
                    cnt[w[i:j]] = cnt.get(w[i:j], 0) + 1
    top = sorted(cnt.items(), key=lambda kv: (-kv[1], kv[0]))[:1500]
    tot = sum(c for _, c in top)
    import math
    scores = {"[UNK]": -20.0}
    for p, c in top:
        scores[p] = round(math.log(c / tot), 6)
    # every single character of the corpus and the test texts (lowercased), so
    # that every text has a segmentation (the Lisp signals otherwise)
    for ch in sorted(set("".join(corpus + texts).lower())):
        scores.setdefault(ch, -15.0)
    with open(os.path.join(OUT, "unigram.json"), "w", encoding="utf-8") as f:
        json.dump(scores, f, ensure_ascii=False)

    with open(os.path.join(OUT, "texts.json"), "w", encoding="utf-8") as f:
        json.dump(texts, f, ensure_ascii=False, indent=0)

    toks = {
        "wordpiece_json": ref.from_json(os.path.join(OUT, "wordpiece.json")),
        "bpe_gpt2_json": ref.from_json(os.path.join(OUT, "bpe_gpt2.json")),
        "bpe_llama3_json": ref.from_json(os.path.join(OUT, "bpe_llama3.json")),
        "wordpiece_txt": ref.from_vocab_txt(os.path.join(OUT, "vocab.txt")),
        "bpe_files": ref.from_vocab_merges(os.path.join(OUT, "vocab.json"),
                                           os.path.join(OUT, "merges.txt"), lowercase=False,
                                           byte_level=True, pretok="llama3",
                                           unk="<unk>", bos=bos, eos=eos),
        "unigram": ref.from_unigram_scores(os.path.join(OUT, "unigram.json")),
    }
    assert toks["bpe_llama3_json"].pretok == "llama3" and toks["bpe_gpt2_json"].pretok == "gpt2"
    assert toks["bpe_gpt2_json"].bos == bos and toks["bpe_gpt2_json"].eos == eos
    expected = {}
    for name, tk in toks.items():
        expected[name] = [tk.encode(t) for t in texts]
    with open(os.path.join(OUT, "expected.json"), "w") as f:
        json.dump(expected, f)

    # pin: where the Lisp algorithm and HF coincide, the restatement equals
    # HF -- WordPiece with the usual advance (the Lisp's "##"-counting advance
    # switched off), byte-level BPE as is
    wp_usual = ref.from_json(os.path.join(OUT, "wordpiece.json"))
    wp_usual.lisp_advance = False
    agree = 0
    for t in texts[160:240]:
        if "'" in t:
            continue
        assert wp.encode(t).ids == wp_usual.encode(t), t
        assert bpe.encode(t).ids == toks["bpe_gpt2_json"].encode(t), t
        agree += 1
    print(f"fixtures written; restatement == HF tokenizers on {agree} plain texts")


if __name__ == "__main__":
    main()
