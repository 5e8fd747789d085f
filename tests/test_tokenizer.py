"""The host tokenizer (include/nemo.h nemo_tokenizer_*) against Hugging Face
`tokenizers`, the library whose tokenizer.json semantics it restates (the
reference tokenizes with its JS port, @huggingface/transformers 3.8.1,
src/main.ts:164-165). The real Nemotron-3-Embed tokenizer.json is not on this
machine, so byte-level BPE tokenizers of the same family are trained here with
`tokenizers` (Tekken-style Split regex + ByteLevel, and GPT-2 ByteLevel) and
both implementations encode the same texts: ids must be identical."""
import numpy as np
import pytest

tokenizers = pytest.importorskip("tokenizers")
from tokenizers import Regex, Tokenizer, decoders, models, pre_tokenizers, processors, trainers  # noqa: E402

from nemo_b200.runtime import NemoError, NemotronTokenizer  # noqa: E402

TEKKEN = (r"[^\r\n\p{L}\p{N}]?[\p{Lu}\p{Lt}\p{Lm}\p{Lo}\p{M}]*[\p{Ll}\p{Lm}\p{Lo}\p{M}]+|[^\r\n\p{L}\p{N}]?"
          r"[\p{Lu}\p{Lt}\p{Lm}\p{Lo}\p{M}]+[\p{Ll}\p{Lm}\p{Lo}\p{M}]*|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n/]*|"
          r"\s*[\r\n]+|\s+(?!\S)|\s+")

PIECES = ["The", "quick", "brown", "fox", "jumps", "over", "the", "lazy", "dog", "WebGPU", "embedding", "benchmark",
          "naïve", "café", "Übermäßig", "straße", "Ελληνικά", "русский", "中文字符", "日本語", "한국어", "العربية",
          "हिन्दी", "é", "ﬁne", "İstanbul", "ǅemal", "12345", "3.14159", "1,000,000", "x²", "½", "٣٤", "🙂", "👍🏽",
          "def f(x):", "return x*2;", "a/b/c", "https://example.com/path?q=1", "foo_bar", "CamelCaseWord",
          "ALLCAPS", "it's", "we're", "they'll", "I'd", "you've", "I'm", "don't", "--", "...", "!?", "#tag", "@user",
          "\t", "\n", "\r\n", "  ", "   \n\n", " ", "　", "<s>", "</s>", "[INST]", "<mask>"]


def corpus(seed, n=3000):
    rng = np.random.default_rng(seed)
    seps = [" ", " ", " ", "\n", ", ", ". ", "  ", "\t"]
    return ["".join(PIECES[i] + seps[j] for i, j in zip(rng.integers(0, len(PIECES), 12),
                                                        rng.integers(0, len(seps), 12))) for _ in range(n)]


def texts(seed, n=300):
    rng = np.random.default_rng(seed)
    seps = [" ", "", "\n", " \n ", "  ", "\r\n", "\t", ".", "/", "'"]
    out = ["", " ", "a", "  leading", "trailing  ", "WebGPU embedding benchmark.", "\n\n\nx", "x\n\n\n", "<s>",
           "a<s>b", "x [INST] y", "word<mask> z", "3<mask>4", "Hello   \n   world", "'s 't 're"]
    for _ in range(n):
        k = int(rng.integers(1, 14))
        out.append("".join(PIECES[i] + seps[j] for i, j in zip(rng.integers(0, len(PIECES), k),
                                                               rng.integers(0, len(seps), k))))
        # random code points, letters and marks and symbols from several blocks
        cps = rng.choice([0x41, 0x61, 0x30, 0x20, 0x2E, 0xE9, 0x301, 0x4E2D, 0x1F642, 0x3B1, 0x2C, 0xA, 0x5F],
                         size=int(rng.integers(1, 20)))
        out.append("".join(chr(int(c)) for c in cps))
    return out


def make_tekken(ignore_merges):
    tok = Tokenizer(models.BPE(ignore_merges=ignore_merges))
    tok.pre_tokenizer = pre_tokenizers.Sequence([
        pre_tokenizers.Split(Regex(TEKKEN), behavior="isolated", invert=False),
        pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)])
    tok.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(vocab_size=1500, special_tokens=["<unk>", "<s>", "</s>", "[INST]"],
                                  initial_alphabet=pre_tokenizers.ByteLevel.alphabet(), show_progress=False)
    tok.train_from_iterator(corpus(1), trainer)
    tok.add_special_tokens([tokenizers.AddedToken("<mask>", lstrip=True, rstrip=False, special=True)])
    tok.post_processor = processors.TemplateProcessing(single="<s> $A </s>", special_tokens=[("<s>", 1), ("</s>", 2)])
    return tok


def make_gpt2():
    tok = Tokenizer(models.BPE())
    tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=True, use_regex=True)
    tok.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(vocab_size=1200, special_tokens=["<s>", "</s>"],
                                  initial_alphabet=pre_tokenizers.ByteLevel.alphabet(), show_progress=False)
    tok.train_from_iterator(corpus(2), trainer)
    tok.post_processor = processors.RobertaProcessing(("</s>", 1), ("<s>", 0))
    return tok


@pytest.mark.parametrize("kind", ["tekken", "tekken_ignore_merges", "gpt2"])
def test_tokenizer_matches_hf_tokenizers(kind):
    ref = make_gpt2() if kind == "gpt2" else make_tekken(kind == "tekken_ignore_merges")
    ours = NemotronTokenizer(ref.to_str().encode("utf-8"))
    try:
        for t in texts(3):
            want = ref.encode(t).ids
            got = ours.encode(t)
            assert got == want, (repr(t), got, want)
        # the engine's call form: tokenizer(text)["input_ids"] is [1 x n] with BOS first
        ids = ours("WebGPU embedding benchmark.")["input_ids"]
        assert ids.shape[0] == 1 and ids[0, 0] == (0 if kind == "gpt2" else 1)
    finally:
        ours.close()


def test_tokenizer_rejects_what_it_does_not_restate():
    tok = make_tekken(False)
    import json
    d = json.loads(tok.to_str())
    d["normalizer"] = {"type": "NFC"}
    with pytest.raises(NemoError, match="normalizers are not supported"):
        NemotronTokenizer(json.dumps(d).encode())
    d = json.loads(tok.to_str())
    d["pre_tokenizer"]["pretokenizers"][0]["pattern"]["Regex"] = r"\w+"
    with pytest.raises(NemoError, match="unsupported pre-tokenizer pattern"):
        NemotronTokenizer(json.dumps(d).encode())
    ours = NemotronTokenizer(tok.to_str().encode())
    with pytest.raises(NemoError, match="UTF-8"):
        import ctypes
        from nemo_b200.runtime import check, load_library
        n = ctypes.c_size_t()
        check(load_library().nemo_tokenizer_encode(ours._h, b"\xff\xfe", 2, None, 0, ctypes.byref(n)))
    ours.close()
