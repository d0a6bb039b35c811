"""The C++ prompt tokenizer (pi05_tokenizer_*) against Python sentencepiece on BPE models trained here
(identity normalization, the kind Gemma's tokenizer is; the Gemma model file itself is not available):
byte fallback on and off, user-defined symbols, dummy prefix and extra-whitespace options; every id
sequence identical, as the reference's tokenizer matched sentencepiece on 4040 sentences
(docs/archive/windows/π05_네이티브엔진.md:83).  Also the pi0.5 prompt layout against a restatement of
openpi's PaligemmaTokenizer.tokenize.  CPU only."""
import numpy as np
import pytest

spm = pytest.importorskip("sentencepiece")

WORDS = ("pick up the red cup and place it on the shelf turn on the radio open the drawer move left right "
         "forward backward grasp release robot arm gripper table kitchen bottle 0 1 2 3 4 5 6 7 8 9 "
         "Task State Action").split()


def corpus(rng, n=3000):
    lines = []
    for _ in range(n):
        k = int(rng.integers(3, 14))
        ws = [WORDS[int(i)] for i in rng.integers(0, len(WORDS), k)]
        if rng.random() < 0.3:
            ws.insert(int(rng.integers(0, k)), str(int(rng.integers(0, 256))))
        if rng.random() < 0.1:
            ws.append("é à ü ñ")
        lines.append(" ".join(ws))
    return lines


def sample_strings(rng):
    out = ["", " ", "a", "pick up the red cup", "  two  spaces  and trailing  ", "tab\tand\nnewline",
           "Task: turn on the radio, State: 12 255 0 7;\nAction: ", "unicode: 한국어 텍스트 ✓ 🤖 ÿ", "<ctl> <ctl><ctl>x",
           "__under_score__", "1234567890 99 100 101", "é à ü ñ ø å"]
    for line in corpus(rng, 300):
        if rng.random() < 0.2:
            line = line.upper()
        out.append(line)
    return out


@pytest.mark.parametrize("opts", [
    dict(byte_fallback=True, add_dummy_prefix=False, remove_extra_whitespaces=False, user_defined_symbols=["<ctl>", "\n"]),
    dict(byte_fallback=True, add_dummy_prefix=True, remove_extra_whitespaces=True),
    dict(byte_fallback=False, add_dummy_prefix=True, remove_extra_whitespaces=False, user_defined_symbols=["Task:"],
         vocab_size=250),
], ids=["gemma_like", "defaults_bytes", "no_bytes"])
def test_encode_matches_sentencepiece(pn, tmp_path, opts):
    rng = np.random.default_rng(7)
    text = tmp_path / "corpus.txt"
    text.write_text("\n".join(corpus(rng)) + "\n")
    prefix = str(tmp_path / "m")
    opts = dict(opts)
    vocab = opts.pop("vocab_size", 400)
    spm.SentencePieceTrainer.train(input=str(text), model_prefix=prefix, vocab_size=vocab, model_type="bpe",
                                   normalization_rule_name="identity", character_coverage=1.0, split_digits=True,
                                   minloglevel=2, **opts)
    sp = spm.SentencePieceProcessor(model_file=prefix + ".model")
    tok = pn.Tokenizer(prefix + ".model")
    assert tok.vocab_size == sp.get_piece_size()
    bad = []
    for s in sample_strings(rng):
        for bos in (False, True):
            want = ([sp.bos_id()] if bos else []) + sp.encode(s)
            got = tok.encode(s, add_bos=bos)
            if got != want:
                bad.append((s, got, want))
    assert not bad, bad[:3]


def openpi_prompt(sp, task, state, max_len):
    """openpi PaligemmaTokenizer.tokenize (pi0.5 layout when a state is given), restated"""
    cleaned = task.strip().replace("_", " ").replace("\n", " ")
    if state is not None:
        bins = np.digitize(state, bins=np.linspace(-1, 1, 256 + 1)[:-1]) - 1
        full = f"Task: {cleaned}, State: {' '.join(map(str, bins))};\nAction: "
        ids = [sp.bos_id()] + sp.encode(full)
    else:
        ids = [sp.bos_id()] + sp.encode(cleaned) + sp.encode("\n")
    n = min(len(ids), max_len)
    ids = (ids + [0] * max_len)[:max_len]
    return np.asarray(ids, np.int32), np.arange(max_len) < n


def test_pi05_prompt_layout(pn, tmp_path):
    rng = np.random.default_rng(8)
    text = tmp_path / "corpus.txt"
    text.write_text("\n".join(corpus(rng)) + "\n")
    prefix = str(tmp_path / "p")
    spm.SentencePieceTrainer.train(input=str(text), model_prefix=prefix, vocab_size=400, model_type="bpe",
                                   normalization_rule_name="identity", byte_fallback=True, add_dummy_prefix=False,
                                   remove_extra_whitespaces=False, split_digits=True, minloglevel=2)
    sp = spm.SentencePieceProcessor(model_file=prefix + ".model")
    tok = pn.Tokenizer(prefix + ".model")
    for task, st, max_len in [("  turn_on the radio\n", rng.uniform(-1.1, 1.1, 23).astype(np.float32), 200),
                              ("pick up the cup", rng.uniform(-1, 1, 23).astype(np.float32), 20),
                              ("open the drawer", None, 48)]:
        ids, mask = tok.prompt(task, st, max_len)
        want_ids, want_mask = openpi_prompt(sp, task, st, max_len)
        np.testing.assert_array_equal(ids, want_ids)
        np.testing.assert_array_equal(mask, want_mask)


def test_tokenizer_rejects_other_files(pn, tmp_path):
    bad = tmp_path / "x.model"
    bad.write_bytes(b"not a model")
    with pytest.raises(pn.Pi05Error):
        pn.Tokenizer(str(bad))
