"""Native genesis-pack against the Python statement of the same algorithm.

A rank table is trained on the test corpus (all 256 bytes plus frequent
merges), the corpus is packed by the C++ tool with 1 and 4 threads, and the
binary files and meta.json are compared with a pure-Python packer."""

import collections
import json
import os
import random

import numpy as np
import pytest

from olympus.data.bpe import BytePairEncoder, CL100K_PATTERN, save_tiktoken_ranks
from olympus.data.genesis_pack import build_genesis_pack, pack_corpus

ALPHABET = (list("abcdefghijklmnopqrstuvwxyzABCDEFGHIJKLMNOPQRSTUVWXYZ0123456789") + list(" \t\n\r.,;:!?'\"()[]{}-_/@#")
            + ["é", "ß", "Ω", "ж", "中", "文", "の", "😀", " ", "٣", "½", "ſ", "'s", "'re", "'LL", "\r\n", "  "])


def _doc(rng):
    words = []
    for _ in range(rng.randint(5, 80)):
        w = "".join(rng.choice(ALPHABET) for _ in range(rng.randint(1, 9)))
        words.append(w)
    return " ".join(words)


def _train_ranks(texts, merges=400):
    import regex

    pat = regex.compile(CL100K_PATTERN)
    ranks = {bytes([b]): b for b in range(256)}
    words = collections.Counter(p.encode() for t in texts for p in pat.findall(t))
    seqs = {w: [w[i:i + 1] for i in range(len(w))] for w in words}
    for _ in range(merges):
        pairs = collections.Counter()
        for w, parts in seqs.items():
            for a, b in zip(parts, parts[1:]):
                pairs[a + b] += words[w]
        if not pairs:
            break
        best = max(pairs.items(), key=lambda kv: (kv[1], kv[0]))[0]
        if best in ranks:
            break
        ranks[best] = len(ranks)
        for w, parts in seqs.items():
            i, out = 0, []
            while i < len(parts):
                if i + 1 < len(parts) and parts[i] + parts[i + 1] == best:
                    out.append(best)
                    i += 2
                else:
                    out.append(parts[i])
                    i += 1
            seqs[w] = out
    return ranks


def _py_pack(files, enc, block, ratio, eos):
    toks, docs, skipped, ntok = [], 0, 0, 0
    for path in files:
        with open(path, "rb") as f:
            data = f.read()
            raws = data.split(b"\n")
            if data.endswith(b"\n"):
                raws = raws[:-1]  # no empty line after the final newline
            for raw in raws:
                try:
                    line = raw.decode("utf-8")
                except UnicodeDecodeError:
                    continue
                if line.endswith("\r"):
                    line = line[:-1]
                try:
                    rec = json.loads(line)
                    assert isinstance(rec, dict)
                except Exception:
                    skipped += 1
                    continue
                text = rec.get("text") if rec.get("text") is not None else rec.get("content")
                if not isinstance(text, str) or len(text.encode()) < 100:
                    skipped += 1
                    continue
                ids = enc.encode_ordinary(text)
                docs += 1
                ntok += len(ids)
                toks += ids + [eos]
    nb = len(toks) // block
    toks = toks[: nb * block]
    tb = int(nb * ratio)
    meta = {"block_size": block, "dtype": "uint32", "vocab_size": 100287, "eos_id": eos, "train_blocks": tb,
            "val_blocks": nb - tb, "total_tokens": ntok, "total_docs": docs, "skipped_docs": skipped,
            "source_files": [os.path.basename(p) for p in files]}
    return np.array(toks[: tb * block], dtype=np.uint32), np.array(toks[tb * block:], dtype=np.uint32), meta


@pytest.fixture(scope="module")
def corpus(tmp_path_factory):
    rng = random.Random(7)
    d = tmp_path_factory.mktemp("corpus")
    texts = [_doc(rng) for _ in range(400)]
    files = []
    for k in range(3):
        p = d / f"part{k}.jsonl"
        with open(p, "w", encoding="utf-8") as f:
            for t in texts[k::3]:
                key = "text" if rng.random() < 0.7 else "content"
                f.write(json.dumps({key: t, "id": rng.randint(0, 99), "meta": {"a": [1, 2.5e3, None]}},
                                   ensure_ascii=rng.random() < 0.5) + "\n")
            f.write('{"text": "too short"}\n')
            f.write("not json\n")
            f.write('{"content": null, "text": null}\n')
            f.write("\n")
        files.append(str(p))
    (d / "ignored.txt").write_text("{}")
    ranks = _train_ranks(texts)
    vocab = d / "test.tiktoken"
    save_tiktoken_ranks(ranks, str(vocab))
    return d, sorted(files), str(vocab), ranks


def test_bpe_pieces_follow_the_pattern():
    from olympus.data.bpe import byte_pair_merge

    ranks = {bytes([b]): b for b in range(256)}
    ranks[b"ab"] = 256
    ranks[b"abc"] = 257
    assert byte_pair_merge(b"abcab", ranks) == [257, 256]
    enc = BytePairEncoder(ranks)
    assert enc.pieces("Hello  world's 12345\n\n x") == ["Hello", " ", " world", "'s", " ", "123", "45", "\n\n", " x"]


@pytest.mark.parametrize("threads", [1, 4])
def test_native_pack_matches_python(corpus, tmp_path, threads):
    d, files, vocab, ranks = corpus
    build_genesis_pack()
    out = tmp_path / "out"
    meta = pack_corpus(str(d), str(out), vocab, block_size=64, train_ratio=0.9, eos_id=3, threads=threads)
    train, val, want = _py_pack(files, BytePairEncoder(ranks), 64, 0.9, 3)
    got_train = np.fromfile(out / "train_input_ids.bin", dtype="<u4")
    got_val = np.fromfile(out / "val_input_ids.bin", dtype="<u4")
    assert meta == want
    assert want["skipped_docs"] >= 4 * 3 and want["total_docs"] > 100
    np.testing.assert_array_equal(got_train, train)
    np.testing.assert_array_equal(got_val, val)
    text = (out / "meta.json").read_text()
    assert text == json.dumps(want, indent=2, sort_keys=True)  # serde_json pretty layout, sorted keys


def test_native_pack_skip_rules(tmp_path, corpus):
    _, _, vocab, _ = corpus
    d = tmp_path / "in"
    d.mkdir()
    long = "x" * 120
    lines = [
        json.dumps({"text": long}),                        # ok
        json.dumps({"text": "é" * 50}),                    # 100 UTF-8 bytes: ok
        json.dumps({"text": "é" * 49 + "a"}),              # 99 bytes: skipped
        '{"text": "%s", "text": "%s"}' % (long, long),     # duplicate field: skipped
        '{"text": 5}',                                     # wrong type: skipped
        '{"content": "%s"}' % long,                        # content fallback: ok
        '{"text": "%s"} trailing' % long,                  # trailing garbage: skipped
        '{"text": "\\ud800"}',                             # lone surrogate: skipped
    ]
    (d / "a.jsonl").write_bytes(("\n".join(lines) + "\n").encode() + b"\xff\xfe bad utf8\n")
    meta = pack_corpus(str(d), str(tmp_path / "o"), vocab, block_size=8, train_ratio=0.5, eos_id=1, threads=2)
    assert meta["total_docs"] == 3 and meta["skipped_docs"] == 5


@pytest.mark.skipif(not os.environ.get("LRB_CL100K_RANKS"),
                    reason="set LRB_CL100K_RANKS to the cl100k_base.tiktoken rank file (not shipped; no network here)")
def test_native_pack_with_the_cl100k_table(tmp_path):
    """With the real cl100k_base rank table: the public token ids of a known
    string, through the Python encoder and through the native packer's stream."""
    from olympus.data.bpe import load_tiktoken_ranks

    ranks = load_tiktoken_ranks(os.environ["LRB_CL100K_RANKS"])
    enc = BytePairEncoder(ranks)
    assert enc.encode_ordinary("hello world") == [15339, 1917]
    d = tmp_path / "in"
    d.mkdir()
    text = "hello world " * 20  # 240 bytes: kept
    (d / "a.jsonl").write_text(json.dumps({"text": text}) + "\n")
    build_genesis_pack()
    meta = pack_corpus(str(d), str(tmp_path / "o"), os.environ["LRB_CL100K_RANKS"], block_size=4, train_ratio=1.0,
                       eos_id=100257, threads=1)
    got = np.fromfile(tmp_path / "o" / "train_input_ids.bin", dtype="<u4")
    want = enc.encode_ordinary(text) + [100257]
    assert meta["total_docs"] == 1
    np.testing.assert_array_equal(got, np.array(want[: len(want) // 4 * 4], dtype=np.uint32))
