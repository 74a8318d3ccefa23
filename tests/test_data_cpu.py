"""Native token-file loader (dion_b200._io) and the data pipeline around it:
file format, window contents, rank sharding, keyed per-epoch shuffling,
resume by position, host-side vocabulary check, tokenization of text files,
and the trainer / checkpoint / validation wiring (CPU)."""
import functools
import json
import math
import os

import numpy as np
import pytest
import torch

from dion_b200.data import (SyntheticTokens, TokenFileLoader, build_loader, expand_paths, token_file_info,
                            write_token_file)


def _stream(n, seed=0, vocab=50000):
    return np.random.default_rng(seed).integers(0, vocab, size=n, dtype=np.int64)


def test_token_file_roundtrip(tmp_path):
    a = _stream(1000, vocab=60000)
    p2 = write_token_file(str(tmp_path / "a.bin"), a)
    assert token_file_info(p2) == {"tokens": 1000, "bytes_per_token": 2, "header_bytes": 32}
    b = a + 70000  # needs 4 bytes per token
    p4 = write_token_file(str(tmp_path / "b.bin"), b)
    assert token_file_info(p4)["bytes_per_token"] == 4
    raw = tmp_path / "raw.u16"
    a.astype("<u2").tofile(raw)
    assert token_file_info(str(raw), 2) == {"tokens": 1000, "bytes_per_token": 2, "header_bytes": 0}
    with pytest.raises(RuntimeError, match="bytes_per_token"):
        token_file_info(str(raw))
    with pytest.raises(ValueError):
        write_token_file(str(tmp_path / "c.bin"), a + 70000, bytes_per_token=2)


def test_sequential_windows_and_rank_sharding(tmp_path):
    S, b, W = 16, 3, 2
    toks = _stream(100 * (S + 1) + 5)
    # two shards, so some windows cross the file boundary
    write_token_file(str(tmp_path / "d-0.bin"), toks[:777])
    write_token_file(str(tmp_path / "d-1.bin"), toks[777:])
    loaders = [TokenFileLoader(str(tmp_path), S, b, rank=r, world=W, shuffle=False) for r in range(W)]
    assert loaders[0].windows == 100 and loaders[0].total_tokens == toks.size
    for step in range(3):
        for r, ld in enumerate(loaders):
            t, l = ld.next()
            assert t.shape == (b, S) and t.dtype == torch.int64
            for i in range(b):
                g = step * W * b + r * b + i
                w = toks[g * (S + 1):(g + 1) * (S + 1)]
                assert torch.equal(t[i], torch.from_numpy(w[:-1]))
                assert torch.equal(l[i], torch.from_numpy(w[1:]))
            assert ld.position == (step + 1) * W * b


def test_shuffle_is_a_keyed_permutation_per_epoch(tmp_path):
    S = 8
    write_token_file(str(tmp_path / "x.bin"), _stream(37 * (S + 1) + 3))
    ld = TokenFileLoader(str(tmp_path / "x.bin"), S, 1, seed=7, shuffle=True)
    n = ld.windows
    assert n == 37
    e0 = [ld.window_of(g) for g in range(n)]
    e1 = [ld.window_of(g) for g in range(n, 2 * n)]
    assert sorted(e0) == list(range(n)) and sorted(e1) == list(range(n))
    assert e0 != list(range(n)) and e0 != e1
    again = TokenFileLoader(str(tmp_path / "x.bin"), S, 1, seed=7, shuffle=True)
    assert [again.window_of(g) for g in range(2 * n)] == e0 + e1
    other = TokenFileLoader(str(tmp_path / "x.bin"), S, 1, seed=8, shuffle=True)
    assert [other.window_of(g) for g in range(n)] != e0
    # the batches read exactly those windows
    toks = np.fromfile(str(tmp_path / "x.bin"), dtype="<u2", offset=32).astype(np.int64)
    for g in range(5):
        t, _ = ld.next()
        w = e0[g]
        assert torch.equal(t[0], torch.from_numpy(toks[w * (S + 1):w * (S + 1) + S]))


def test_resume_by_position(tmp_path):
    write_token_file(str(tmp_path / "r.bin"), _stream(50 * 33))
    a = TokenFileLoader(str(tmp_path / "r.bin"), 32, 2, rank=1, world=2, seed=3)
    for _ in range(4):
        a.next()
    sd = a.state_dict()
    assert sd == {"samples": 16}
    want = [a.next() for _ in range(3)]
    b = TokenFileLoader(str(tmp_path / "r.bin"), 32, 2, rank=1, world=2, seed=3)
    b.load_state_dict(sd)
    got = [b.next() for _ in range(3)]
    for (t0, l0), (t1, l1) in zip(want, got):
        assert torch.equal(t0, t1) and torch.equal(l0, l1)
    # a resume at another world size continues at the same global sample
    c = TokenFileLoader(str(tmp_path / "r.bin"), 32, 4, rank=0, world=1, seed=3, position=sd["samples"])
    assert c.window_of(sd["samples"]) == a.window_of(sd["samples"])


def test_vocab_check_and_errors(tmp_path):
    toks = _stream(20 * 9, vocab=100)
    toks[100] = 500
    write_token_file(str(tmp_path / "v.bin"), toks)
    ld = TokenFileLoader(str(tmp_path / "v.bin"), 8, 20, vocab=100, shuffle=False)
    with pytest.raises(RuntimeError, match="outside the vocabulary"):
        ld.next()
    write_token_file(str(tmp_path / "small.bin"), _stream(5))
    with pytest.raises(RuntimeError, match="fewer than one window"):
        TokenFileLoader(str(tmp_path / "small.bin"), 8, 1)
    with pytest.raises(FileNotFoundError):
        expand_paths(str(tmp_path / "nothing-*.bin"))


def test_synthetic_state_replays(tmp_path):
    a = SyntheticTokens(100, 8, 2, seed=4, rank=1, world=2)
    for _ in range(3):
        a.next()
    sd = a.state_dict()
    want = a.next()
    b = SyntheticTokens(100, 8, 2, seed=4, rank=1, world=2)
    b.load_state_dict(sd)
    got = b.next()
    assert torch.equal(want[0], got[0]) and torch.equal(want[1], got[1])
    assert isinstance(build_loader("synthetic", vocab=10, seq_len=4, local_batch=1, seed=0, rank=0, world=1),
                      SyntheticTokens)


def test_tokenize_text_inputs(tmp_path):
    from dion_b200.data.tokenize import ByteTokenizer, main

    docs = [{"text": f"document number {i} " + "x" * i} for i in range(12)]
    with open(tmp_path / "a.jsonl", "w") as f:
        for d in docs[:8]:
            f.write(json.dumps(d) + "\n")
    with open(tmp_path / "b.json", "w") as f:
        json.dump(docs[8:11], f)
    (tmp_path / "c.txt").write_text(docs[11]["text"])
    res = main(["--input", str(tmp_path / "a.jsonl"), str(tmp_path / "b.json"), str(tmp_path / "c.txt"),
                "--output", str(tmp_path / "out" / "tok"), "--val-docs", "2", "--shard-tokens", "120"])
    assert res["documents"] == 12 and res["vocab_size"] == 258 and len(res["train"]) > 1 and len(res["val"]) == 1
    tok = ByteTokenizer()
    stream = np.concatenate([np.fromfile(p, dtype="<u2", offset=32) for p in res["train"]]).tolist()
    # documents are [BOS] + bytes + [EOS], concatenated in input order
    texts, cur = [], None
    for t in stream:
        if t == tok.bos_id:
            cur = []
        elif t == tok.eos_id:
            texts.append(tok.decode(cur))
        else:
            cur.append(t)
    assert texts == [d["text"] for d in docs[2:]]
    assert res["train_tokens"] == len(stream)


def test_tokenize_parquet(tmp_path):
    pa = pytest.importorskip("pyarrow")
    import pyarrow.parquet as pq

    from dion_b200.data.tokenize import tokenize_to_files

    pq.write_table(pa.table({"text": ["alpha", "beta gamma"]}), str(tmp_path / "p.parquet"))
    res = tokenize_to_files([str(tmp_path / "p.parquet")], str(tmp_path / "pq"))
    assert res["train_tokens"] == (5 + 2) + (10 + 2)


def _corpus(tmp_path, n_tokens=40000, vocab=256):
    d = tmp_path / "corpus"
    write_token_file(str(d / "train-00000.bin"), _stream(n_tokens, seed=1, vocab=vocab))
    write_token_file(str(d / "train-00001.bin"), _stream(n_tokens, seed=2, vocab=vocab))
    write_token_file(str(tmp_path / "val.bin"), _stream(8000, seed=3, vocab=vocab))
    return str(d), str(tmp_path / "val.bin")


def test_trainer_on_token_files_with_validation_and_resume(tmp_path):
    from dion_b200 import train

    train_dir, val = _corpus(tmp_path)
    ck = tmp_path / "ck"
    out = tmp_path / "m"
    args = ["--config", "llama3_debug_muon", "--training.seq_len", "32", "--training.local_batch_size", "2",
            "--dataloader.dataset", train_dir, "--validator.enable",
            "--validator.dataset", val, "--validator.freq", "2", "--validator.steps", "2",
            "--checkpoint.enable", "--checkpoint.folder", str(ck), "--checkpoint.interval", "2",
            "--checkpoint.no-last_save_model_only", "--metrics.log_freq", "1"]
    losses = train.main(args + ["--training.steps", "2", "--metrics.save_jsonl", str(out)])
    assert len(losses) == 2 and all(math.isfinite(v) for v in losses)
    with open(out / "optimizer_metrics.jsonl") as fh:
        vals = [json.loads(l)["val_loss"] for l in fh if "val_loss" in l]
    assert len(vals) == 1 and math.isfinite(vals[0])
    # the checkpoint holds the data position (2 steps x 2 samples)
    import torch.distributed.checkpoint as dcp

    keys = dcp.FileSystemReader(str(ck / "step-2")).read_metadata().state_dict_metadata
    assert "train_state.data_samples" in keys
    losses = train.main(args + ["--training.steps", "4"])
    assert len(losses) == 2


def test_trainer_resume_restores_data_position(tmp_path):
    from dion_b200.checkpoint import CheckpointManager
    from dion_b200.integration.hybrid_optimizer import HybridOptimizersContainer
    from dion_b200.integration.trainer import Trainer, TrainerConfig

    train_dir, val = _corpus(tmp_path)
    cfg = TrainerConfig(model="debug", model_overrides=dict(vocab_size=256), seq_len=32, local_batch_size=2,
                        steps=4, warmup_steps=0, optimizer=HybridOptimizersContainer.Config(name="Muon"),
                        dataset=train_dir, val_dataset=val)
    tr = Trainer(cfg, device=torch.device("cpu"))
    ckm = CheckpointManager(str(tmp_path / "ck"), tr.model, tr.optimizers, interval=2, model_only_last=False)
    for s in (1, 2):
        tr.train_step(*tr.data.next())
        ckm.maybe_save(tr, s)
    nxt = tr.data.next()
    v1 = tr.validate(2)
    assert math.isfinite(v1) and v1 == tr.validate(2)  # the validation pass always starts at the first file

    tr2 = Trainer(cfg, device=torch.device("cpu"))
    CheckpointManager(str(tmp_path / "ck"), tr2.model, tr2.optimizers).maybe_load(tr2)
    assert tr2.step_idx == 2 and tr2.data.position == 4
    got = tr2.data.next()
    assert torch.equal(nxt[0], got[0]) and torch.equal(nxt[1], got[1])


def test_loader_rejects_bad_output_buffers(tmp_path):
    write_token_file(str(tmp_path / "o.bin"), _stream(10 * 9))
    ld = TokenFileLoader(str(tmp_path / "o.bin"), 8, 2)
    with pytest.raises(ValueError, match="shape"):
        ld._impl.next(torch.empty(2, 7, dtype=torch.int64), torch.empty(2, 8, dtype=torch.int64))
    with pytest.raises(ValueError, match="int64"):
        ld._impl.next(torch.empty(2, 8, dtype=torch.int32), torch.empty(2, 8, dtype=torch.int64))


def _validate_body(train_dir, val, rank, world):
    from dion_b200.integration.hybrid_optimizer import HybridOptimizersContainer
    from dion_b200.integration.trainer import Trainer, TrainerConfig

    cfg = TrainerConfig(model="debug", model_overrides=dict(vocab_size=256), seq_len=32, local_batch_size=4 // world,
                        steps=4, warmup_steps=0, optimizer=HybridOptimizersContainer.Config(name="Muon"),
                        dataset=train_dir, val_dataset=val, dp_shard=world)
    torch.manual_seed(0)
    tr = Trainer(cfg, device=torch.device("cpu"))
    return [tr.validate(3)]


def test_validation_is_split_over_data_parallel_ranks(tmp_path):
    """FSDP over 2 ranks: each rank evaluates its half of every validation
    batch and all ranks return the global mean, equal to one process
    evaluating the whole batches."""
    from test_distributed_cpu import spawn

    train_dir, val = _corpus(tmp_path)
    two = spawn(functools.partial(_validate_body, train_dir, val), world=2)
    one = spawn(functools.partial(_validate_body, train_dir, val), world=1)
    for out in (two, one):
        for r, (status, res) in out.items():
            assert status == "ok", res
    assert two[0][1] == two[1][1]
    assert abs(two[0][1][0] - one[0][1][0]) < 1e-4, (two[0][1], one[0][1])


def test_tokenize_with_worker_processes_keeps_order(tmp_path):
    from dion_b200.data.tokenize import tokenize_to_files

    with open(tmp_path / "d.jsonl", "w") as f:
        for i in range(300):
            f.write(json.dumps({"text": f"doc {i} " * (i % 7 + 1)}) + "\n")
    one = tokenize_to_files([str(tmp_path / "d.jsonl")], str(tmp_path / "one"), "byte")
    many = tokenize_to_files([str(tmp_path / "d.jsonl")], str(tmp_path / "many"), "byte", workers=3)
    a = np.fromfile(one["train"][0], dtype="<u2", offset=32)
    b = np.fromfile(many["train"][0], dtype="<u2", offset=32)
    assert one["documents"] == many["documents"] == 300 and np.array_equal(a, b)


def _docs(tmp_path, n=60):
    p = tmp_path / "docs.jsonl"
    with open(p, "w") as f:
        for i in range(n):
            f.write(json.dumps({"text": f"document {i}: " + "abc " * (i % 9 + 3)}) + "\n")
    return str(p)


def test_text_stream_loader_windows_ranks_and_resume(tmp_path):
    from dion_b200.data import TextStreamLoader
    from dion_b200.data.tokenize import ByteTokenizer, _encode_doc

    path = _docs(tmp_path)
    tok = ByteTokenizer()
    texts = [json.loads(l)["text"] for l in open(path)]
    S, b, W = 16, 2, 2
    for r in range(W):
        ld = TextStreamLoader(path, "byte", S, b, rank=r, world=W, vocab=258)
        stream = [t for i, txt in enumerate(texts) if i % W == r for t in _encode_doc(tok, txt)]
        got = [ld.next() for _ in range(3)]
        for k, (t, l) in enumerate(got):
            for i in range(b):
                w = stream[(k * b + i) * (S + 1):(k * b + i + 1) * (S + 1)]
                assert t[i].tolist() == w[:-1] and l[i].tolist() == w[1:]
        sd = ld.state_dict()
        assert sd == {"samples": 6}
        want = ld.next()
        again = TextStreamLoader(path, "byte", S, b, rank=r, world=W)
        again.load_state_dict(sd)
        nxt = again.next()
        assert torch.equal(want[0], nxt[0]) and torch.equal(want[1], nxt[1])
        ld.close()
        again.close()
    with pytest.raises(ValueError, match="vocabulary"):
        TextStreamLoader(path, "byte", S, b, vocab=100)


def test_trainer_on_text_stream(tmp_path):
    from dion_b200 import train

    path = _docs(tmp_path, 200)
    losses = train.main(["--config", "llama3_debug_muon", "--training.steps", "3", "--training.seq_len", "32",
                         "--training.local_batch_size", "2", "--metrics.log_freq", "1",
                         "--dataloader.dataset", "text:" + path, "--dataloader.tokenizer", "byte"])
    assert len(losses) == 3 and all(math.isfinite(v) for v in losses)


def test_validation_on_text_stream(tmp_path):
    from dion_b200.integration.hybrid_optimizer import HybridOptimizersContainer
    from dion_b200.integration.trainer import Trainer, TrainerConfig

    path = _docs(tmp_path, 120)
    cfg = TrainerConfig(model="debug", model_overrides=dict(vocab_size=512), seq_len=32, local_batch_size=2,
                        steps=2, warmup_steps=0, optimizer=HybridOptimizersContainer.Config(name="Muon"),
                        dataset="text:" + path, val_dataset="text:" + path)
    tr = Trainer(cfg, device=torch.device("cpu"))
    v1 = tr.validate(2)
    tr.train_step(*tr.data.next())
    assert math.isfinite(v1) and tr.validate(2) != v1  # same batches, trained weights


def test_text_stream_reads_a_directory(tmp_path):
    from dion_b200.data import TextStreamLoader, expand_paths

    d = tmp_path / "corpus"
    d.mkdir()
    _docs(d)
    (d / "notes.md").write_text("not an input")
    assert [os.path.basename(p) for p in expand_paths(str(d), (".jsonl",))] == ["docs.jsonl"]
    ld = TextStreamLoader(str(d), "byte", 16, 2)
    t, l = ld.next()
    assert t.shape == (2, 16)
    ld.close()


def test_token_file_info_cli(tmp_path, capsys):
    from dion_b200.data.__main__ import main

    write_token_file(str(tmp_path / "t.bin"), list(b"hello token files"))
    assert main(["info", str(tmp_path / "t.bin"), "--seq-len", "4", "--decode-byte", "5"]) == 0
    out = capsys.readouterr().out
    assert "17 tokens" in out and "3 windows of 5 tokens" in out and "'hello'" in out


def _fsdp_text_body(path, rank, world):
    from dion_b200.integration.hybrid_optimizer import HybridOptimizersContainer
    from dion_b200.integration.trainer import Trainer, TrainerConfig

    cfg = TrainerConfig(model="debug", model_overrides=dict(vocab_size=512), seq_len=32, local_batch_size=2,
                        steps=2, warmup_steps=0, optimizer=HybridOptimizersContainer.Config(name="Dion"),
                        dataset="text:" + path, dp_shard=world, seed=3)
    torch.manual_seed(0)
    tr = Trainer(cfg, device=torch.device("cpu"))
    t, _ = tr.data.next()
    loss = float(tr.train_step(t, _))
    return [loss] + t[0].tolist()


def test_text_stream_under_fsdp_gives_each_rank_its_documents(tmp_path):
    from test_distributed_cpu import spawn

    path = _docs(tmp_path, 100)
    out = spawn(functools.partial(_fsdp_text_body, path), world=2)
    for r, (status, res) in out.items():
        assert status == "ok", res
        assert math.isfinite(res[0])
    # rank 0 starts with document 0, rank 1 with document 1: "[BOS]document 0: ..." / "[BOS]document 1: ..."
    from dion_b200.data.tokenize import ByteTokenizer

    tok = ByteTokenizer()
    assert tok.decode(out[0][1][2:13]) == "document 0:" and tok.decode(out[1][1][2:13]) == "document 1:"
