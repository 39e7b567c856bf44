"""CPU tests: stores, datasets, sampler, collate functions, preprocessing pipeline."""

import json
import os

import pytest
import torch


def write_bin_dataset(root, seqs, key="sequence", record=False):
    from astrai_b200.serialization import save_bin

    save_bin(os.path.join(root, "shard_0000"), {key: [torch.tensor(s, dtype=torch.int32) for s in seqs]},
             record_keys=[key] if record else None)


def test_window_math_matches_reference_formula(tmpdir_path):
    from astrai_b200.dataset import DatasetFactory

    write_bin_dataset(tmpdir_path, [list(range(100)), list(range(100, 137))])
    ds = DatasetFactory.load("seq", tmpdir_path, window_size=16, stride=10)
    total = 137
    assert len(ds) == (total - 1 - 16) // 10 + 1
    last = ds[len(ds) - 1]
    begin = min((len(ds) - 1) * 10, total - 1 - 16)
    assert last["input_ids"][0].item() == begin
    for i in range(len(ds)):  # crosses the shard boundary without concatenating shards
        s = ds[i]
        assert torch.equal(s["target_ids"][:-1], s["input_ids"][1:])


def test_bin_record_mode_and_detect(tmpdir_path):
    from astrai_b200.dataset import StoreFactory, detect_format

    write_bin_dataset(tmpdir_path, [[1, 2, 3], [4, 5], [6]], key="chosen", record=True)
    assert detect_format(tmpdir_path) == "bin"
    st = StoreFactory.create("bin")
    st.load(tmpdir_path)
    assert st.num_records == 3
    assert st.fetch_record(1, "chosen").tolist() == [4, 5]


def test_sampler_deterministic_resumable_and_sharded():
    from astrai_b200.dataset import RDSampler

    data = list(range(10))
    full = list(RDSampler(data, seed=5))
    assert sorted(full) == data
    assert list(RDSampler(data, seed=5)) == full
    resumed = list(RDSampler(data, seed=5, start_iter=4))
    assert resumed == full[4:]
    s = RDSampler(data, seed=5)
    list(s)
    assert list(s) != full  # next epoch reshuffles (seed + epoch)


def test_collate_functions():
    from astrai_b200.dataset import dpo_collate_fn, grpo_collate_fn

    b = dpo_collate_fn([{"chosen": torch.tensor([1, 2, 3]), "rejected": torch.tensor([4]),
                         "chosen_mask": torch.tensor([0, 1, 1], dtype=torch.bool),
                         "rejected_mask": torch.tensor([1], dtype=torch.bool)}])
    assert b["chosen"].shape == b["rejected"].shape == (1, 3)
    g = grpo_collate_fn([{"prompts": torch.tensor([7, 8]), "responses": [torch.tensor([1]), torch.tensor([2, 3])],
                          "masks": [torch.tensor([True]), torch.tensor([True, True])],
                          "rewards": torch.tensor([0.5, 1.0])},
                         {"prompts": torch.tensor([9]), "responses": [torch.tensor([4, 5, 6]), torch.tensor([7])],
                          "masks": [torch.tensor([True] * 3), torch.tensor([True])],
                          "rewards": torch.tensor([0.0, 1.0])}])
    assert g["prompts"].tolist()[1] == [0, 9] and g["prompt_mask"].tolist()[1] == [False, True]
    assert g["responses"].shape == (2, 2, 3)


def test_preprocess_pipeline_sft_bfd_doc_reset(tokenizer_dir, tmpdir_path):
    from astrai_b200.config.preprocess_config import PipelineConfig
    from astrai_b200.dataset import DatasetFactory
    from astrai_b200.preprocessing import Pipeline

    src = os.path.join(tmpdir_path, "in.jsonl")
    with open(src, "w") as fh:
        for i in range(20):
            fh.write(json.dumps({"messages": [{"role": "user", "content": f"hello {i}"},
                                              {"role": "assistant", "content": "the quick brown fox " * (i % 3 + 1)}]})
                     + "\n")
    cfg = PipelineConfig.from_dict({
        "input": {"sections": [{"field": "messages", "action": "$role", "template": True}]},
        "mask": {"user": "mask", "assistant": "train"},
        "preprocessing": {"packing_strategy": "bfd", "max_packed_len": 64},
        "output": {"position_ids_mode": "doc_reset"},
    })
    out = os.path.join(tmpdir_path, "out")
    stats = Pipeline(cfg, [src], out, tokenizer_dir).run()
    assert stats["records"] == 20
    ds = DatasetFactory.load("sft", out, window_size=32)
    s = ds[0]
    assert set(s) == {"input_ids", "target_ids", "position_ids", "loss_mask"}
    assert s["loss_mask"].any() and not s["loss_mask"].all()
    assert (s["position_ids"] == 0).any()


def test_jsonl_store_default_messages_and_dpo_lazy(tokenizer_dir, tmpdir_path):
    from astrai_b200.dataset import DatasetFactory

    sft_dir = os.path.join(tmpdir_path, "sft")
    os.makedirs(sft_dir)
    with open(os.path.join(sft_dir, "a.jsonl"), "w") as fh:
        for i in range(8):
            fh.write(json.dumps({"messages": [{"role": "user", "content": "q" * 5},
                                              {"role": "assistant", "content": "hello world " * 4}]}) + "\n")
    ds = DatasetFactory.load("sft", sft_dir, window_size=16, tokenizer_path=tokenizer_dir)
    assert len(ds) > 0 and ds[0]["loss_mask"].dtype == torch.bool
    dpo = os.path.join(tmpdir_path, "dpo.jsonl")
    with open(dpo, "w") as fh:
        for i in range(3):
            fh.write(json.dumps({"prompt": "hi", "chosen": "good answer", "rejected": "bad"}) + "\n")
    d = DatasetFactory.load("dpo", dpo, tokenizer_path=tokenizer_dir)
    assert len(d) == 3
    r = d[0]
    assert r["chosen_mask"].any() and not r["chosen_mask"][0]


def test_checkpoint_roundtrip(tmpdir_path):
    from astrai_b200.serialization import Checkpoint

    ck = Checkpoint(state_dict={"w": torch.ones(3)}, epoch=2, consumed_samples=40, extra={"optimizer": {"a": 1}},
                    meta={"x": 1}, config={"hidden_size": 8})
    ck.save(tmpdir_path)
    back = Checkpoint.load_any(tmpdir_path)
    assert back.epoch == 2 and back.consumed_samples == 40 and back.extra["optimizer"] == {"a": 1}
    assert sorted(os.listdir(tmpdir_path)) == ["config.json", "meta.json", "model.safetensors", "optimizer.pt"]
