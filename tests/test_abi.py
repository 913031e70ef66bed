"""The C-ABI library loads and exports every entry point include/lora_ce.h
declares; host-side argument checks fail cleanly.  No GPU needed."""
import ctypes as C
import os
import re

import numpy as np
import pytest

import lora_ce

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    src = open(os.path.join(REPO, "include", "lora_ce.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(lora_ce_\w+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = lora_ce.load_library()
    names = header_functions()
    assert len(names) >= 16
    for n in names:
        assert hasattr(lib, n), n
    assert sorted(lora_ce.EXPORTS) == names


def test_default_config_is_reference_defaults():
    cfg = lora_ce.default_config(576, 49152, 8, 256)
    assert (cfg.dim, cfg.vocab, cfg.rank, cfg.max_tokens) == (576, 49152, 8, 256)
    assert cfg.scale == 2.0  # alpha 16 / rank 8 (cmd_train)
    assert np.float32(cfg.lr) == np.float32(1e-4)
    assert np.float32(cfg.beta1) == np.float32(0.9) and np.float32(cfg.beta2) == np.float32(0.999)
    assert np.float32(cfg.eps) == np.float32(1e-8)
    assert cfg.weight_decay == 0.0 and cfg.clip_norm == 0.0


@pytest.mark.parametrize("field,value", [("dim", 100), ("rank", 257), ("rank", 0), ("max_tokens", 0),
                                         ("vocab", 0), ("beta1", 1.0)])
def test_create_rejects_bad_config(field, value):
    cfg = lora_ce.default_config(576, 49152, 4, 256)
    setattr(cfg, field, value)
    with pytest.raises(lora_ce.LoraCEError, match="EINVAL"):
        lora_ce.LoraCE(cfg)


def test_null_arguments_fail_cleanly():
    lib = lora_ce.load_library()
    assert lib.lora_ce_create(None, None) == -1
    assert lib.lora_ce_step(None, None, 0, 1, None, None) == -1
    assert lib.lora_ce_destroy(None) == 0
    assert lib.lora_ce_nccl_unique_id(None) == -1
    assert lib.lora_ce_last_error()  # message set


def test_body_library_exports_every_declared_symbol():
    src = open(os.path.join(REPO, "include", "lora_body.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = sorted(set(re.findall(r"\b(lora_body_\w+)\s*\(", src)))
    lib = lora_ce.load_library()
    for n in names:
        assert hasattr(lib, n), n
    assert sorted(lora_ce.BODY_EXPORTS) == names


def test_body_create_rejects_bad_config():
    lib = lora_ce.load_library()
    assert lib.lora_body_create(None, None) == -1
    for kw in (dict(dim=100), dict(n_heads=8), dict(max_seq=0), dict(n_kv_heads=2)):
        args = dict(n_layers=2, dim=576, n_heads=9, n_kv_heads=3)
        args.update(kw)
        with pytest.raises(lora_ce.LoraCEError, match="EINVAL"):
            lora_ce.LoraBody(**args)
