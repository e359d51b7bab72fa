"""The cuda_<variant> plugin slot mirrors the reference registry API (CPU-only checks)."""

from __future__ import annotations

import pytest

from linattn_b200 import AttnConfig, KERNEL_VARIANTS, build, describe_kernel, list_kernel_variants


def test_kernel_variant_names():
    assert "cuda_quest" in KERNEL_VARIANTS and KERNEL_VARIANTS["cuda_quest"] == "quest"
    assert list_kernel_variants() == list(KERNEL_VARIANTS)


def test_build_reads_reference_config_keys():
    cfg = AttnConfig(n_heads=8, n_kv_heads=2, head_dim=64, block_size=16, topk_blocks=5,
                     extras={"page_size": 32, "gqa_union": False, "dense_layers": 0, "layer_idx": 1})
    var = build("cuda_quest", cfg)
    assert var.page_size == 32 and var.gqa_union is False and var.dense_layers == 0 and var.layer_idx == 1
    assert var.read_budget(4096) == min(4096, 5 * 16 + cfg.window_size)
    assert var.flops(1024) > 0


def test_unknown_names_raise_keyerror():
    with pytest.raises(KeyError):
        build("cuda_nonexistent")
    with pytest.raises(KeyError):
        describe_kernel("mlx_quest")


def test_describe_kernel():
    meta = describe_kernel("cuda_quest")
    assert meta["reference"] == "quest" and meta["family"] == "cuda"


def test_bad_gqa_config_rejected():
    with pytest.raises(ValueError):
        build("cuda_quest", AttnConfig(n_heads=6, n_kv_heads=4))
