"""The Python surface of the MoE path keeps the reference's names, argument order and
defaults (aiter/fused_moe.py:22, 70-80, 118-144, 514-567, 606), so callers switch by
import alone (CPU, no kernel runs)."""
import importlib
import inspect

from aiter_b200 import ActivationType, QuantType

fm = importlib.import_module("aiter_b200.fused_moe")  # the module (the package exports the function)


def test_fused_moe_signature_matches_the_reference():
    params = list(inspect.signature(fm.fused_moe).parameters.values())
    names = [p.name for p in params]
    # the reference's parameters in its order (aiter/fused_moe.py:118-144), then moe_buf
    assert names == ["hidden_states", "w1", "w2", "topk_weight", "topk_ids", "expert_mask", "activation",
                     "quant_type", "doweight_stage1", "w1_scale", "w2_scale", "a1_scale", "a2_scale",
                     "block_size_M", "num_local_tokens", "moe_sorting_dispatch_policy", "dtype", "hidden_pad",
                     "intermediate_pad", "bias1", "bias2", "splitk", "moe_buf"]
    d = {p.name: p.default for p in params}
    assert d["activation"] == ActivationType.Silu and d["quant_type"] == QuantType.No
    assert d["doweight_stage1"] is False and d["moe_sorting_dispatch_policy"] == 0
    assert d["hidden_pad"] == 0 and d["intermediate_pad"] == 0 and d["splitk"] == 0
    assert d["block_size_M"] is None and d["dtype"] is None and d["moe_buf"] is None


def test_moe_sorting_default_block_is_the_references():
    """moe_sorting's default sort unit is the reference module's BLOCK_SIZE_M = 32
    (aiter/fused_moe.py:22,70-80); fused_moe sorts with the GEMM's 128-row tile."""
    sig = inspect.signature(fm.moe_sorting)
    assert list(sig.parameters)[:6] == ["topk_ids", "topk_weights", "num_experts", "model_dim", "moebuf_dtype",
                                        "block_size"]
    assert sig.parameters["block_size"].default == 32 == fm.BLOCK_SIZE_M
    assert fm.GEMM_BLOCK_M == 128


def test_heuristic_helpers():
    assert fm.get_padded_M(1) == 1 and fm.get_padded_M(3) == 4 and fm.get_padded_M(4096) == 4096
    assert fm.get_padded_M(40000) == 32768
    assert fm.get_block_size_M(4096, 8, 128, 1536) == fm.GEMM_BLOCK_M
    assert fm.get_ksplit(1, 8, 128, 1536, 4096) == 0
    # use_nt: the reference's rule, tokens per expert below 64 (aiter/fused_moe.py:531-537)
    fm.use_nt.cache_clear()
    assert fm.use_nt(16, 8, 128) is True and fm.use_nt(4096, 8, 128) is False
    cfg = fm.get_2stage_cfgs(4096, 4096, 1536, 128, 8, None, None, None, QuantType.per_1x128, True,
                             ActivationType.Silu, False)
    assert cfg.block_m == fm.GEMM_BLOCK_M and cfg.ksplit == 0 and cfg.run_1stage is False
