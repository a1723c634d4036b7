"""The reference's import name: code written for ``wbridge`` imports and runs on this library."""
import sys


def test_reference_import_names_resolve_to_this_library():
    import weightbridge_b200 as wb
    import wbridge
    from wbridge import (WeightData, WeightReceiver, WeightReceiverController, WeightSender,  # noqa: F401
                         dtype_str_to_torch, dtype_to_str)
    from wbridge.frontend import WeightSender as FrontSender
    from wbridge.utils.data import _check_shard_compatibility, original_total_numel, shards_iterator  # noqa: F401
    from wbridge.utils.megatron_utils import convert_to_wb as meg_convert
    from wbridge.utils.sglang_utils import convert_to_wb as sgl_convert
    assert WeightSender is wb.WeightSender and FrontSender is wb.WeightSender
    assert WeightData is wb.WeightData and wbridge.utils.data.WeightData is wb.WeightData
    assert callable(meg_convert) and callable(sgl_convert)
    assert "wbridge.utils.data" in sys.modules


def test_reference_test_contract_through_wbridge_names():
    """The reference's own test cases, written against ``wbridge`` (pair-form alignment, single
    shard overlap form, JSON round trip)."""
    from wbridge import WeightData
    from wbridge.utils.data import _check_shard_compatibility
    assert _check_shard_compatibility([(0, 24, 24)], [(0, 4, 4), (0, 6, 6)]) == ([(0, 4, 4), (0, 6, 6)],
                                                                                  [(0, 4, 4), (0, 6, 6)])
    assert _check_shard_compatibility([(0, 4, 4), (0, 6, 6)], [(0, 6, 6), (0, 4, 4)]) is None
    s = WeightData({"w": {"shard": [(0, 4, 4), (0, 6, 6)], "dtype": "float32"}})
    r = WeightData({"w": {"shard": [(2, 3, 4), (2, 5, 6)], "dtype": "float32"}})
    ov = WeightData.compute_overlap(s, r)
    assert ov["w"]["shard"] == [(2, 3, 4), (2, 5, 6)]
    assert WeightData(str(ov)).to_jsonable() == ov.to_jsonable()
