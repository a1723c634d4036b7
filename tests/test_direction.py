"""Which side runs the copy program of a gpu_direct session."""
from weightbridge_b200 import TransferConfig
from weightbridge_b200.control.sender import session_direction
from weightbridge_b200.models.arch import get_arch
from weightbridge_b200.parallel.sglang import SGLangLayout


def _meta(quant=None):
    lay = SGLangLayout(get_arch("tiny-qwen3-moe"), tp=1, quant=quant)
    return lay.to_wb(lay.allocate(device="meta"))[0]


def test_pull_by_default_push_with_fp8_workers_or_when_asked():
    plain, fp8 = _meta(), _meta("fp8_experts")
    assert TransferConfig().direction == "pull"
    assert session_direction(TransferConfig(), [plain, plain]) == "pull"
    assert session_direction(TransferConfig(), [plain, fp8]) == "push"          # a worker quantises
    assert session_direction(TransferConfig(direction="push"), [plain]) == "push"
    for mode in ("nvls", "nccl", "cpu_direct"):                                  # stores by nature
        assert session_direction(TransferConfig(mode=mode), [plain]) == "push"
