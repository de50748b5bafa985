"""The CUDA lane's keys of crosslane's stage config (clb_lane_config_parse), parsed as
strictly as the reference parses its own (engine/strata/sycl/stage/wiring/common.hpp:55-125):
comments and empty lines skipped; a line without '=', a duplicate or unknown key, a
non-canonical number or an unknown mode is an error. CPU only."""
import pytest

import crosslane_b200 as cb

EXACT, PER_LAYER, TIMING = 1, 2, 4


def test_defaults_are_lane_off():
    c = cb.lane_config_parse("")
    assert c["experts"] == 0 and c["exact_math"] == 0 and c["bytes"] == 0 and c["timing"] == 0
    assert c["device_first"] == 0 and c["device_last"] == 0 and c["bank_flags"] == 0


def test_full_config():
    c = cb.lane_config_parse("# CUDA lane\nwarm_cuda_experts=stack-v1\ncuda_expert_math=cpu-q8k-v1\n\n"
                             "warm_cuda_bytes=137438953472\ncuda_devices=0..7\nwarm_cuda_timing=1\n")
    assert c["experts"] == 2 and c["exact_math"] == 1 and c["bytes"] == 137438953472
    assert (c["device_first"], c["device_last"]) == (0, 7) and c["timing"] == 1
    assert c["bank_flags"] == EXACT | TIMING


def test_layer_batch_mode_selects_per_layer_kernels():
    c = cb.lane_config_parse("warm_cuda_experts=layer-batch-v1\ncuda_devices=3")
    assert c["experts"] == 1 and c["bank_flags"] == PER_LAYER and (c["device_first"], c["device_last"]) == (3, 3)


@pytest.mark.parametrize("text,needle", [
    ("warm_cuda_experts", "without '='"),
    ("warm_cuda_experts=stack-v1\nwarm_cuda_experts=off", "duplicate"),
    ("warm_hip_experts=serial-v1", "unknown lane config key"),
    ("warm_cuda_experts=fast", "unknown warm_cuda_experts"),
    ("warm_cuda_experts=stack-v1\ncuda_expert_math=per32-v1", "unknown cuda_expert_math"),
    ("warm_cuda_experts=stack-v1\nwarm_cuda_bytes=0100", "invalid warm_cuda_bytes"),
    ("warm_cuda_experts=stack-v1\nwarm_cuda_bytes=-1", "invalid warm_cuda_bytes"),
    ("warm_cuda_experts=stack-v1\nwarm_cuda_bytes=18446744073709551616", "invalid warm_cuda_bytes"),
    ("warm_cuda_experts=stack-v1\ncuda_devices=7..0", "cuda_devices"),
    ("warm_cuda_experts=stack-v1\ncuda_devices=0..", "cuda_devices"),
    ("warm_cuda_experts=stack-v1\nwarm_cuda_timing=yes", "warm_cuda_timing"),
    ("cuda_expert_math=cpu-q8k-v1", "need warm_cuda_experts on"),
    ("warm_cuda_experts=off\nwarm_cuda_bytes=1", "need warm_cuda_experts on"),
])
def test_rejects(text, needle):
    with pytest.raises(cb.ClbError) as ei:
        cb.lane_config_parse(text)
    assert ei.value.code == 1 and needle in str(ei.value), str(ei.value)
