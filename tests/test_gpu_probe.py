"""The latency probes (tans_probe) run on the GPU and give cycles per step in their plausible
ranges: a shared-memory load tens of cycles, an L2 load a few hundred, one step of the rANS
arithmetic chains between the two."""
import pytest

pytestmark = pytest.mark.gpu

RANGES = {"smem_chase": (10, 120), "l2_chase": (100, 1500), "l2_chase_busy": (100, 3000),
          "pop32_step": (20, 600), "push32_step": (10, 600), "pop64_step": (20, 600), "push64_step": (10, 600)}


@pytest.mark.parametrize("kind", sorted(RANGES))
def test_probe_runs_and_is_plausible(kind):
    from torch_ans_b200 import capi
    steps = {"l2_chase": 1 << 14, "l2_chase_busy": 1 << 12}.get(kind, 1 << 16)
    c = capi.probe(kind, steps)
    lo, hi = RANGES[kind]
    assert lo <= c <= hi, (kind, c)
