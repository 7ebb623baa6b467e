"""Host-side checks of the per-launch timing probe (no GPU: CUDA events are
created lazily and never recorded here)."""
import pytest

from kvm_b200.timing import PhaseProbe


def test_probe_needs_start_first():
    with pytest.raises(ValueError):
        PhaseProbe(1, ["router", "start"])
    with pytest.raises(ValueError):
        PhaseProbe(1, [])


def test_probe_rejects_marks_out_of_order():
    p = PhaseProbe(2, ["start", "a", "b"]).next_call()
    with pytest.raises(RuntimeError):
        p.mark("a")            # "start" is due first
    with pytest.raises(RuntimeError):
        p.mark("b")


def test_layer_phase_lists_are_probe_ready():
    from kvm_b200.moe import MoELayer
    from kvm_b200.ep import ExpertParallelMoE
    for phases in (MoELayer.PHASES, ExpertParallelMoE.PHASES_SERIAL,
                   ExpertParallelMoE.PHASES_OVERLAP):
        assert phases[0] == "start" and len(set(phases)) == len(phases)
        PhaseProbe(1, phases)
