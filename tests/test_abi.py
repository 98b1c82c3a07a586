"""The C-ABI library loads and exports every symbol include/jalapeno.h
declares; host-side argument checks work without a GPU."""
import ctypes
import re

import pytest

from conftest import REPO, has_gpu

import jalapeno as J


def declared_symbols():
    text = (REPO / "include" / "jalapeno.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(jl_[a-z_0-9]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    names = declared_symbols()
    assert len(names) >= 25
    assert sorted(J.EXPORTS) == names
    lib = ctypes.CDLL(str(J.LIB_PATH))
    for n in names:
        assert hasattr(lib, n), n


def test_version_and_errors():
    assert b"sm_100a" in J.lib.jl_version()
    with pytest.raises(J.JlError) as e:
        J.DraftSchedule.fixed(0)
    assert e.value.status == J.JL_ERR_INVALID_ARG
    assert "gamma" in e.value.message


def test_schedules_validate_like_the_reference():
    # scheduler.rs:9-27
    assert J.DraftSchedule.fixed(5).gamma == 5
    assert J.DraftSchedule.adaptive(4, 5).gamma == 4
    with pytest.raises(J.JlError):
        J.DraftSchedule.adaptive(0, 8)
    with pytest.raises(J.JlError):
        J.DraftSchedule.adaptive(9, 8)


@pytest.mark.skipif(has_gpu(), reason="checks the no-GPU error path")
def test_no_cpu_fallback_without_a_device():
    assert J.device_count() == 0
    with pytest.raises(J.JlError) as e:
        J.Model.synthesize(1, 256, 2, 1, 512, 1000, True, 0)
    assert e.value.status == J.JL_ERR_NO_DEVICE


def test_null_arguments_are_rejected():
    assert J.lib.jl_weights_load(None, None) == J.JL_ERR_INVALID_ARG
    assert J.lib.jl_model_synthesize(None, None, None) == J.JL_ERR_INVALID_ARG
    assert J.lib.jl_cache_truncate(None, 0) == J.JL_ERR_INVALID_ARG


def test_benchmark_prompts_equal_the_oracle_prompts():
    """The package's synthetic prompt generator (the GPU benchmark's inputs)
    gives the ids the oracle's parity tests use."""
    import oracle as O

    for n, vocab, seed in ((1, 10, 0), (20, 1000, 2), (4096, 151936, 3), (33, 8192, 1002), (7, 5, 2**33 + 5)):
        assert J.prompt_ids(n, vocab, seed) == O.prompt_ids(n, vocab, seed)


def test_timeline_is_refused_by_the_normal_build():
    """jl_timeline_read belongs to the diagnostic build (make timeline); the
    normal library answers with an error instead of stamps."""
    if "timeline" in str(J.LIB_PATH):
        pytest.skip("running against the timeline build")
    n = ctypes.c_size_t()
    assert J.lib.jl_timeline_read(None, 0, ctypes.byref(n)) == J.JL_ERR_INVALID_ARG
    assert b"timeline" in J.lib.jl_last_error()
    assert J.lib.jl_timeline_kernel(0) is None
