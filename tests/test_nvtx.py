import torch


def test_nvtx_fn_passthrough():
    from llm_research_b200.utils.nvtx import nvtx_fn, nvtx_range

    @nvtx_fn("lrb/test")
    def f(a, b=2):
        return a + b

    assert f(1) == 3 and f.__name__ == "f"
    with nvtx_range("lrb/test2"):
        x = torch.ones(2)
    assert x.sum() == 2
