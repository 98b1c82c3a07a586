"""A/B benchmark, tensor-core side: the library's MXFP4 projections
(k_mx_gemv, tcgen05 block-scaled MMA) on Qwen3-8B shapes at 1, 5 and 8
rows, timed through jl_time_projection (back-to-back launches on the
model's stream, CUDA events).  The CUDA-core side is cuda_core_projection.cu
in this folder; both print microseconds per launch and weight GB/s.

Run (B200, after `make -C jalapenos-at-home_b200`):
    python jalapenos-at-home_b200/ab/tensor_core_projection.py
"""
import pathlib
import sys

sys.path.insert(0, str(pathlib.Path(__file__).resolve().parents[1]))
import jalapeno as J  # noqa: E402


def main() -> None:
    # two Qwen3-8B layers (hidden 4096, 32/8 heads, inter 12288) and a short
    # vocabulary: only layer 0's projections are timed
    m = J.Model.synthesize(layers=2, hidden=4096, q_heads=32, kv_heads=8, inter=12288, vocab=8192,
                           tied=False, seed=0, mxfp4=True, kv_pool_tokens=1024, max_pass_rows=64)
    m.predict([(7 * i + 3) % 8192 for i in range(32)], m.cache())
    for rows in (1, 5, 8):
        for name, which in (("gate/up", J.PROJ_GATE_UP), ("down", J.PROJ_DOWN), ("qkv", J.PROJ_QKV),
                            ("o", J.PROJ_O)):
            ms, nb = m.time_projection(0, which, rows, iters=50)
            print(f"tensor-core k_mx_gemv rows={rows} {name}: {ms * 1000:.2f} us/launch, "
                  f"{nb / ms / 1e6:.0f} GB/s", flush=True)


if __name__ == "__main__":
    main()
