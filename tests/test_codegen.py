"""The generated CUDA scheme header is current (mirrors the reference's
generator-determinism tests, tests/test_slp.py:58-59 and
tests/test_generate_triton_scheme.py:169-198)."""

from rdna3_fastmm import codegen


def test_generated_header_is_current():
    assert codegen.generate() == codegen.GENERATED_HEADER.read_text()


def test_generated_header_names_every_scheme_side():
    text = codegen.GENERATED_HEADER.read_text()
    for camel in ("Rank7", "Rank48", "Rank49"):
        for side in ("Left", "Right", "Output"):
            assert f"struct {camel}{side} {{" in text


def test_rank48_scalings_are_exact_literals():
    text = codegen.GENERATED_HEADER.read_text()
    assert "vscale(" in text
    assert "0.25f" in text and "0.5f" in text and "2.0f" in text
