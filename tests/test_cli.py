"""CLI parser and dry-run behaviour (restating the reference's tests/test_cli_smoke.py)."""

import pytest

from decodebench_b200.cli import build_parser, main


def test_parsers():
    p = build_parser()
    a = p.parse_args(["demo", "f1", "--dim", "2048", "--batch", "4", "--dry-run"])
    assert (a.command, a.name, a.dim, a.batch, a.dry_run) == ("demo", "f1", 2048, 4, True)
    a = p.parse_args(["profile", "module.py:build_fn", "--trials", "50", "--dry-run"])
    assert (a.command, a.target, a.trials, a.dry_run) == ("profile", "module.py:build_fn", 50, True)
    a = p.parse_args(["sweep", "f4", "--batch", "1,2,4", "--dim", "2048", "--dry-run"])
    assert (a.command, a.name, a.batch, a.dim) == ("sweep", "f4", [1, 2, 4], 2048)
    with pytest.raises(SystemExit):
        p.parse_args(["demo", "invalid_name"])


def test_dry_runs(capsys):
    assert main(["demo", "f1", "--dim", "4096", "--batch", "1", "--dry-run"]) == 0
    assert "[dry-run] demo f1 with dim=4096, batch=1" in capsys.readouterr().out
    assert main(["profile", "user_module.py:build_seq", "--dry-run"]) == 0
    assert "[dry-run] profile target user_module.py:build_seq" in capsys.readouterr().out
    assert main(["sweep", "f2", "--batch", "1,2", "--dim", "4096", "--dry-run"]) == 0
    assert "[dry-run] sweep demo f2 with batch=[1, 2], dim=4096" in capsys.readouterr().out


def test_profile_target_validation(capsys):
    assert main(["profile", "user_module.py"]) == 2
    assert "Error: Target must be in the format 'path/to/module.py:build_fn'" in capsys.readouterr().err


def test_gpu_commands_fail_cleanly_without_gpu(capsys):
    import torch

    if torch.cuda.is_available():
        pytest.skip("has a GPU")
    assert main(["demo", "f1"]) == 1
    assert "GPU/CUDA is not available" in capsys.readouterr().err


def test_layer_demo_is_a_choice(capsys):
    from decodebench_b200.cli import main
    from decodebench_b200.demos.llama_decode import DEMO_NAMES

    assert "layer" in DEMO_NAMES
    assert main(["demo", "layer", "--dry-run"]) == 0
    assert "layer" in capsys.readouterr().out
