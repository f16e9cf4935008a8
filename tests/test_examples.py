"""The example scripts run end to end on CPU at tiny sizes."""

from __future__ import annotations

import importlib.util
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _load(name):
    spec = importlib.util.spec_from_file_location(name, os.path.join(ROOT, "examples", f"{name}.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_basic_usage(capsys):
    _load("basic_usage").main(["--device", "cpu"])
    out = capsys.readouterr().out
    assert "train step: loss=" in out and "params equal=True" in out


@pytest.mark.parametrize("model", ["mac", "mag"])
def test_long_sequence(capsys, model):
    _load("long_sequence").main(["--device", "cpu", "--model", model, "--tokens", "256", "--chunk", "64"])
    out = capsys.readouterr().out
    assert "continuation identical after reload = True" in out
