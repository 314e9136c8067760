"""Sampler settings from the front ends (pz_params_*), on the CPU: the
reference's CLI and API defaults and clamps, and the added fields."""
import numpy as np
import pytest


def _f(x):
    return float(np.float32(x))


def test_cli_defaults_and_reference_flags(pz_cpu):
    p = pz_cpu.params_from_args(["prog"])
    assert _f(p.cfg.temperature) == _f(0.7) and _f(p.cfg.top_p) == _f(0.9)      # args.c:82-83
    assert p.seed == -1 and p.cfg.top_k == 0 and p.cfg.repetition_penalty == 1.0
    p = pz_cpu.params_from_args(["prog", "--model", "m.gguf", "--temperature", "0.25", "--top-p", "0.5",
                                 "--seed", "1234", "--threads", "4"])
    assert p.cfg.temperature == 0.25 and p.cfg.top_p == 0.5 and p.seed == 1234


def test_cli_added_flags(pz_cpu):
    p = pz_cpu.params_from_args(["prog", "--top-k", "40", "--repeat-penalty", "1.1", "--frequency-penalty",
                                 "0.2", "--presence-penalty", "0.1", "--top-logprobs", "50"])
    assert p.cfg.top_k == 40 and _f(p.cfg.repetition_penalty) == _f(1.1)
    assert _f(p.cfg.frequency_penalty) == _f(0.2) and _f(p.cfg.presence_penalty) == _f(0.1)
    assert p.logprobs == 1 and p.top_logprobs == 20                                # clamped
    cfg = p.as_config(3)
    assert cfg["top_k"].tolist() == [40, 40, 40]


def test_api_defaults_clamps_and_fields(pz_cpu):
    p = pz_cpu.params_from_json('{"model": "local", "messages": [{"role": "user", "content": "hi {x}"}]}')
    assert p.cfg.temperature == 1.0 and p.cfg.top_p == 1.0 and p.seed == -1        # json_parse.c:299-300
    p = pz_cpu.params_from_json('{"temperature": 3.5, "top_p": 1.5, "stream": true}')
    assert p.cfg.temperature == 2.0 and p.cfg.top_p == 1.0                         # http_server.c:415-417
    p = pz_cpu.params_from_json('{"temperature": -1, "top_p": -0.2}')
    assert p.cfg.temperature == 0.0 and p.cfg.top_p == 1.0
    body = ('{"messages": [{"role": "user", "content": [{"type": "text", "text": "a \\"q\\" b"}]}], '
            '"top_k": 50, "top_p": 0.9, "temperature": 0.7, "frequency_penalty": 3, '
            '"presence_penalty": -0.5, "repetition_penalty": 1.1, "seed": 42, "logprobs": true, '
            '"top_logprobs": 5, "max_tokens": 16}')
    p = pz_cpu.params_from_json(body)
    assert p.cfg.top_k == 50 and _f(p.cfg.top_p) == _f(0.9) and _f(p.cfg.temperature) == _f(0.7)
    assert p.cfg.frequency_penalty == 2.0 and p.cfg.presence_penalty == -0.5
    assert _f(p.cfg.repetition_penalty) == _f(1.1) and p.seed == 42
    assert p.logprobs == 1 and p.top_logprobs == 5
    assert pz_cpu.params_from_json('{"seed": null, "logprobs": false}').seed == -1


def test_api_rejects_what_is_not_an_object(pz_cpu):
    for bad in ("", "[1, 2]", '{"temperature": }', '{"temperature" 1}', '{"a": [1, 2}'):
        with pytest.raises(pz_cpu.PZError):
            pz_cpu.params_from_json(bad)
