"""The experiment manager's config files and command line (reference tests: tests/test_experiments.py): YAML and
JSON bundles load, unknown training options fail before a run folder is made, the best pointer moves only to a better
run, ``compare`` shows only the options that differ and draws its charts, and ``run``/``list``/``compare`` work from
the command line."""

import json
import xml.dom.minidom

import pytest
import yaml

from quantaweave_b200.tools.experiment_manager import compare_runs, load_config, load_summaries, main, run_experiment


def _train_options(tmp_path, **extra):
    data = tmp_path / "d.jsonl"
    if not data.exists():
        data.write_text("".join(json.dumps({"text": f"story {i}: a fox and a dog."}) + "\n" for i in range(40)))
    options = dict(data=[str(data)], examples=40, tokenizer="char", sequence_length=16, hidden_size=16, layers=1,
                   ffn_size=16, attention_heads=2, total_experts=2, active_experts=1, batch_size=2, steps=2,
                   device="cpu", no_power_tracking=True)
    options.update(extra)
    return options


def test_yaml_and_json_bundles_load_to_the_same_config(tmp_path):
    config = {"name": "x", "train": {"steps": 3, "lr": 0.001}, "tags": ["a"], "objective": "train.final_loss"}
    (tmp_path / "c.yaml").write_text(yaml.safe_dump(config))
    (tmp_path / "c.json").write_text(json.dumps(config))
    assert load_config(tmp_path / "c.yaml") == load_config(tmp_path / "c.json") == config


def test_unknown_options_fail_before_a_run_folder_exists(tmp_path):
    with pytest.raises((SystemExit, ValueError, TypeError)):
        run_experiment({"name": "bad", "train": {"not_an_option": 1}}, tmp_path / "runs")
    assert not (tmp_path / "runs").exists() or not any((tmp_path / "runs").iterdir())


def test_the_best_pointer_only_moves_to_a_better_run_and_compare_shows_what_differs(tmp_path):
    runs = tmp_path / "runs"
    first = run_experiment({"name": "a", "train": _train_options(tmp_path, lr=1e-3)}, runs)
    second = run_experiment({"name": "b", "train": _train_options(tmp_path, lr=0.3)}, runs)
    best = json.loads((runs / "best.json").read_text())
    winner = min((first, second), key=lambda s: s["train"]["final_loss"])
    assert best["run_id"] == winner["run_id"] and best["value"] == winner["train"]["final_loss"]
    table = compare_runs(load_summaries([runs / first["run_id"], runs / second["run_id"]]), "train.final_loss")
    header = table.splitlines()[0]
    assert "lr" in header and "hidden_size" not in header  # only the options that differ get a column


def test_the_command_line_runs_lists_and_compares(tmp_path, capsys):
    runs = tmp_path / "runs"
    for name, lr in (("one", 1e-3), ("two", 3e-3)):
        path = tmp_path / f"{name}.yaml"
        path.write_text(yaml.safe_dump({"name": name, "train": _train_options(tmp_path, lr=lr)}))
        main(["run", "--config", str(path), "--runs-dir", str(runs)])
    capsys.readouterr()
    main(["list", "--runs-dir", str(runs)])
    listing = capsys.readouterr().out
    assert "best:" in listing and listing.count("| ") > 2
    dirs = sorted(d for d in runs.iterdir() if d.is_dir())
    main(["compare", *map(str, dirs), "--metric", "train.final_loss", "--markdown", str(tmp_path / "cmp.md"),
          "--charts-dir", str(tmp_path / "charts")])
    assert (tmp_path / "cmp.md").read_text().strip() == capsys.readouterr().out.strip()
    for chart in ("loss_curves.svg", "metric_bars.svg"):
        xml.dom.minidom.parseString((tmp_path / "charts" / chart).read_text())  # well-formed SVG
    main(["compare", *map(str, dirs), "--objectives", "train.final_loss:min", "train.tokens_per_second:max"])
    pareto = capsys.readouterr().out
    assert "pareto-optimal" in pareto.splitlines()[0] and pareto.count("| yes |") >= 1
    bad = tmp_path / "bad.yaml"
    bad.write_text(yaml.safe_dump({"name": "broken", "train": _train_options(tmp_path, data=[str(tmp_path / "no")])}))
    with pytest.raises(SystemExit, match="run failed"):
        main(["run", "--config", str(bad), "--runs-dir", str(runs)])
