"""``tt-atom run`` (tt_atom/cli.py; the reference's tt_atom/cli.py:179-256).

CPU: extended-XYZ round trip, --devices parsing, the report (failed structures make the exit
code 1, the others are written), and the choice between the single-GPU and the fan-out path.
GPU: the command end to end on a tiny bundle, single GPU and fanned out through MultiCardSim,
with a structure that has no edges."""
import numpy as np
import pytest

from tt_atom import cli


def _fcc_xyz(tmp_path, name="fcc.xyz"):
    from tt_atom import configs
    s = configs.fcc_alloy(reps=(2, 2, 2), seed=1)
    p = tmp_path / name
    cli.write_xyz(p, s["Z"], s["pos"], s["cell"], True)
    return p, s


def test_xyz_round_trip(tmp_path):
    p, s = _fcc_xyz(tmp_path)
    a = cli.read_xyz(p)
    assert np.array_equal(a.get_atomic_numbers(), s["Z"])
    assert np.allclose(a.get_positions(), s["pos"], atol=1e-7)
    assert np.allclose(a.get_cell(), s["cell"], atol=1e-7) and a.get_pbc().all()
    q = tmp_path / "mol.xyz"
    q.write_text("3\ncomment\nO 0 0 0\nH 0.96 0 0\n1 -0.24 0.93 0\n")
    m = cli.read_xyz(q)
    assert m.get_atomic_numbers().tolist() == [8, 1, 1] and not m.get_pbc().any()


def test_parse_devices():
    assert cli.parse_devices("0,1, 3") == (0, 1, 3)
    with pytest.raises(SystemExit, match="twice"):
        cli.parse_devices("0,0")
    with pytest.raises(SystemExit, match="comma-separated"):
        cli.parse_devices("a,b")


def test_run_reports_failures_and_writes_the_rest(tmp_path, monkeypatch, capsys):
    p, s = _fcc_xyz(tmp_path)
    calls = {}

    def fake_fan_out(args, structures, devices):
        calls["fan_out"] = devices
        ok = dict(ok=True, energy=-1.5, forces=np.zeros((len(s["Z"]), 3)), pos=s["pos"],
                  Z=s["Z"], nsteps=0)
        return [ok, dict(ok=False, error="ValueError: no edges within cutoff", tb="")]

    monkeypatch.setattr(cli, "_fan_out", fake_fan_out)
    monkeypatch.setattr(cli, "_single_gpu", lambda *a: pytest.fail("single path taken"))
    out = tmp_path / "res"
    rc = cli.main(["run", str(p), str(p), "--devices", "0", "--out", str(out)])
    text = capsys.readouterr().out
    assert rc == 1 and calls["fan_out"] == (0,)
    assert "[1] FAILED: ValueError: no edges within cutoff" in text
    written = out / "fcc_0.xyz"
    assert written.exists() and not (out / "fcc_1.xyz").exists()
    back = cli.read_xyz(written)
    assert np.allclose(back.get_positions(), s["pos"], atol=1e-7)


def test_run_single_structure_takes_the_single_gpu_path(tmp_path, monkeypatch):
    p, _ = _fcc_xyz(tmp_path)
    monkeypatch.setattr(cli, "_fan_out", lambda *a: pytest.fail("fan-out taken"))
    monkeypatch.setattr(cli, "_single_gpu", lambda args, st: [dict(
        ok=True, energy=0.0, forces=np.zeros((len(st[0]), 3)), pos=st[0].get_positions(),
        Z=st[0].get_atomic_numbers())])
    assert cli.main(["run", str(p)]) == 0


@pytest.mark.gpu
def test_run_end_to_end_on_the_gpu(tmp_path, capsys):
    from tt_atom import configs
    from tt_atom.ase_compat import SimpleAtoms
    from tt_atom.calculator import TTAtomCalculator
    from tt_atom.weights import WeightBundle
    cfg = configs.model_config("tiny")
    arrs = configs.random_bundle_arrays(cfg, seed=0)
    bundle = tmp_path / "tiny.npz"
    np.savez(bundle, **arrs)
    m = configs.tiny_molecule(seed=0)
    good = tmp_path / "mol.xyz"
    cli.write_xyz(good, m["Z"], m["pos"])
    lonely = tmp_path / "lonely.xyz"
    lonely.write_text("2\n\nC 0 0 0\nO 20 0 0\n")
    calc = TTAtomCalculator(WeightBundle.from_arrays(arrs))
    a = SimpleAtoms(m["Z"], m["pos"], info=dict(charge=0.0, spin=1.0))   # the CLI defaults
    a.calc = calc
    e_ref = float(a.get_potential_energy())
    # single GPU
    assert cli.main(["run", str(good), "--model", str(bundle), "--out",
                     str(tmp_path / "one.xyz")]) == 0
    assert f"E={e_ref:.6f} eV" in capsys.readouterr().out
    # fanned out over the listed GPUs (one here), with a structure that has no edges
    rc = cli.main(["run", str(good), str(lonely), str(good), "--model", str(bundle),
                   "--devices", "0", "--out", str(tmp_path / "many")])
    text = capsys.readouterr().out
    assert rc == 1
    assert "[1] FAILED: ValueError: no edges within cutoff" in text
    assert text.count(f"E={e_ref:.6f} eV") == 2
    assert (tmp_path / "many" / "mol_0.xyz").exists() and (tmp_path / "many" / "mol_2.xyz").exists()
