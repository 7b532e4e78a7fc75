"""The loopback runner (/health, /compile, /run) over the back end: request
validation, the compile cache and the failure replies on CPU; launches on the
GPU (tools/local_runner.py:345-375 is the interface mirrored)."""
from __future__ import annotations

import json
import threading
import urllib.error
import urllib.request

import numpy as np
import pytest

from conftest import GOLDEN, pkg

CASES = GOLDEN / "cases"


def _case_body(name):
    folder = CASES / name
    meta = json.loads((folder / "meta.json").read_text())
    irs = {p.name[:-len(".ir.json")]: json.loads(p.read_text()) for p in sorted(folder.glob("*.ir.json"))}
    return {"meta": meta, "irs": irs}


@pytest.fixture()
def server(tmp_path, request):
    srv = pkg("server")
    device = getattr(request, "param", 0)
    httpd = srv.serve(0, tmp_path / "cache", device)
    thread = threading.Thread(target=httpd.serve_forever, daemon=True)
    thread.start()
    yield f"http://127.0.0.1:{httpd.server_address[1]}"
    httpd.shutdown()
    httpd.server_close()


def _call(url, path, body=None, raw=None):
    data = raw if raw is not None else (None if body is None else json.dumps(body).encode())
    req = urllib.request.Request(url + path, data=data, method="GET" if data is None else "POST",
                                 headers={"Content-Type": "application/json"})
    try:
        with urllib.request.urlopen(req, timeout=120) as reply:
            return reply.status, json.loads(reply.read())
    except urllib.error.HTTPError as err:
        return err.code, json.loads(err.read())


def test_health(server):
    status, body = _call(server, "/health")
    assert status == 200 and body["ok"] and body["can_compile"]
    assert "matmul" in body["families"] and "attention" in body["families"]


def test_compile_recognises_and_caches(server):
    status, first = _call(server, "/compile", _case_body("p01_vector_add-5e973341ada3"))
    assert status == 200 and first["ok"], first
    assert len(first["kernel_id"]) == 64 and [k["kind"] for k in first["kernels"]] == ["pointwise"]
    status, again = _call(server, "/compile", _case_body("p01_vector_add-5e973341ada3"))
    assert again == first


def test_compile_single_ir_field(server):
    body = _case_body("m01_matmul_512-cd9a29496fcc")
    (graph,) = body.pop("irs").values()
    status, reply = _call(server, "/compile", {**body, "ir": graph})
    assert status == 200 and reply["ok"] and reply["kernels"][0]["kind"] == "matmul"


def test_compile_outside_the_families(server):
    status, reply = _call(server, "/compile", _case_body("case-14-f188ef762959"))
    assert status == 200 and not reply["ok"] and reply["stage"] == "compile"
    assert "Unsupported" in reply["stderr"]


def test_pipeline_with_an_unrecognised_kernel(server):
    """attention-0 is recognised kernel by kernel; with its softmax's
    exponentials turned into square roots one kernel matches no family and
    the whole pipeline is refused."""
    body = _case_body("attention-0-9170e7b0641d")
    status, reply = _call(server, "/compile", body)
    assert status == 200 and reply["ok"] and [k["kind"] for k in reply["kernels"]] == ["matmul", "row_softmax",
                                                                                         "matmul"]
    graph = json.dumps(body["irs"]["k_probs_104771"]).replace("ElementwiseImpl('exp')", "ElementwiseImpl('sqrt')")
    body["irs"]["k_probs_104771"] = json.loads(graph)
    status, reply = _call(server, "/compile", body)
    assert status == 200 and not reply["ok"] and reply["stage"] == "compile"


@pytest.mark.parametrize("body, fragment", [
    ({}, "meta"),
    ({"meta": {"kernels": []}, "ir": {}}, "meta"),
    ({"meta": {"kernels": [{"entry": "k", "args": [{"shape": [1 << 27]}]}]}, "ir": {}}, "shape dimension"),
    ({"meta": {"kernels": [{"entry": "k", "args": [{"shape": [1 << 14, 1 << 13]}]}]}, "ir": {}}, "2^26"),
    ({"meta": {"kernels": [{"entry": "not an id", "args": []}]}, "ir": {}}, "entry"),
    ({"meta": {"kernels": [{"entry": "k", "args": []}]}}, "give ir"),
])
def test_compile_rejects_malformed_requests(server, body, fragment):
    status, reply = _call(server, "/compile", body)
    assert status == 422 and reply["stage"] == "request" and fragment in reply["stderr"]


def test_bad_json_and_unknown_paths(server):
    status, reply = _call(server, "/compile", raw=b"{not json")
    assert status == 422 and not reply["ok"]
    assert _call(server, "/nowhere")[0] == 404
    assert _call(server, "/launch", {"x": 1})[0] == 404


@pytest.mark.parametrize("body, fragment", [
    ({"kernel_id": "abc"}, "SHA256"),
    ({"kernel_id": "0" * 64, "iters": 0}, "iters"),
    ({"kernel_id": "0" * 64, "warmup": 21}, "warmup"),
    ({"kernel_id": "0" * 64, "inputs": {"x": {"data": [1], "seed": 2}}}, "exactly one"),
    ({"kernel_id": "0" * 64, "inputs": {"x": {"seed": -1}}}, "seed"),
])
def test_run_rejects_malformed_requests(server, body, fragment):
    status, reply = _call(server, "/run", body)
    assert status == 422 and fragment in reply["stderr"]


def test_run_unknown_kernel(server):
    status, reply = _call(server, "/run", {"kernel_id": "0" * 64})
    assert status == 200 and reply == {"ok": False, "stage": "lookup", "stderr": "unknown kernel_id"}


@pytest.mark.parametrize("server", [99], indirect=True)
def test_run_worker_failure_is_reported(server):
    """A worker that cannot open its device ends with an error; the server answers
    with stage "run" and keeps serving."""
    status, reply = _call(server, "/run", _case_body("p01_vector_add-5e973341ada3"))
    assert status == 200 and not reply["ok"] and reply["stage"] == "run" and reply["stderr"]
    assert _call(server, "/health")[1]["ok"]


# --------------------------------------------------------------------------- GPU
@pytest.mark.gpu
def test_run_given_and_seeded_inputs(server):
    status, compiled = _call(server, "/compile", _case_body("p01_vector_add-5e973341ada3"))
    assert compiled["ok"]
    x0 = np.arange(1024, dtype=np.float32) / 7
    status, reply = _call(server, "/run", {"kernel_id": compiled["kernel_id"], "warmup": 1, "iters": 3,
                                           "inputs": {"x0": {"data": x0.tolist()}, "x1": {"seed": 5}}})
    assert status == 200 and reply["ok"], reply
    x1 = np.random.default_rng(5).standard_normal(1024).astype(np.float32)
    assert reply["outputs"]["add"]["values"] == (x0 + x1).tolist()
    assert reply["median_us"] > 0 and reply["iters"] == 3


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["p01_vector_add-5e973341ada3", "m01_matmul_512-cd9a29496fcc",
                                  "m02_matmul_rect-aeb1568894b7", "f02_row_softmax-89d56c168a0b",
                                  "a01_attention-c10866af73f8", "attention-0-9170e7b0641d"])
def test_compile_then_run_matches_expected(server, name):
    """The runner's success path (tools/local_runner.py:345-375): POST
    /compile, then /run with the case's inputs.npz by kernel_id; the returned
    values equal expected.npz at the case's tolerance and the returned sum is
    the sum of those values (the output summary of local_runner.py:333-342)."""
    oracle = pytest.importorskip("oracle.refs")
    folder = CASES / name
    meta = json.loads((folder / "meta.json").read_text())
    with np.load(folder / "inputs.npz") as data:
        inputs = {k: {"data": data[k].reshape(-1).tolist()} for k in data.files}
    with np.load(folder / "expected.npz") as data:
        expected = {k: data[k] for k in data.files}
    status, compiled = _call(server, "/compile", _case_body(name))
    assert status == 200 and compiled["ok"], compiled
    status, reply = _call(server, "/run", {"kernel_id": compiled["kernel_id"], "inputs": inputs, "warmup": 1,
                                           "iters": 2, "max_return": 1 << 20})
    assert status == 200 and reply["ok"], reply
    for out, want in expected.items():
        summary = reply["outputs"][out]
        got = np.asarray(summary["values"], np.float32).reshape(want.shape)
        assert not summary["truncated"] and summary["shape"] == list(want.shape)
        ok, bad, err = oracle.allclose_report(got, want, meta["rtol"], meta["atol"])
        assert ok, (out, bad, err)
        assert np.isclose(summary["sum"], float(got.astype(np.float64).sum()), rtol=1e-5, atol=1e-3)
