"""Service plugin contract and per-process output logs (CPU only).

Mirrors the reference's plugin and logging checks (``tests/test_service_plugin.py``,
``tests/test_service_logging.py``):

* a ``ServiceConfig`` subclass that names its implementation resolves without a registry entry; GPU and CPU
  plugins enter the generic topology with ports from their declared bases;
* a GPU plugin without port bases, two colocated plugins with the same port bases, and a plugin with neither
  an implementation nor a known role are refused with a clear message;
* ``redirect_output`` sends a role's stdout and stderr (Python and native writes alike) to its log file.
"""

import subprocess
import sys
import textwrap
from dataclasses import dataclass
from pathlib import Path
from typing import ClassVar

import pytest

from meshy_b200.config import ServiceConfig
from meshy_b200.service.base import GPU, Service, ServiceGroup
from meshy_b200.service.registry import resolve_service
from meshy_b200.service.runtime import RuntimeDir
from meshy_b200.service.topology import build_topology


@dataclass
class CustomGPUConfig(ServiceConfig):
    role: ClassVar[str] = "custom_gpu"
    service_cls: ClassVar[str] = "meshy_b200.service.base:Service"
    endpoint_port_base: ClassVar[int] = 33500
    dist_port_base: ClassVar[int] = 43500


@dataclass
class CustomCPUConfig(ServiceConfig):
    role: ClassVar[str] = "custom_cpu"
    service_cls: ClassVar[str] = "meshy_b200.service.base:Service"
    uses_gpu: ClassVar[bool] = False


def _gpus(n=1):
    return [GPU(global_rank=i, host="127.0.0.1", local_rank=i) for i in range(n)]


def test_custom_service_resolves_without_registry_entry():
    assert resolve_service(CustomGPUConfig()) is Service


def test_custom_gpu_and_cpu_services_enter_generic_topology():
    topo = build_topology([
        ServiceGroup("compute", 2, 1, CustomGPUConfig()),
        ServiceGroup("driver", 1, 0, CustomCPUConfig()),
    ], _gpus(2))
    assert topo.by_name("compute-0").endpoint_port == 33500
    assert topo.by_name("compute-1").dist_port == 43501  # base + the replica's first global rank
    assert [s.name for s in topo.gpu_services()] == ["compute-0", "compute-1"]
    assert [s.name for s in topo.cpu_services()] == ["driver-0"]
    assert topo.services_by_role("custom_cpu")[0].name == "driver-0"


def test_custom_gpu_service_must_declare_port_bases():
    @dataclass
    class MissingPortsConfig(ServiceConfig):
        role: ClassVar[str] = "missing_ports"
        service_cls: ClassVar[str] = "meshy_b200.service.base:Service"

    with pytest.raises(ValueError, match="must declare endpoint_port_base"):
        build_topology([ServiceGroup("broken", 1, 1, MissingPortsConfig())], _gpus())


def test_colocated_custom_services_must_use_distinct_port_bases():
    @dataclass
    class CollidingConfig(ServiceConfig):
        role: ClassVar[str] = "colliding"
        service_cls: ClassVar[str] = "meshy_b200.service.base:Service"
        endpoint_port_base: ClassVar[int] = 33500
        dist_port_base: ClassVar[int] = 43500

    with pytest.raises(ValueError, match="collision"):
        build_topology([
            ServiceGroup("first", 1, 1, CustomGPUConfig()),
            ServiceGroup("second", 1, 1, CollidingConfig(), colocate_with="first"),
        ], _gpus())


def test_service_config_must_declare_implementation():
    @dataclass
    class MissingImplementationConfig(ServiceConfig):
        role: ClassVar[str] = "missing_implementation"

    with pytest.raises(ValueError, match="declares no service_cls"):
        resolve_service(MissingImplementationConfig())


def test_role_output_is_redirected_to_runtime_log(tmp_path):
    log_path = Path(RuntimeDir(str(tmp_path)).process_log_path("training-0", 2))
    assert log_path.name == "training-0-2.log"
    child = textwrap.dedent(f"""
        import os, sys
        from meshy_b200.service.base import redirect_output

        redirect_output({str(log_path)!r})
        print("stdout from role")
        print("stderr from role", file=sys.stderr)
        os.write(1, b"native write to fd 1\\n")
        os.system("echo from a child process")
    """)
    res = subprocess.run([sys.executable, "-c", child], check=True, capture_output=True,
                         cwd=str(Path(__file__).resolve().parents[1]))
    assert res.stdout == b"" and res.stderr == b""
    text = log_path.read_text()
    for line in ("stdout from role", "stderr from role", "native write to fd 1", "from a child process"):
        assert line in text, text
