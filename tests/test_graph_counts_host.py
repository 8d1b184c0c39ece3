"""Host logic of layer.graph_kernel_counts, against a fake of the CUDA driver bindings.

The bench's ``gpu_launches`` for the layer workloads comes from this count: the kernel
nodes of a captured step graph, and among them this library's (names mangled in
namespace ``moe``).  Any failed driver call must give None, never a partial count.
"""
import sys
import types

import pytest

from moe_overlap_b200.layer import graph_kernel_counts

KERNEL, MEMSET = 0, 2


def _fake_driver(nodes, fail=None):
    """nodes: list of (type, func handle, mangled name)."""
    cu = types.SimpleNamespace()
    ok, bad = "ok", "bad"
    cu.CUresult = types.SimpleNamespace(CUDA_SUCCESS=ok)
    cu.CUgraphNodeType = types.SimpleNamespace(CU_GRAPH_NODE_TYPE_KERNEL=KERNEL)
    cu.CUgraph = lambda raw: ("graph", raw)
    by_func = {func: name for _, func, name in nodes}

    def get_nodes(g, n):
        assert g == ("graph", 1234)
        if n == 0:
            return ok, None, len(nodes)
        return ok, list(range(len(nodes))), len(nodes)

    def node_type(i):
        return (bad, None) if fail == "type" else (ok, nodes[i][0])

    def params(i):
        return ok, types.SimpleNamespace(func=nodes[i][1])

    def func_name(func):
        return (bad, None) if fail == "name" else (ok, by_func[func])

    cu.cuGraphGetNodes = get_nodes
    cu.cuGraphNodeGetType = node_type
    cu.cuGraphKernelNodeGetParams = params
    cu.cuFuncGetName = func_name
    return cu


class _Graph:
    def raw_cuda_graph(self):
        return 1234


@pytest.fixture
def install(monkeypatch):
    def _install(cu):
        pkg = types.ModuleType("cuda.bindings")
        pkg.driver = cu
        monkeypatch.setitem(sys.modules, "cuda.bindings", pkg)
        monkeypatch.setitem(sys.modules, "cuda.bindings.driver", cu)
    return _install


NODES = [
    (KERNEL, 11, b"_ZN3moe2gg4pair24grouped_gemm_pair_kernelILb1ELb1ELb0EEEvNS0_6ParamsE"),
    (MEMSET, 0, b""),
    (KERNEL, 12, b"_ZN2at6native29vectorized_elementwise_kernelILi4EEEvv"),
    (KERNEL, 13, b"_ZN3moe2ep12pull_kernelILi4ELi2EEEvNS0_6ParamsE"),
    (KERNEL, 14, b"_ZN3moe12_GLOBAL__N_121expert_offsets_kernelEPKviii"),
]


def test_counts_kernel_nodes_and_this_librarys_by_name(install):
    install(_fake_driver(NODES))
    assert graph_kernel_counts(_Graph()) == {"total": 4, "ours": 3}


@pytest.mark.parametrize("fail", ["type", "name"])
def test_a_failed_driver_call_gives_no_count(install, fail):
    install(_fake_driver(NODES, fail=fail))
    assert graph_kernel_counts(_Graph()) is None


def test_a_kernel_node_without_a_function_handle_gives_no_count(install):
    install(_fake_driver([(KERNEL, 0, b"")]))
    assert graph_kernel_counts(_Graph()) is None


def test_a_graph_without_a_raw_handle_gives_no_count(install):
    install(_fake_driver(NODES))
    assert graph_kernel_counts(object()) is None
