"""The vLLM plugin surface that a user of the reference relies on, without a GPU.

monochromegane/vllm-expert-pager declares the entry point
``[project.entry-points."vllm.general_plugins"] expert_pager =
"vllm_expert_pager.plugin:register"`` (pyproject.toml:24-25) and reads its
settings from ``VLLM_EXPERT_PAGER_*`` variables with fixed defaults
(experts.py:39-72).  Both must be the same here for the package to be a drop-in.
"""

import ast
import os
import tomllib

PKG = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                   "vllm-expert-pager_b200")

# The reference's settings and defaults (experts.py:39-72); None: no default.
REFERENCE_SETTINGS = {
    "VLLM_EXPERT_PAGER_CACHE_SLOTS": "32",
    "VLLM_EXPERT_PAGER_RAM_SLOTS": None,
    "VLLM_EXPERT_PAGER_SSD_PATH": None,
    "VLLM_EXPERT_PAGER_COMPRESS": "auto",
    "VLLM_EXPERT_PAGER_PITCH": "0.89",
    "VLLM_EXPERT_PAGER_WORKING_ROWS": "64",
    "VLLM_EXPERT_PAGER_LOG_INTERVAL": "1000",
}


def test_entry_point_is_the_references():
    with open(os.path.join(PKG, "pyproject.toml"), "rb") as f:
        meta = tomllib.load(f)
    eps = meta["project"]["entry-points"]["vllm.general_plugins"]
    assert eps == {"expert_pager": "vllm_expert_pager.plugin:register"}
    assert meta["project"]["name"] == "vllm-expert-pager"


def test_register_is_a_function_of_the_plugin_module():
    tree = ast.parse(open(os.path.join(PKG, "vllm_expert_pager", "plugin.py")).read())
    funcs = [n.name for n in tree.body if isinstance(n, ast.FunctionDef)]
    assert "register" in funcs


def test_settings_and_defaults_are_the_references():
    # Read os.environ.get("VLLM_EXPERT_PAGER_...", default) calls from experts.py
    # without importing it (it needs a vLLM with RoutedExperts).
    tree = ast.parse(open(os.path.join(PKG, "vllm_expert_pager", "experts.py")).read())
    found = {}
    for node in ast.walk(tree):
        if (isinstance(node, ast.Call) and isinstance(node.func, ast.Attribute)
                and node.func.attr == "get" and node.args
                and isinstance(node.args[0], ast.Constant)
                and str(node.args[0].value).startswith("VLLM_EXPERT_PAGER_")):
            default = node.args[1].value if len(node.args) > 1 else None
            found[node.args[0].value] = default
    for name, default in REFERENCE_SETTINGS.items():
        assert name in found, name
        assert found[name] == default, (name, found[name], default)
