"""kv_skill_v2_b200 -- B200-native Library read of xenc (Rickyzhaoweihan/KV_skill_v2).

Public API, mirroring the reference's xenc package for this path:
    Library, PagedLibrary                       (xenc/library.py)
    XEncInjector, LibraryInjector, itf_*        (xenc/injector.py)
    LayerSelector                               (xenc/selector.py)
    TopKLibrary, TopKSelector, TopKLibraryInjector, attach_sel_keys (xenc/topk_read.py, the D8 top-k slot read)
    ModelInterface, LinearInterface, make_interface, EncoderLens, interface_param_groups,
    save_interface, load_interface, count_params (xenc/interface.py)
    DEPTHS, CAND, rho_layer_map, injection_layers, for_reader, KVSkill (xenc/__init__.py, xenc/depth_skill.py)
The compute runs in libxencb.so (include/xencb.h), hand-written CUDA for sm_100a; `ops` exposes one
function per C-ABI entry point.
"""

from .depth import CAND, DEPTHS, DepthCollisionError, KVSkill, for_reader, injection_layers, rho_layer_map
from .injector import ExternalSkillInjector, LibraryInjector, XEncInjector, itf_gain, itf_gate, itf_query, itf_write
from .interface import (EncoderLens, LinearInterface, ModelInterface, count_params, interface_param_groups,
                        load_interface, make_interface, save_interface)
from .library import Library, PagedLibrary
from .selector import LayerSelector
from .topk_read import TopKLibrary, TopKLibraryInjector, TopKSelector, attach_sel_keys

__all__ = ["CAND", "DEPTHS", "DepthCollisionError", "KVSkill", "for_reader", "injection_layers", "rho_layer_map",
           "ExternalSkillInjector", "LibraryInjector", "XEncInjector", "itf_gain", "itf_gate", "itf_query",
           "itf_write", "EncoderLens", "LinearInterface", "ModelInterface", "count_params",
           "interface_param_groups", "load_interface", "make_interface", "save_interface", "Library",
           "PagedLibrary", "LayerSelector", "TopKLibrary", "TopKLibraryInjector", "TopKSelector", "attach_sel_keys"]
