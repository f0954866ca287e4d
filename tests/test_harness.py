"""Host-only regressions of the harness mirror, in the style of the
reference's tests/test_external_ascendc.py and tests/test_kernel_names.py:
registry and external-driver contracts, profiler kernel-name matching, the
bench's prepare -> inputs -> adapt order and compile-phase selection, and the
B200 backends' declarations and argument checks."""

import unittest
from types import SimpleNamespace
from unittest.mock import Mock, patch

import torch

from fa_b200.core import profiler, registry
from fa_b200.core.drivers import external


class ExternalTests(unittest.TestCase):
    def test_registration_and_precompile_selection(self):
        prebuilt = SimpleNamespace(META=SimpleNamespace(type="external"))
        source = SimpleNamespace(META=prebuilt.META, build=Mock())
        self.assertIs(registry.driver_for(prebuilt.META), external)
        self.assertFalse(registry.needs_compile(prebuilt))
        self.assertTrue(registry.needs_compile(source))

    def test_unknown_types_are_rejected(self):
        for kind in ("torch", "tilelang", "ascendc"):
            with self.assertRaises(KeyError):
                registry.driver_for(SimpleNamespace(type=kind))

    def test_optional_build_and_opaque_argument_object(self):
        args = {"q": "tensor", "custom": 123}
        spec = SimpleNamespace(adapt=Mock(return_value=args), call=Mock(return_value="out"))
        external.compile(spec, "case")
        call = external.make_call(spec, "case", "canonical")
        spec.adapt.assert_called_once_with("case", "canonical")
        self.assertEqual(call(), "out")
        self.assertEqual(call(), "out")
        spec.call.assert_called_with(args)
        spec.build = Mock()
        external.compile(spec, "case")
        external.make_call(spec, "case", "canonical")
        self.assertEqual(spec.build.call_count, 2)
        spec.build = "not callable"
        with self.assertRaises(TypeError):
            external.compile(spec, "case")

    def test_generic_prepare_defers_adaptation_until_inputs_exist(self):
        spec = SimpleNamespace(META=SimpleNamespace(type="external"), adapt=Mock(return_value="args"),
                               call=Mock(return_value="out"))
        bind = registry.prepare_call(spec, "case")
        spec.adapt.assert_not_called()
        call = bind("canonical")
        spec.adapt.assert_called_once_with("case", "canonical")
        self.assertEqual(call(), "out")

    def test_bench_prepares_backends_before_inputs(self):
        from fa_b200.core import bench
        from fa_b200.problem import canonical

        events = []
        spec = SimpleNamespace(META=SimpleNamespace(type="external", op_type="Test", is_reference=True))

        def prepare(spec, case):
            events.append("load")

            def bind(inputs):
                events.append("adapt")
                return lambda: None

            return bind

        def inputs(case, seed):
            events.append("inputs")
            return {}

        with (
            patch.object(registry, "get", return_value=spec),
            patch.object(registry, "prepare_call", side_effect=prepare),
            patch.object(canonical, "build_canonical", side_effect=inputs),
            patch.object(bench.torch.cuda, "synchronize", Mock()),
            patch.object(bench.profiler, "profile_case_us", return_value={"test": 1.0}),
            patch.dict("os.environ"),
        ):
            bench.process_case(0, 0, session_dir="unused", backend_names=["test"], ref_name="test",
                               iters=1, do_check=False, seed=0, atol=0, rtol=0)
        self.assertEqual(events, ["load", "inputs", "adapt"])

    def test_bench_selects_only_backends_with_a_build_hook(self):
        from fa_b200.core import bench

        specs = {name: SimpleNamespace(META=SimpleNamespace(type="external"))
                 for name in ("prebuilt", "source", "torch_op")}
        specs["source"].build = Mock()
        seen = []

        def collect(tasks, worker):
            seen.extend(tasks)
            return []

        with (
            patch.object(registry, "_BACKENDS", specs),
            patch.object(bench.schedule, "parallel_compile", side_effect=collect),
        ):
            bench.compile_phase(list(specs), [0, 1])
        self.assertEqual(seen, [("source", 0), ("source", 1)])

    def test_check_output_applies_both_bars(self):
        from fa_b200.core.bench import check_output

        ref = torch.zeros(4, 8)
        self.assertEqual(check_output(ref + 1e-4, ref, 1e-2, 1e-2, 2e-3, 2e-4)[0], "PASS")
        self.assertEqual(check_output(ref + 1e-3, ref, 1e-2, 1e-2, 2e-3, 2e-4)[0], "FAIL")  # mean bar
        bad = ref.clone()
        bad[0, 0] = 5e-3
        self.assertEqual(check_output(bad, ref, 1e-2, 1e-2, 2e-3, 2e-4)[0], "FAIL")  # max bar
        bad[0, 0] = 0.5
        self.assertEqual(check_output(bad, ref, 1e-2, 1e-2, 1.0, 1.0)[0], "FAIL")  # legacy assert_close


class RegistryTests(unittest.TestCase):
    def test_discovery_finds_the_b200_backends_and_one_reference(self):
        names = registry.all_names()
        for n in ("b200_fa_fp16", "b200_fa_fp32", "torch_fp32_ref"):
            self.assertIn(n, names)
        ref, mod = registry.get_reference()
        self.assertEqual(ref, "torch_fp32_ref")
        self.assertTrue(mod.META.is_reference)
        self.assertEqual(registry.name_of(registry.get("b200_fa_fp16")), "b200_fa_fp16")

    def test_vendor_attention_backend_is_discovered_and_expands_kv_heads(self):
        from fa_b200.problem.cases import CASES

        spec = registry.get("torch_sdpa")
        self.assertFalse(spec.META.is_reference)
        self.assertEqual(spec.META.type, "external")
        case = CASES[3]  # Hq = 12, Hkv = 1
        k = torch.arange(2 * 8 * 128, dtype=torch.float16).reshape(1, 2, 8, 128)[:, :1]
        args = spec.adapt(case, {"q": torch.zeros(1, 12, 8, 128, dtype=torch.float16), "k": k, "v": k + 1})
        self.assertEqual(tuple(args["k"].shape), (1, 12, 8, 128))
        for h in range(12):
            self.assertTrue(torch.equal(args["k"][0, h], k[0, 0]))
            self.assertTrue(torch.equal(args["v"][0, h], k[0, 0] + 1))
        self.assertEqual(args["scale"], case.scale)

    def test_registry_rejects_unregistered_or_ambiguous_module(self):
        spec = SimpleNamespace(META=SimpleNamespace(is_reference=False))
        for registered in ({}, {"one": spec, "two": spec}):
            with patch.object(registry, "_BACKENDS", registered):
                with self.assertRaises(ValueError):
                    registry.name_of(spec)

    def test_reference_must_be_unique(self):
        ref = SimpleNamespace(META=SimpleNamespace(is_reference=True))
        with patch.object(registry, "_BACKENDS", {"a": ref, "b": ref}):
            with self.assertRaises(ValueError):
                registry.get_reference()

    def test_diagnostic_backends_are_excluded(self):
        diag = SimpleNamespace(META=SimpleNamespace(diagnostic=True))
        with patch.object(registry, "_BACKENDS", {"diag": diag}):
            self.assertEqual(registry.all_names(), [])
            with self.assertRaises(ValueError):
                registry.require_attention(diag)

    def test_b200_backends_declare_kernel_symbols_containing_their_names(self):
        from fa_b200 import lib

        for name, variant in (("b200_fa_fp16", lib.VARIANT_FP16), ("b200_fa_fp32", lib.VARIANT_FP32)):
            spec = registry.get(name)
            self.assertEqual(spec.META.type, "external")
            self.assertTrue(callable(spec.build))
            self.assertIn(name, lib.kernel_name(variant))
            self.assertIn(name, spec.META.op_type)


class ProfileNameTests(unittest.TestCase):
    def test_exact_symbols_disambiguate_prefixes_without_legacy_fallback(self):
        names = ["tl_stream", "tl_stream_v3", "torch_fp32_ref"]
        symbols = {n: f"{n}_kernel" for n in names[:2]}
        op_types = {n: "main_kernel" for n in names[:2]}
        op_types["torch_fp32_ref"] = "torch_fp32_ref"
        expected = {
            "tl_stream_kernel": "tl_stream",
            "tl_stream_v3_kernel": "tl_stream_v3",
            "main_kernel": None,
            "tl_stream_v30_kernel": None,
            "prefix_tl_stream_v3_kernel": None,
        }
        for symbol, backend in expected.items():
            with self.subTest(symbol=symbol):
                self.assertEqual(profiler._match_backend(symbol, names, op_types, symbols), backend)

    def test_b200_kernels_match_their_backends_by_substring(self):
        names = ["b200_fa_fp16", "b200_fa_fp32", "torch_fp32_ref"]
        op_types = {n: registry.get(n).META.op_type for n in names}
        for kernel, backend in (("b200_fa_fp16_kernel", "b200_fa_fp16"),
                                ("b200_fa_fp32_kernel", "b200_fa_fp32"),
                                ("ampere_sgemm_128x64_nn", None)):
            name = profiler._kernel_base_name(kernel + "(b200fa::FwdParams)")
            self.assertEqual(profiler._match_backend(name, names, op_types, {}), backend)


class OperatorArgumentTests(unittest.TestCase):
    """The operator rejects bad arguments like the reference binding (binding.py:219-231)."""

    def setUp(self):
        from fa_b200.ops import Operator

        self.op = Operator("fp16")
        self.q = torch.zeros(1, 2, 256, 128, dtype=torch.float16)
        self.k = torch.zeros(1, 1, 256, 128, dtype=torch.float16)

    def test_rank_and_shape(self):
        with self.assertRaisesRegex(ValueError, r"Q/K/V must be \[B,H,N,128\]"):
            self.op(self.q[0], self.k, self.k)
        with self.assertRaisesRegex(ValueError, r"Q/K/V must be \[B,H,N,128\]"):
            self.op(self.q, self.k, self.k[:, :, :128])

    def test_geometry(self):
        with self.assertRaisesRegex(ValueError, "invalid attention geometry"):
            self.op(self.q[..., :64], self.k[..., :64], self.k[..., :64])
        with self.assertRaisesRegex(ValueError, "invalid attention geometry"):
            k3 = torch.zeros(1, 3, 256, 128, dtype=torch.float16)
            self.op(self.q, k3, k3)
        with self.assertRaisesRegex(ValueError, "invalid attention geometry"):
            self.op(self.q[:, :, :0], self.k, self.k)

    def test_device_and_dtype(self):
        with self.assertRaisesRegex(ValueError, "contiguous FP16 on the same CUDA device"):
            self.op(self.q, self.k, self.k)  # CPU tensors: no CPU fallback
        with self.assertRaisesRegex(ValueError, "contiguous FP16"):
            self.op(self.q.float(), self.k.float(), self.k.float())

    def test_unknown_variant(self):
        from fa_b200.ops import Operator

        with self.assertRaises(ValueError):
            Operator("bf16")


if __name__ == "__main__":
    unittest.main()
