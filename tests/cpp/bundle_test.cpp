// Host checks of lrrt::bundle (no device needed): manifest parsing, launch
// configuration, kernarg packing and the error texts callers match on. The
// cases restate light-rocm-runtime tests/bundle.cpp (parse :58-103, kernarg
// buffer :105-150, manifest validation :152-175, multiple kernels :190-240,
// field order :242-285, invalid manifests :287-480, grid limits :482-500)
// with manifests of this file's own.
#include "lrrt/bundle.hpp"

#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

int failures = 0;

void expect(bool condition, const char *what) {
  if (!condition) {
    std::fprintf(stderr, "FAILED: %s\n", what);
    ++failures;
  }
}

// Expects `body` to throw; when `text` is given the message must contain it.
template <typename Body> void expect_error(Body body, const char *what, const char *text = nullptr) {
  try {
    body();
  } catch (const std::exception &error) {
    if (text != nullptr && std::strstr(error.what(), text) == nullptr) {
      std::fprintf(stderr, "FAILED: %s: message '%s' lacks '%s'\n", what, error.what(), text);
      ++failures;
    }
    return;
  }
  std::fprintf(stderr, "FAILED: %s: no error\n", what);
  ++failures;
}

lrrt::KernelManifest parse(const std::string &json, const char *name = nullptr) {
  return name == nullptr ? lrrt::parse_bundle_manifest(json.data(), json.size())
                         : lrrt::parse_bundle_manifest(json.data(), json.size(), name);
}

// One kernel entry; `body` holds the fields after "name".
std::string kernel(const char *name, const std::string &body) {
  return std::string(R"({"name":")") + name + "\"," + body + "}";
}

std::string manifest(const std::string &kernels, const char *head =
                                                     R"("manifest_version":1,"target":"sm_100a",)") {
  return std::string("{") + head + R"("kernels":[)" + kernels + "]}";
}

const char *kAxpyBody =
    R"("symbol":"axpy_kernel","code_object":"ops/axpy.cubin",
       "args":[{"name":"a","type":"f32","offset":0,"size":4},
               {"name":"x","type":"ptr","offset":8,"size":8},
               {"name":"y","type":"ptr","offset":16,"size":8}],
       "kernarg_size":24,"block":[256,1,1],"grid":["ceil_div(n, 1024) * 256",1,1],
       "shared_memory_bytes":64,"workspace_bytes":123456789012)";

void parse_and_configure() {
  const lrrt::KernelManifest m = parse(manifest(kernel("axpy", kAxpyBody)));
  expect(m.manifest_version == lrrt::kSupportedBundleManifestVersion, "version");
  expect(m.target == "sm_100a" && m.name == "axpy" && m.symbol == "axpy_kernel", "names");
  expect(m.code_object == "ops/axpy.cubin", "code object inside a subdirectory");
  expect(m.kernarg_size == 24 && m.shared_memory_bytes == 64, "sizes");
  expect(m.workspace_bytes == 123456789012ull, "64-bit workspace");
  expect(m.block[0] == 256 && m.block[1] == 1 && m.block[2] == 1, "block");
  expect(m.grid_divisor == 1024 && m.grid_multiplier == 256, "grid rule");
  expect(m.arg_offsets == std::vector<size_t>({0, 8, 16}), "offsets");
  expect(m.args.size() == 3 && m.args[1].name == "x" && m.args[1].type == "ptr" &&
             !m.args[1].optional,
         "argument metadata");
  const lr_launch_config_t c = lrrt::launch_config_from_manifest(m, 3000);
  expect(c.grid.x == 3 * 256 && c.grid.y == 1 && c.grid.z == 1, "grid = ceil(n/D)*M threads");
  expect(c.block.x == 256 && c.shared_memory_bytes == 64, "block and shared memory");
  lrrt::require_kernarg_layout(m, 24, {0, 8, 16});
  expect_error([&] { lrrt::require_kernarg_layout(m, 32, {0, 8, 16}); }, "size mismatch",
               "does not match kernarg layout");
  expect_error([&] { lrrt::require_kernarg_layout(m, 24, {0, 8, 20}); }, "offset mismatch",
               "does not match kernarg layout");
}

void kernarg_packing() {
  lrrt::KernelManifest m = parse(manifest(kernel("axpy", kAxpyBody)));
  lrrt::KernargBuffer args(m);
  expect(args.size() == 24, "buffer size");
  expect_error([&] { args.validate(); }, "nothing bound", "missing required bundle kernarg: a");
  const float a = 2.5f;
  const void *x = reinterpret_cast<const void *>(0x10000);
  void *y = reinterpret_cast<void *>(0x20000);
  args.set("a", a);
  args.set(size_t{1}, x);
  expect_error([&] { args.validate(); }, "one missing", "missing required bundle kernarg: y");
  args.set(2, y);
  args.validate();
  args.validate(m);
  const unsigned char *bytes = static_cast<const unsigned char *>(args.data());
  float a_back;
  const void *x_back;
  void *y_back;
  std::memcpy(&a_back, bytes, 4);
  std::memcpy(&x_back, bytes + 8, 8);
  std::memcpy(&y_back, bytes + 16, 8);
  expect(a_back == a && x_back == x && y_back == y, "packed at manifest offsets");
  expect_error([&] { args.set(3, y); }, "index past the end", "index is out of range");
  expect_error([&] { args.set(-1, y); }, "negative index", "index is out of range");
  expect_error([&] { args.set("z", y); }, "unknown name", "bundle kernarg not found: z");
  expect_error([&] { args.set("", y); }, "empty name", "bundle kernarg name is empty");
  const double wide = 1.0;
  expect_error([&] { args.set("a", wide); }, "value wider than its slot",
               "exceeds argument slot");
  expect_error([&] { args.set_raw(size_t{0}, nullptr, 4); }, "null value", "value is null");

  m.args[2].optional = true;
  lrrt::KernargBuffer optional(m);
  optional.set("a", a);
  optional.set("x", x);
  optional.validate(); // an unbound optional argument is allowed
  std::vector<unsigned char> poison(8, 0xab);
  optional.bind_optional_nulls();
  std::memcpy(poison.data(), static_cast<const unsigned char *>(optional.data()) + 16, 8);
  expect(poison == std::vector<unsigned char>(8, 0), "optional pointer bound to null");

  m.args[2].type = "u64";
  lrrt::KernargBuffer not_pointer(m);
  expect_error([&] { not_pointer.bind_optional_nulls(); }, "optional non-pointer",
               "optional null binding requires ptr argument: y");

  lrrt::KernelManifest other = parse(manifest(kernel("axpy", kAxpyBody)));
  lrrt::KernargBuffer checked(other);
  checked.set("a", a);
  checked.set("x", x);
  checked.set("y", y);
  lrrt::KernelManifest resized = other;
  resized.kernarg_size = 32;
  expect_error([&] { checked.validate(resized); }, "manifest size differs",
               "does not match kernel manifest");
  lrrt::KernelManifest renamed = other;
  renamed.args[0].name = "alpha";
  expect_error([&] { checked.validate(renamed); }, "manifest argument differs",
               "does not match kernel manifest");
}

void several_kernels() {
  const std::string body = R"("symbol":"k","code_object":"k.cubin",
      "args":[{"name":"p","type":"ptr","offset":0,"size":8}],"kernarg_size":8,
      "block":[32,1,1],"grid":["ceil_div(n, 32) * 32",1,1])";
  const std::string json =
      manifest(kernel("one", body) + "," + kernel("two", body + R"(,"shared_memory_bytes":512)") +
               "," + kernel("three", body));
  const lrrt::KernelManifest first = parse(json);
  expect(first.name == "one" && first.shared_memory_bytes == 0 && first.workspace_bytes == 0,
         "first kernel and defaults");
  const std::vector<lrrt::KernelManifest> all = lrrt::parse_bundle_manifests(json.data(),
                                                                            json.size());
  expect(all.size() == 3 && all[0].name == "one" && all[1].name == "two" &&
             all[2].name == "three",
         "all kernels in order");
  expect(parse(json, "two").shared_memory_bytes == 512, "kernel selected by name");
  expect_error([&] { parse(json, "four"); }, "unknown kernel", "bundle kernel not found: four");
  expect_error([&] { parse(json, ""); }, "empty kernel name", "bundle kernel name is empty");
  expect_error([&] { parse(manifest(kernel("one", body) + "," + kernel("one", body))); },
               "duplicate kernel", "duplicate kernel name in bundle manifest: one");
}

void field_order_and_nesting() {
  const std::string json = R"({
    "kernels": [{
      "workspace_bytes": 0,
      "producer": {"name": "ignored", "target": "ignored", "shared_memory_bytes": 7},
      "grid": ["ceil_div( n , 8 )*64", 1, 1],
      "args": [{"size": 8, "type": "ptr", "offset": 0, "name": "values"},
               {"offset": 8, "name": "count", "size": 4, "type": "u32"}],
      "block": [64, 1, 1], "kernarg_size": 16, "symbol": "s",
      "code_object": "a/b/c.cubin", "name": "late"
    }],
    "target": "sm_100a",
    "manifest_version": 1
  })";
  const lrrt::KernelManifest m = parse(json, "late");
  expect(m.target == "sm_100a" && m.name == "late" && m.symbol == "s",
         "top-level fields win over nested ones");
  expect(m.shared_memory_bytes == 0, "nested shared memory ignored");
  expect(m.grid_divisor == 8 && m.grid_multiplier == 64, "grid rule with extra spaces");
  expect(m.args.size() == 2 && m.args[0].name == "values" && m.args[1].name == "count",
         "argument fields in any order");
}

void invalid_manifests() {
  const std::string good_args = R"("args":[{"name":"p","type":"ptr","offset":0,"size":8}])";
  const std::string shape = R"("block":[32,1,1],"grid":["ceil_div(n, 32) * 32",1,1])";
  auto entry = [&](const std::string &extra, const std::string &args, const std::string &grid,
                   const char *code = "k.cubin", const char *kernarg = "8") {
    return manifest(kernel("bad", std::string(R"("symbol":"k","code_object":")") + code +
                                      R"(","kernarg_size":)" + kernarg + "," + args + "," +
                                      grid + extra));
  };
  expect_error([] { lrrt::parse_bundle_manifest(nullptr, 0); }, "no bytes",
               "bundle manifest is empty");
  expect_error([] { std::string j = "[1,2]"; parse(j); }, "root array", "root is not object");
  expect_error([] { std::string j = "{\"manifest_version\":1"; parse(j); }, "truncated JSON");
  expect_error([] { parse(manifest("", R"("target":"sm_100a",)")); }, "no version",
               "missing manifest token \"manifest_version\"");
  expect_error([] { parse(manifest("", R"("manifest_version":3,"target":"sm_100a",)")); },
               "future version", "unsupported bundle manifest_version: 3");
  expect_error([] { parse(manifest("", R"("manifest_version":1,)")); }, "no target",
               "missing manifest token \"target\"");
  expect_error([] { parse(manifest("", R"("manifest_version":1,"target":"",)")); },
               "empty target", "bundle manifest target is empty");
  expect_error([] { parse(manifest("")); }, "no kernels", "bundle manifest has no kernels");
  expect_error([] { parse(R"({"manifest_version":1,"target":"x","kernels":{}})"); },
               "kernels not an array", "manifest kernels is not array");
  expect_error([] { parse(manifest(kernel("bad", R"("symbol":"k")"))); }, "missing fields",
               "bundle manifest kernels[0] 'bad': missing manifest token \"code_object\"");
  expect_error([&] {
    parse(entry("", R"("args":[{"name":"p","type":"ptr","offset":0}])", shape));
  }, "argument without size",
               "bundle manifest kernels[0] 'bad': args[0]: missing manifest token \"size\"");
  expect_error([&] {
    parse(entry("", R"("args":[{"name":"p","type":"ptr","offset":0,"size":8},
                              {"name":"p","type":"ptr","offset":8,"size":8}])",
                shape, "k.cubin", "16"));
  }, "duplicate argument", "bundle manifest kernels[0] 'bad': args[1] 'p': duplicate argument name");
  expect_error([&] {
    parse(entry("", R"("args":[{"name":"p","type":"ptr","offset":0,"size":8},
                              {"name":"q","type":"ptr","offset":0,"size":8}])",
                shape, "k.cubin", "16"));
  }, "repeated offset", "argument offsets must be strictly increasing");
  expect_error([&] {
    parse(entry("", R"("args":[{"name":"p","type":"ptr","offset":8,"size":8}])", shape));
  }, "argument past kernarg_size", "argument range exceeds kernarg_size");
  expect_error([&] { parse(entry("", R"("args":[])", shape)); }, "no arguments",
               "bundle manifest has no arguments");
  expect_error([&] {
    parse(entry("", R"("args":[{"name":"p","type":"ptr","offset":-1,"size":8}])", shape));
  }, "negative offset", "invalid manifest integer: offset");
  expect_error([&] {
    parse(entry("", R"("args":[{"name":"p","type":"ptr","offset":0,"size":8,"optional":1}])",
                shape));
  }, "non-boolean optional", "manifest field is not boolean: optional");
  expect_error([&] {
    parse(entry("", good_args, R"("block":[32,1,1],"grid":["ceil_div(n, 32) * 32",1,4])"));
  }, "grid z", "bundle grid z dimension must be 1");
  expect_error([&] {
    parse(entry("", good_args, R"("block":[32,1,1],"grid":["ceil_div(n, 32) * 32",3,1])"));
  }, "grid y", "bundle grid y dimension must be 1");
  expect_error([&] {
    parse(entry("", good_args, R"("block":[32,1,1],"grid":["n * 32",1,1])"));
  }, "other grid rule", "unsupported bundle grid expression");
  expect_error([&] {
    parse(entry("", good_args, R"("block":[32,1,1],"grid":["ceil_div(n, 32) * 32 + 1",1,1])"));
  }, "grid rule suffix", "unsupported bundle grid expression");
  expect_error([&] {
    parse(entry("", good_args, R"("block":[32,1,1],"grid":["ceil_div(n, 4294967296) * 1",1,1])"));
  }, "huge divisor", "bundle grid expression is too large");
  expect_error([&] {
    parse(entry("", good_args, R"("block":[32,1],"grid":["ceil_div(n, 32) * 32",1,1])"));
  }, "two block dimensions", "invalid manifest array: block");
  expect_error([&] { parse(entry("", good_args, shape, "../k.cubin")); }, "parent directory",
               "bundle code object path must stay in bundle");
  expect_error([&] { parse(entry("", good_args, shape, "/abs/k.cubin")); }, "absolute path",
               "bundle code object path must stay in bundle");
  expect_error([&] { parse(entry(R"(,"shared_memory_bytes":4294967296)", good_args, shape)); },
               "shared memory above 32 bits", "bundle shared memory requirement is too large");
  expect_error([&] { parse(entry("", good_args, shape, "k.cubin", "\"8\"")); },
               "string kernarg size", "manifest field is not integer: kernarg_size");
}

void launch_limits() {
  lrrt::KernelManifest m = parse(manifest(kernel("axpy", kAxpyBody)));
  expect_error([&] { lrrt::launch_config_from_manifest(m, 0); }, "n = 0",
               "grid dimensions must be non-zero");
  lrrt::KernelManifest wide = m;
  wide.block[1] = 65536;
  expect_error([&] { lrrt::launch_config_from_manifest(wide, 4096); }, "block above 16 bits",
               "exceed HSA packet limits");
  lrrt::KernelManifest narrow = m;
  narrow.grid_multiplier = 128; // one program of 128 threads < block 256
  expect_error([&] { lrrt::launch_config_from_manifest(narrow, 1); }, "grid below block",
               "cover the workgroup");
  lrrt::KernelManifest huge = m;
  huge.grid_divisor = 1;
  huge.grid_multiplier = 0x80000000u;
  expect_error([&] { lrrt::launch_config_from_manifest(huge, 2); }, "grid above 32 bits",
               "bundle grid size is too large");
  lrrt::KernelManifest zero = m;
  zero.block[2] = 0;
  expect_error([&] { lrrt::launch_config_from_manifest(zero, 8); }, "zero block",
               "block dimensions must be non-zero");
}

} // namespace

int main() {
  parse_and_configure();
  kernarg_packing();
  several_kernels();
  field_order_and_nesting();
  invalid_manifests();
  launch_limits();
  if (failures == 0) {
    std::printf("bundle checks: ok\n");
  }
  return failures == 0 ? 0 : 1;
}
