// ref_check_main.cpp -- TEST INFRASTRUCTURE ONLY.  Command-line wrapper of
// ref_check_gguf (ref_shim.cpp): runs the reference's own GGUF loader, weight
// map and execution plan over a file and prints the plan dimensions, in a
// process of its own.
#include <cstdio>
#include <cstdlib>

extern "C" int ref_check_gguf(const char* path, unsigned long long context_tokens, long long* dims, char* err,
                              int err_len);

int main(int argc, char** argv) {
  if (argc < 2) {
    std::fprintf(stderr, "usage: kib_ref_check model.gguf [context_tokens]\n");
    return 2;
  }
  long long dims[8] = {0};
  char err[512] = {0};
  const unsigned long long ctx = argc > 2 ? std::strtoull(argv[2], nullptr, 10) : 4096;
  const int rc = ref_check_gguf(argv[1], ctx, dims, err, sizeof(err));
  if (rc != 0) {
    std::printf("error %s\n", err);
    return 1;
  }
  std::printf("ok");
  for (long long d : dims) std::printf(" %lld", d);
  std::printf("\n");
  return 0;
}
