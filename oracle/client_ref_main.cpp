// client_ref_main.cpp -- TEST INFRASTRUCTURE, not product code.
//
// Runs the reference client's own text decoder (decode_tokens and
// fix_mojibake, rtl/vc707/host/bfp_client.cpp:904-1027) on cases read from
// stdin, so that the Python client port can be pinned to the C++ it
// replaces.  The reference translation unit is compiled where it lies: its
// path comes in as BFP_CLIENT_CPP and its main() is renamed by the build
// recipe (oracle/build_client_ref.sh), nothing of it is copied here.
//
// Usage:  bfp_client_ref <vocab.bin>  < cases
// Each input line is one case; each output line is the hex of the result:
//   "T id id id ..."   decode_tokens(vocab, ids)  (ids decimal, may be empty)
//   "M hexbytes"       fix_mojibake(bytes)        (hex, may be empty)
#ifndef BFP_CLIENT_CPP
#error "build with -DBFP_CLIENT_CPP=\"<path of bfp_client.cpp>\""
#endif
#include BFP_CLIENT_CPP
#undef main  // the recipe renamed the reference's main() only

#include <iostream>

namespace {

std::string to_hex(const std::string& s) {
  static const char* d = "0123456789abcdef";
  std::string o;
  o.reserve(2 * s.size());
  for (unsigned char c : s) {
    o.push_back(d[c >> 4]);
    o.push_back(d[c & 15]);
  }
  return o;
}

std::string from_hex(const std::string& h) {
  std::string o;
  for (size_t i = 0; i + 1 < h.size(); i += 2) o.push_back(static_cast<char>(std::stoi(h.substr(i, 2), nullptr, 16)));
  return o;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 2) {
    std::fprintf(stderr, "usage: %s <vocab.bin> < cases\n", argv[0]);
    return 2;
  }
  const Vocab v = Vocab::load(argv[1]);
  std::string line;
  while (std::getline(std::cin, line)) {
    if (line.empty()) continue;
    std::istringstream in(line.substr(1));
    if (line[0] == 'T') {
      std::vector<uint16_t> ids;
      unsigned long t;
      while (in >> t) ids.push_back(static_cast<uint16_t>(t));
      std::cout << to_hex(decode_tokens(v, ids)) << '\n';
    } else if (line[0] == 'M') {
      std::string h;
      in >> h;
      std::cout << to_hex(fix_mojibake(from_hex(h))) << '\n';
    } else {
      std::fprintf(stderr, "bad case line: %s\n", line.c_str());
      return 2;
    }
  }
  return 0;
}
