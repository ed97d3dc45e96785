// A host program written against the reference's q38::NvidiaDriver interface
// (include/q38/driver.hpp) and linked to libq38driver_b200.so: it opens the
// device, runs the pattern, VMM and RMSNorm smokes and the GEMV smokes on the
// matrices a manifest lists, and prints the reference's `key: value` lines.
//
//   facade_smoke MANIFEST
//
// Manifest lines: `kind path cols rows [qh_offset qs_offset]`, kind one of
// q4k, q5k, q6k, iq4xs, q5k_sm86.  Exit status 0 and a final PASS line when
// every smoke succeeded.
#include "q38/driver.hpp"

#include <cstdio>
#include <fstream>
#include <iostream>
#include <iterator>
#include <sstream>
#include <string>
#include <vector>

static std::vector<std::byte> read_file(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    std::vector<char> raw((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    std::vector<std::byte> out(raw.size());
    for (size_t i = 0; i < raw.size(); ++i) out[i] = static_cast<std::byte>(raw[i]);
    return out;
}

int main(int argc, char** argv) {
    if (argc < 2) {
        std::cerr << "usage: facade_smoke MANIFEST\n";
        return 2;
    }
    q38::NvidiaDriver d;
    try {
        d.open();
    } catch (const std::exception& e) {
        std::cerr << "open: " << e.what() << "\n";
        return 3;
    }
    std::cout << "device: " << d.device_name() << "\nsm: " << d.sm_major() << d.sm_minor()
              << "\nis_target_sm: " << (d.is_sm86() ? 1 : 0) << "\n";
    bool ok = true;
    std::string err;
    ok &= d.probe_vmm(64u << 20, &err);
    std::cout << "vmm_probe: " << (err.empty() ? "ok" : err) << "\n";
    ok &= d.run_sm86_smoke(&err);
    double ma = 0, mr = 0, ms = 0, g1 = 0, g2 = 0;
    ok &= d.run_rmsnorm_smoke(&err, &ma, &mr);
    std::cout << "rmsnorm_max_abs: " << ma << "\n";
    std::ifstream man(argv[1]);
    std::string line;
    while (std::getline(man, line)) {
        std::istringstream ls(line);
        std::string kind, path;
        uint32_t cols = 0, rows = 0;
        size_t qh = 0, qs = 0;
        ls >> kind >> path >> cols >> rows >> qh >> qs;
        const std::vector<std::byte> m = read_file(path);
        err.clear();
        bool r = false;
        if (kind == "q4k") r = d.run_q4k_gemv_smoke(m.data(), cols, rows, &err, &ma, &mr, &ms, &g1);
        else if (kind == "q5k") r = d.run_q5k_gemv_smoke(m.data(), cols, rows, &err, &ma, &mr, &ms, &g1);
        else if (kind == "q6k") r = d.run_q6k_gemv_smoke(m.data(), cols, rows, &err, &ma, &mr, &ms, &g1);
        else if (kind == "iq4xs") r = d.run_iq4xs_gemv_smoke(m.data(), cols, rows, &err, &ma, &mr, &ms, &g1);
        else if (kind == "q5k_sm86")
            r = d.run_q5k_sm86_gemv_smoke(m.data(), qh, qs, cols, rows, &err, &ma, &mr, &ms, &g1, &g2);
        else err = "unknown kind " + kind;
        std::cout << kind << "_ok: " << (r ? 1 : 0) << "\n" << kind << "_max_abs: " << ma << "\n"
                  << kind << "_max_rel: " << mr << "\n" << kind << "_ms: " << ms << "\n"
                  << kind << "_gbps: " << g1 << "\n";
        if (!r) std::cout << kind << "_error: " << err << "\n";
        ok &= r;
    }
    err.clear();
    const bool gdn = d.run_gdn_ar_smoke(128, 16, 48, nullptr, &err);
    std::cout << "gdn_ar_smoke: " << (gdn ? "ran" : err) << "\n";
    d.close();
    std::cout << (ok ? "PASS" : "FAIL") << "\n";
    return ok ? 0 : 1;
}
