// vmb_pool.cuh -- the VM's constant pool and slot table of a .vmb program,
// parsed on the host and held in device memory: the load half of Vm::load
// (core/src/interp.rs:123-220) and bind_slots (:351-397), with the OP_LAYERB
// base (:438-475, :1019-1045). Container layout: core/src/format.rs.
#pragma once
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

namespace vmlm {

constexpr uint32_t kVmbMagic = 0x4D4C4D56u;  // "VMLM" little-endian (format.rs MAGIC)
constexpr size_t kVmbHeader = 28;            // magic u32, version u16, pad u16, text off/len, const off/len, meta off
constexpr size_t kVmbMetaHdr = 28;           // META_HDR
constexpr size_t kVmbConstEnt = 24;          // CONST_ENT: off, len, rows, cols, dtype (u8 at 16), name hash (at 20)
constexpr size_t kVmbSlotEnt = 16;           // SLOT_ENT: kind, idx_or_off, rows, cols
constexpr size_t kVmbInsSize = 16;           // INS_SIZE: op u8, fl u8, dt u16, dst, a, b
constexpr uint32_t kVmbSlotConst = 0, kVmbSlotAct = 1, kVmbSlotState = 2, kVmbSlotGrad = 3, kVmbSlotParam = 4;
constexpr uint8_t kVmbOpGemm = 10;           // trans/src/opcode.rs OP_GEMM
// Opcodes whose fields the load-time dtype audit treats specially (trans/src/opcode.rs:11, 17, 50, 65, 81, 82, 94)
constexpr uint8_t kVmbOpSlice = 6, kVmbOpEmb = 14, kVmbOpShape = 52, kVmbOpWritecol = 71, kVmbOpPush = 86,
                  kVmbOpPop = 87, kVmbOpLoopCnt = 89;
constexpr uint8_t kVmbDtF32 = 0, kVmbDtI8 = 2, kVmbDtBf16 = 4;
constexpr size_t kVmbRegionPad = 64;         // Vm::load allocates every scratch region with 64 bytes of slack

// format.rs dtype_size: bytes per element, 0 for an unknown dtype.
inline size_t vmb_dtype_size(uint8_t dt) {
  switch (dt) {
    case 0: return 4;         // DT_F32
    case 1: case 4: return 2; // DT_F16, DT_BF16
    case 2: return 1;         // DT_I8
    case 3: return 4;         // DT_I32
    default: return 0;
  }
}

// format.rs hash32: FNV-1a over the name's bytes.
inline uint32_t vmb_hash32(const char* s) {
  uint32_t h = 0x811c9dc5u;
  for (; *s; ++s) {
    h ^= static_cast<uint8_t>(*s);
    h *= 0x01000193u;
  }
  return h;
}

struct VmbConst {
  uint32_t off, len, rows, cols, hash;
  uint8_t dtype;
};

struct VmbSlot {
  uint32_t kind;   // kVmbSlot*; kinds past 4 bind to the activation region, as bind_slots does
  uint64_t off;    // byte offset inside its region
  uint32_t rows, cols;
  uint8_t dtype;   // the constant's dtype for const / param slots, DT_F32 otherwise
  uint32_t name;   // slot name hash
};

struct VmbLayout {
  uint64_t text_off = 0, text_len = 0, const_off = 0, const_len = 0, meta_off = 0;
  uint64_t act_bytes = 0, state_bytes = 0, grad_bytes = 0;
  std::vector<VmbConst> consts;
  std::vector<VmbSlot> slots;
};

inline uint32_t vmb_u32(const uint8_t* p) {
  uint32_t v;
  std::memcpy(&v, p, 4);
  return v;
}

// Parse and check a .vmb image of `len` bytes. Every table read is bounds-checked
// (the VM trusts the file). Returns 0, or a VMLM status with `msg` set:
//   VMLM_ERR_ARG      "bad magic" (the VM prints it and exits 3)
//   VMLM_ERR_SHAPE    a header, table, constant or slot that lies outside the image or its region
//   VMLM_ERR_OPERATOR "const has unknown dtype" (bind_slots: the VM prints it and exits 9)
// `const_avail` is the size of the constant bytes the pool will hold: the CONST
// section of the image, or the separate weights buffer of load_weights_mapped.
inline int vmb_parse(const uint8_t* b, size_t len, bool separate_weights, size_t weights_len, VmbLayout* out,
                     const char** msg) {
  auto bad = [&](int code, const char* m) {
    *msg = m;
    return code;
  };
  if (len < kVmbHeader) return bad(2, "vmb: image shorter than its header");
  if (vmb_u32(b) != kVmbMagic) return bad(1, "bad magic");
  VmbLayout L;
  L.text_off = vmb_u32(b + 8);
  L.text_len = vmb_u32(b + 12);
  L.const_off = vmb_u32(b + 16);
  L.const_len = vmb_u32(b + 20);
  L.meta_off = vmb_u32(b + 24);
  if (L.text_off + L.text_len > len || L.text_len % kVmbInsSize) return bad(2, "vmb: TEXT section outside the image");
  if (separate_weights) {
    if (weights_len < L.const_len) return bad(2, "vmb: weights buffer shorter than the header's const length");
  } else if (L.const_off + L.const_len > len) {
    return bad(2, "vmb: CONST section outside the image");
  }
  const uint64_t mo = L.meta_off;
  if (mo + kVmbMetaHdr > len) return bad(2, "vmb: META header outside the image");
  const uint64_t n_const = vmb_u32(b + mo), n_slot = vmb_u32(b + mo + 4), slots_off = vmb_u32(b + mo + 8);
  L.act_bytes = vmb_u32(b + mo + 12);
  L.state_bytes = vmb_u32(b + mo + 16);
  L.grad_bytes = vmb_u32(b + mo + 20);
  const uint64_t names_off = vmb_u32(b + mo + 24);
  if (mo + kVmbMetaHdr + n_const * kVmbConstEnt > len) return bad(2, "vmb: const table outside the image");
  if (mo + slots_off + n_slot * kVmbSlotEnt > len) return bad(2, "vmb: slot table outside the image");
  if (mo + names_off + n_slot * 4 > len) return bad(2, "vmb: slot name table outside the image");
  L.consts.resize(n_const);
  for (uint64_t i = 0; i < n_const; ++i) {
    const uint8_t* e = b + mo + kVmbMetaHdr + i * kVmbConstEnt;
    L.consts[i] = VmbConst{vmb_u32(e), vmb_u32(e + 4), vmb_u32(e + 8), vmb_u32(e + 12), vmb_u32(e + 20), e[16]};
  }
  L.slots.resize(n_slot);
  for (uint64_t i = 0; i < n_slot; ++i) {
    const uint8_t* e = b + mo + slots_off + i * kVmbSlotEnt;
    VmbSlot s{vmb_u32(e), vmb_u32(e + 4), vmb_u32(e + 8), vmb_u32(e + 12), 0, vmb_u32(b + mo + names_off + i * 4)};
    const uint64_t elems = static_cast<uint64_t>(s.rows) * s.cols;
    if (s.kind == kVmbSlotConst || s.kind == kVmbSlotParam) {
      if (s.off >= n_const) return bad(2, "vmb: a slot names a constant past the const table");
      const VmbConst& c = L.consts[s.off];
      s.dtype = c.dtype;
      const size_t esz = vmb_dtype_size(c.dtype);
      if (esz == 0) return bad(8, "const has unknown dtype");
      if (c.off + elems * esz > L.const_len) return bad(2, "vmb: a constant slot extends past the constant pool");
      s.off = c.off;
    } else {
      const uint64_t region = s.kind == kVmbSlotState ? L.state_bytes : s.kind == kVmbSlotGrad ? L.grad_bytes
                                                                                              : L.act_bytes;
      if (s.off + elems * 4 > region + kVmbRegionPad) return bad(2, "vmb: a scratch slot extends past its region");
    }
    L.slots[i] = s;
  }
  *out = std::move(L);
  return 0;
}

// OP_LAYERB (core/src/interp.rs:1019-1045): a signed delta; d >= 0 adds
// `d as usize` (saturating), d < 0 subtracts `(-d) as usize` (saturating);
// Rust's float-to-integer casts saturate and map NaN to 0.
inline uint64_t vmb_layerb(uint64_t base, float d) {
  auto to_u = [](float x) -> uint64_t {
    if (!(x > 0.f)) return 0;
    if (x >= 18446744073709551616.0f) return UINT64_MAX;
    return static_cast<uint64_t>(x);
  };
  if (d >= 0.f) {
    const uint64_t add = to_u(d);
    return base > UINT64_MAX - add ? UINT64_MAX : base + add;
  }
  const uint64_t back = to_u(-d);
  return base > back ? base - back : 0;
}

// The load-time dtype audit of Vm::load (audit_const_dtypes, core/src/interp.rs:241-345): a non-f32
// constant may be read only as the B operand of OP_GEMM (bf16 or i8; any other non-f32 B has no kernel) or
// as the bf16 table of OP_EMB with an f32 destination; every other instruction field that names a slot must
// name an f32 one. Fields that hold numbers rather than slots are not checked: SHAPE (all), LOOP_CNT's dst
// and b, the b of SLICE / WRITECOL / PUSH / POP. Slot numbers past the table are skipped, as the VM's probe
// skips them (the VM's GEMM / EMB arms would read past the table there). Returns 0, or 8 with the VM's
// message (it prints it and exits 9).
inline int vmb_audit(const uint8_t* b, const VmbLayout& L, std::string* msg) {
  const size_t n_ins = L.text_len / kVmbInsSize;
  const size_t n_slots = L.slots.size();
  auto dtype = [&](uint32_t s) { return s < n_slots ? L.slots[s].dtype : kVmbDtF32; };
  for (size_t i = 0; i < n_ins; ++i) {
    const uint8_t* ins = b + L.text_off + i * kVmbInsSize;
    const uint8_t op = ins[0];
    const uint32_t dst = vmb_u32(ins + 4), a = vmb_u32(ins + 8), bb = vmb_u32(ins + 12);
    if (op == kVmbOpGemm) {
      const uint8_t bdt = dtype(bb);
      if (bdt == kVmbDtBf16 || bdt == kVmbDtI8 || bdt == kVmbDtF32) continue;
      *msg = "gemm B has no kernel for this dtype";
      return 8;
    }
    if (op == kVmbOpEmb) {
      if (dtype(a) != kVmbDtBf16) continue;
      if (dtype(dst) == kVmbDtF32) continue;
    }
    bool cd = true, ca = true, cb = true;
    if (op == kVmbOpShape) {
      cd = ca = cb = false;
    } else if (op == kVmbOpLoopCnt) {
      cd = cb = false;
    } else if (op == kVmbOpSlice || op == kVmbOpWritecol || op == kVmbOpPush || op == kVmbOpPop) {
      cb = false;
    }
    const uint32_t fields[3] = {dst, a, bb};
    const bool check[3] = {cd, ca, cb};
    for (int f = 0; f < 3; ++f) {
      if (!check[f] || fields[f] >= n_slots) continue;
      const uint8_t dt = L.slots[fields[f]].dtype;
      if (dt == kVmbDtF32) continue;
      const char* what = dt == kVmbDtBf16 ? " uses bf16 const at slot " : dt == kVmbDtI8 ? " uses i8 const at slot "
                                                                                         : " uses non-f32 const at slot ";
      *msg = "op " + std::to_string(op) + what + std::to_string(fields[f]) +
             " (only a GEMM may read a non-f32 operand)";
      return 8;
    }
  }
  return 0;
}

}  // namespace vmlm
