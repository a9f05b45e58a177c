// transaction.hpp — the execution transaction over a multi-partition plan
// (src/execution_transaction/transaction.rs:27-644): prepare reserves and
// validates, execute runs the accepted operations in order, commit publishes
// the staged write-set atomically once the declared boundary is reached, and
// abort releases or retires everything with no partial publication. Host
// code only; the device work behind an operation belongs to the backend.
//
// Partitions are the ranks of a tensor-parallel group (ordinals 0-63, one
// bit each in participant masks). An operation is identified by its kind and
// a 64-bit reference (the reference's LaunchRef / TransferRef /
// CollectiveRef / BarrierRef strings).
#pragma once

#include <chrono>
#include <cstdint>
#include <map>
#include <optional>
#include <set>
#include <string>
#include <tuple>
#include <utility>
#include <vector>

#include "faber_gpu.h"

namespace faber {
namespace txn {

enum class OpKind : uint32_t { Launch = 0, Transfer = 1, Broadcast = 2, Barrier = 3 };

// One operation of the accepted plan (TransactionOperation,
// src/execution_transaction/mirror.rs:635-656).
struct Op {
  OpKind kind = OpKind::Launch;
  uint32_t partition = 0;     // launch: its partition; transfer, broadcast: the source
  uint32_t destination = 0;   // transfer: the destination
  uint64_t participants = 0;  // broadcast, barrier: partition mask
  uint64_t ref = 0;
  uint64_t bytes = 0;         // launch: output bytes; transfer, broadcast: byte count
  bool operator==(const Op& o) const {
    return kind == o.kind && partition == o.partition && destination == o.destination &&
           participants == o.participants && ref == o.ref && bytes == o.bytes;
  }
  bool operator!=(const Op& o) const { return !(*this == o); }
};

using OpKey = std::pair<uint32_t, uint64_t>;  // OperationRef: (kind, ref)

inline OpKey op_key(const Op& op) { return {(uint32_t)op.kind, op.ref}; }

inline std::set<uint32_t> mask_partitions(uint64_t mask) {
  std::set<uint32_t> s;
  for (uint32_t p = 0; p < 64; ++p)
    if (mask >> p & 1) s.insert(p);
  return s;
}

// Partitions an operation involves (mirror.rs:686-696).
inline std::set<uint32_t> op_partitions(const Op& op) {
  switch (op.kind) {
    case OpKind::Launch: return {op.partition};
    case OpKind::Transfer: return {op.partition, op.destination};
    default: return mask_partitions(op.participants);
  }
}

// Bytes an executed operation moved (mirror.rs:698-706).
inline uint64_t op_byte_count(const Op& op) {
  switch (op.kind) {
    case OpKind::Transfer: return op.bytes;
    case OpKind::Broadcast: {
      const uint64_t n = (uint64_t)op_partitions(op).size();
      return op.bytes * (n ? n - 1 : 0);
    }
    default: return 0;
  }
}

// OperationEvent: one completion per involved partition (mirror.rs:708-752).
struct Event {
  uint32_t kind = 0, partition = 0;
  uint64_t ref = 0;
  bool operator<(const Event& o) const {
    return std::tie(kind, partition, ref) < std::tie(o.kind, o.partition, o.ref);
  }
};

inline std::set<Event> op_events(const Op& op) {
  std::set<Event> e;
  for (uint32_t p : op_partitions(op)) e.insert({(uint32_t)op.kind, p, op.ref});
  return e;
}

// A staged output: launch output, transfer destination, broadcast copy per
// non-source participant (mirror.rs:754-788).
struct Write {
  uint32_t kind = 0, partition = 0;
  uint64_t ref = 0, bytes = 0;
  std::tuple<uint32_t, uint64_t, uint32_t> key() const { return {kind, ref, partition}; }
};

using WriteKey = std::tuple<uint32_t, uint64_t, uint32_t>;

inline std::vector<Write> op_writes(const Op& op) {
  std::vector<Write> w;
  switch (op.kind) {
    case OpKind::Launch: w.push_back({0, op.partition, op.ref, op.bytes}); break;
    case OpKind::Transfer: w.push_back({1, op.destination, op.ref, op.bytes}); break;
    case OpKind::Broadcast:
      for (uint32_t p : op_partitions(op))
        if (p != op.partition) w.push_back({2, p, op.ref, op.bytes});
      break;
    case OpKind::Barrier: break;
  }
  return w;
}

// Backend error classes (src/execution_transaction/backend.rs:17-54).
enum class ErrClass : int32_t { Allocation = 1, Operation = 2, DeviceLoss = 3, Cancelled = 4, Timeout = 5 };

struct BackendError {
  ErrClass cls = ErrClass::Operation;
  uint32_t partition = 0;
  std::string detail;
};

using MaybeError = std::optional<BackendError>;

// TransactionFailure (state_machine.rs:63-72).
enum class FailKind : int32_t { None = 0, Backend = 1, PublishFailed = 2, Cancelled = 3 };

struct Failure {
  FailKind kind = FailKind::None;
  BackendError error;  // Backend, PublishFailed
  std::string detail;  // PublishFailed detail or Cancelled reason
};

enum class State : int32_t { New = 0, Prepared = 1, Executing = 2, Committed = 3, Failed = 4, Aborted = 5 };

// Per-partition reservation (reservation.rs:41-110): class 6 staging and
// class 3 output buffers, event objects and transaction scratch.
struct Reservation {
  uint64_t staging = 0, output = 0, events = 0, scratch = 0;
  uint64_t class_six() const { return staging; }
  uint64_t class_three() const { return output + events + scratch; }
};

constexpr uint64_t kEventObjectBytes = 64;       // reservation.rs:13
constexpr uint64_t kScratchPerPartition = 4096;  // reservation.rs:18

// derive_reservation (reservation.rs:112-170): a transfer stages its bytes
// at both ends and writes them at the destination; a broadcast stages at
// every participant and writes at every non-source one; a launch writes its
// output; every operation costs one event object per partition it involves.
inline std::map<uint32_t, Reservation> derive_reservation(const std::vector<Op>& ops,
                                                          const std::set<uint32_t>& referenced) {
  std::map<uint32_t, uint64_t> staging, outputs, events;
  for (const Op& op : ops) {
    for (uint32_t p : op_partitions(op)) events[p] += kEventObjectBytes;
    switch (op.kind) {
      case OpKind::Launch: outputs[op.partition] += op.bytes; break;
      case OpKind::Transfer:
        staging[op.partition] += op.bytes;
        staging[op.destination] += op.bytes;
        outputs[op.destination] += op.bytes;
        break;
      case OpKind::Broadcast:
        for (uint32_t p : op_partitions(op)) {
          staging[p] += op.bytes;
          if (p != op.partition) outputs[p] += op.bytes;
        }
        break;
      case OpKind::Barrier: break;
    }
  }
  std::map<uint32_t, Reservation> r;
  for (uint32_t p : referenced) r[p] = {staging[p], outputs[p], events[p], kScratchPerPartition};
  return r;
}

// The device side of a transaction (DeviceExecutionBackend,
// backend.rs:89-118).
class Backend {
 public:
  virtual ~Backend() = default;
  virtual MaybeError reserve(uint32_t partition, const Reservation& r) = 0;
  virtual MaybeError run_operation(const Op& op) = 0;
  virtual bool event_completed(const Event& e) const = 0;
  virtual MaybeError stage_write(const Write& w) = 0;
  virtual MaybeError publish() = 0;
  virtual uint64_t staged_bytes() const = 0;
  virtual uint64_t published_bytes() const = 0;
  virtual void release(uint32_t partition) = 0;
  virtual void retire(uint32_t partition, const Failure& f) = 0;
};

// The happy-path fake (FakeExecutionBackend, backend.rs:120-360): holds
// reservations, stages and publishes writes in host maps, and completes
// every dispatched event at once unless auto-completion is off.
class FakeBackend : public Backend {
 public:
  std::map<uint32_t, Reservation> reservations;
  std::map<WriteKey, Write> staged, published;
  uint64_t staged_total = 0, published_total = 0;
  bool published_once = false;
  std::vector<Op> executed;
  std::set<Event> dispatched, completed;
  std::set<uint32_t> released, retired;
  bool auto_complete = true;

  void complete_event(const Event& e) {
    dispatched.insert(e);
    completed.insert(e);
  }
  MaybeError reserve(uint32_t p, const Reservation& r) override {
    if (reservations.count(p))
      return BackendError{ErrClass::Allocation, p,
                          "partition " + std::to_string(p) + " already holds a reservation"};
    reservations[p] = r;
    return std::nullopt;
  }
  MaybeError run_operation(const Op& op) override {
    executed.push_back(op);
    for (const Event& e : op_events(op)) {
      dispatched.insert(e);
      if (auto_complete) completed.insert(e);
    }
    return std::nullopt;
  }
  bool event_completed(const Event& e) const override { return completed.count(e) > 0; }
  MaybeError stage_write(const Write& w) override {
    if (staged.count(w.key())) return BackendError{ErrClass::Allocation, w.partition, "output staged twice"};
    staged_total += w.bytes;
    staged[w.key()] = w;
    return std::nullopt;
  }
  MaybeError publish() override {
    if (published_once)
      return BackendError{ErrClass::Operation, 0, "publish called twice: publication is one-shot"};
    published = staged;  // all or nothing
    published_total = staged_total;
    published_once = true;
    return std::nullopt;
  }
  uint64_t staged_bytes() const override { return staged_total; }
  uint64_t published_bytes() const override { return published_total; }
  void release(uint32_t p) override {
    reservations.erase(p);
    released.insert(p);
  }
  void retire(uint32_t p, const Failure&) override {
    for (auto it = staged.begin(); it != staged.end();) {
      if (it->second.partition == p) {
        staged_total -= it->second.bytes;
        it = staged.erase(it);
      } else {
        ++it;
      }
    }
    reservations.erase(p);
    retired.insert(p);
  }
};

// Fault classes (src/fake_device.rs:60-90).
enum class FaultClass : int32_t { Cancel = 1, Timeout = 2, TransferError = 3, KernelError = 4, DeviceLoss = 5 };

inline const char* fault_spelling(FaultClass c) {
  switch (c) {
    case FaultClass::Cancel: return "cancel";
    case FaultClass::Timeout: return "timeout";
    case FaultClass::TransferError: return "transfer-error";
    case FaultClass::KernelError: return "kernel-error";
    default: return "device-loss";
  }
}

// The backend error a fault surfaces as (FaultInjection::to_backend_error).
inline ErrClass fault_error_class(FaultClass c) {
  switch (c) {
    case FaultClass::Cancel: return ErrClass::Cancelled;
    case FaultClass::Timeout: return ErrClass::Timeout;
    case FaultClass::DeviceLoss: return ErrClass::DeviceLoss;
    default: return ErrClass::Operation;  // transfer and kernel errors
  }
}

struct Fault {
  OpKey op;
  uint32_t partition = 0;
  FaultClass cls = FaultClass::KernelError;
};

struct DeliveredFault {
  Fault fault;
  BackendError error;
  uint64_t reclaimed_copy_bytes = 0;  // an in-flight copy reclaimed by the fault
};

// The fault-injecting backend (FaultInjectingBackend,
// src/fake_device.rs:184-318): one-shot faults per (operation, partition)
// over the fake, and the write-set of the last successful publication,
// which a failed transaction never changes. A reserve while no reservation
// is held starts a fresh transaction with fresh staging.
class FaultBackend : public Backend {
 public:
  FakeBackend inner;
  std::vector<Fault> faults;
  std::vector<DeliveredFault> delivered;
  std::map<WriteKey, Write> committed;
  uint64_t committed_total = 0;
  std::optional<ErrClass> fail_publish;  // one-shot publication failure

  MaybeError reserve(uint32_t p, const Reservation& r) override {
    if (inner.reservations.empty()) {
      const bool ac = inner.auto_complete;
      inner = FakeBackend();
      inner.auto_complete = ac;
    }
    return inner.reserve(p, r);
  }
  MaybeError run_operation(const Op& op) override {
    const std::set<uint32_t> parts = op_partitions(op);
    for (size_t i = 0; i < faults.size(); ++i) {
      const Fault f = faults[i];
      if (f.op != op_key(op) || !parts.count(f.partition)) continue;
      faults.erase(faults.begin() + (long)i);
      BackendError e{fault_error_class(f.cls), f.partition,
                     std::string("injected ") + fault_spelling(f.cls) + " on operation " + std::to_string(op.ref)};
      const bool copy = op.kind == OpKind::Transfer &&
                        (f.cls == FaultClass::Timeout || f.cls == FaultClass::TransferError);
      delivered.push_back({f, e, copy ? op.bytes : 0});
      return e;
    }
    return inner.run_operation(op);
  }
  bool event_completed(const Event& e) const override { return inner.event_completed(e); }
  MaybeError stage_write(const Write& w) override { return inner.stage_write(w); }
  MaybeError publish() override {
    if (fail_publish) {
      const ErrClass c = *fail_publish;
      fail_publish.reset();
      return BackendError{c, 0, "injected publication failure"};
    }
    MaybeError e = inner.publish();
    if (!e) {
      committed = inner.published;
      committed_total = inner.published_total;
    }
    return e;
  }
  uint64_t staged_bytes() const override { return inner.staged_bytes(); }
  uint64_t published_bytes() const override { return inner.published_bytes(); }
  void release(uint32_t p) override { inner.release(p); }
  void retire(uint32_t p, const Failure& f) override { inner.retire(p, f); }
};

// Error kinds of the lifecycle calls (errors.rs:12-125).
enum TxnError : int32_t {
  kTxnOk = 0,
  kTxnDegeneratePlan = 1,
  kTxnEmptySnapshot = 2,
  kTxnInvalidState = 3,
  kTxnUnknownPartition = 4,
  kTxnDuplicateOperation = 5,
  kTxnUndeclaredBoundaryBarrier = 6,
  kTxnUndeclaredBoundaryLaunch = 7,
  kTxnMissingAdmittedBudget = 8,
  kTxnReservationExceedsBudget = 9,
  kTxnBackend = 10,
  kTxnOperationOutsideSnapshot = 11,
  kTxnBoundaryNotReached = 12,
  kTxnPublishFailed = 13,
  kTxnAlreadyCommitted = 14
};

struct Outcome {
  int32_t kind = kTxnOk;
  std::string message;
  BackendError backend;       // kTxnBackend, kTxnPublishFailed
  uint32_t partition = 0;     // partition-scoped errors
  int32_t budget_class = 0;   // 6 or 3 for kTxnReservationExceedsBudget
  uint64_t missing = 0;       // kTxnBoundaryNotReached: boundary refs not reached
  bool ok() const { return kind == kTxnOk; }
};

inline Outcome fail_with(int32_t kind, std::string msg) {
  Outcome o;
  o.kind = kind;
  o.message = std::move(msg);
  return o;
}

inline const char* state_name(State s) {
  static const char* n[] = {"New", "Prepared", "Executing", "Committed", "Failed", "Aborted"};
  return n[(int)s];
}

// A partition of the bound plan: its admitted ledger, if it has one.
struct BoundPartition {
  bool admitted = false;
  FaberPartitionLedgerV1 ledger{};
};

class Transaction {
 public:
  // ExecutionTransaction::new (transaction.rs:60-95): a plan over fewer
  // than two partitions and an empty snapshot are refused.
  static Outcome create(std::map<uint32_t, BoundPartition> plan, std::vector<Op> ops,
                        std::vector<uint64_t> boundary_barriers, std::vector<uint64_t> boundary_launches,
                        Transaction& out) {
    if (plan.size() < 2) return fail_with(kTxnDegeneratePlan, "DegeneratePlan: fewer than two partitions");
    if (ops.empty()) return fail_with(kTxnEmptySnapshot, "EmptySnapshot: no operations");
    out = Transaction();
    out.plan_ = std::move(plan);
    out.ops_ = std::move(ops);
    out.barriers_ = std::move(boundary_barriers);
    out.launches_ = std::move(boundary_launches);
    return {};
  }

  State state() const { return state_; }
  const Failure& failure() const { return failure_; }
  const std::map<uint32_t, Reservation>& reservation() const { return reservation_; }
  uint64_t declared_write_bytes() const {
    uint64_t b = 0;
    for (const auto& kv : declared_) b += kv.second.bytes;
    return b;
  }
  size_t declared_writes() const { return declared_.size(); }

  // prepare (transaction.rs:200-316): the five checks in order (topology,
  // unique identities, declared boundary, admitted budgets, reservation
  // within classes 6 and 3), then the reservation held on the backend. Any
  // failure reserves nothing and leaves the transaction New.
  Outcome prepare(Backend& be) {
    if (state_ != State::New) return invalid_state("prepare");
    const auto t0 = std::chrono::steady_clock::now();
    for (size_t i = 0; i < ops_.size(); ++i)
      for (uint32_t p : op_partitions(ops_[i]))
        if (!plan_.count(p)) {
          Outcome o = fail_with(kTxnUnknownPartition, "UnknownPartition: partition " + std::to_string(p) +
                                                          " of operation " + std::to_string(i));
          o.partition = p;
          return o;
        }
    std::map<OpKey, size_t> keys;
    for (size_t i = 0; i < ops_.size(); ++i)
      if (!keys.emplace(op_key(ops_[i]), i).second)
        return fail_with(kTxnDuplicateOperation, "DuplicateOperation: " + std::to_string(ops_[i].ref));
    for (uint64_t b : barriers_)
      if (!find_op(OpKind::Barrier, b))
        return fail_with(kTxnUndeclaredBoundaryBarrier, "UndeclaredBoundaryBarrier: " + std::to_string(b));
    for (uint64_t l : launches_)
      if (!find_op(OpKind::Launch, l))
        return fail_with(kTxnUndeclaredBoundaryLaunch, "UndeclaredBoundaryLaunch: " + std::to_string(l));
    std::set<uint32_t> referenced;
    for (const Op& op : ops_)
      for (uint32_t p : op_partitions(op)) referenced.insert(p);
    for (uint32_t p : referenced)
      if (!plan_.at(p).admitted) {
        Outcome o =
            fail_with(kTxnMissingAdmittedBudget, "MissingAdmittedBudget: partition " + std::to_string(p));
        o.partition = p;
        return o;
      }
    const auto res = derive_reservation(ops_, referenced);
    for (const auto& kv : res) {
      const FaberPartitionLedgerV1& L = plan_.at(kv.first).ledger;
      const bool six = kv.second.class_six() > L.transfer_staging_bytes;
      if (six || kv.second.class_three() > L.activation_scratch_bytes) {
        Outcome o = fail_with(kTxnReservationExceedsBudget,
                              std::string("ReservationExceedsBudget: partition ") + std::to_string(kv.first) +
                                  (six ? " class 6 " : " class 3 ") +
                                  std::to_string(six ? kv.second.class_six() : kv.second.class_three()) +
                                  " bytes over an admitted " +
                                  std::to_string(six ? L.transfer_staging_bytes : L.activation_scratch_bytes));
        o.partition = kv.first;
        o.budget_class = six ? 6 : 3;
        return o;
      }
    }
    std::vector<uint32_t> held;
    for (const auto& kv : res) {
      if (MaybeError e = be.reserve(kv.first, kv.second)) {
        for (uint32_t p : held) be.release(p);  // nothing stays reserved
        return backend_outcome(kTxnBackend, *e);
      }
      held.push_back(kv.first);
    }
    keys_ = std::move(keys);
    reservation_ = res;
    declared_.clear();
    for (const Op& op : ops_)
      for (const Write& w : op_writes(op)) declared_[w.key()] = w;
    prepare_ns_ = elapsed(t0);
    state_ = State::Prepared;
    return {};
  }

  // execute (transaction.rs:318-342): every accepted operation in plan
  // order; a backend failure moves to Failed. Execute cannot run twice.
  Outcome execute(Backend& be) {
    if (state_ != State::Prepared) return invalid_state("execute");
    const auto t0 = std::chrono::steady_clock::now();
    state_ = State::Executing;
    const std::vector<Op> snapshot = ops_;
    for (const Op& op : snapshot) {
      Outcome o = execute_operation(be, op);
      if (!o.ok()) {
        execute_ns_ = elapsed(t0);
        return o;
      }
    }
    execute_ns_ = elapsed(t0);
    return {};
  }

  // execute_operation (transaction.rs:344-406): only an operation of the
  // prepare snapshot, with the same declared facts, can run.
  Outcome execute_operation(Backend& be, const Op& op) {
    if (state_ != State::Executing) return invalid_state("execute_operation");
    auto it = keys_.find(op_key(op));
    if (it == keys_.end() || ops_[it->second] != op)
      return fail_with(kTxnOperationOutsideSnapshot, "OperationOutsideSnapshot: " + std::to_string(op.ref));
    if (MaybeError e = be.run_operation(op)) {
      fail_backend(*e);
      return backend_outcome(kTxnBackend, *e);
    }
    for (const Write& w : op_writes(op)) {
      if (MaybeError e = be.stage_write(w)) {
        fail_backend(*e);
        return backend_outcome(kTxnBackend, *e);
      }
      staged_[w.key()] = w;
    }
    executed_.push_back(op);
    executed_bytes_ += op_byte_count(op);
    for (const Event& e : op_events(op))
      if (be.event_completed(e)) events_.insert(e);
    return {};
  }

  // commit (transaction.rs:408-470): a missing boundary is transient
  // (nothing published, still Executing); then one atomic publication and
  // every reservation released. A publication failure moves to Failed.
  Outcome commit(Backend& be, uint64_t ordinal) {
    if (state_ != State::Executing) return invalid_state("commit");
    const auto t0 = std::chrono::steady_clock::now();
    for (const Op& op : ops_)
      for (const Event& e : op_events(op))
        if (be.event_completed(e)) events_.insert(e);
    const uint64_t missing = missing_boundary();
    if (missing) {
      Outcome o = fail_with(kTxnBoundaryNotReached,
                            "BoundaryNotReached: " + std::to_string(missing) + " boundary reference(s) pending");
      o.missing = missing;
      return o;
    }
    if (MaybeError e = be.publish()) {
      failure_ = {FailKind::PublishFailed, *e, e->detail};
      state_ = State::Failed;
      return backend_outcome(kTxnPublishFailed, *e);
    }
    for (const auto& kv : reservation_) {
      be.release(kv.first);
      released_.insert(kv.first);
    }
    published_staged_ = be.staged_bytes();
    published_bytes_ = be.published_bytes();
    published_ = true;
    decision_ = 1;
    ordinal_ = ordinal;
    state_ = State::Committed;
    finalize_ns_ = elapsed(t0);
    return {};
  }

  // abort (transaction.rs:472-528): idempotent; partitions holding staged
  // writes are retired, the other reservations released. A committed
  // transaction cannot be aborted.
  Outcome abort(Backend& be, const std::string& reason) {
    if (state_ == State::Aborted) return {};
    if (state_ == State::Committed) return fail_with(kTxnAlreadyCommitted, "AlreadyCommitted: cannot abort");
    const auto t0 = std::chrono::steady_clock::now();
    std::set<uint32_t> staged_parts;
    for (const auto& kv : staged_) staged_parts.insert(kv.second.partition);
    const Failure f = state_ == State::Failed ? failure_ : Failure{FailKind::Cancelled, {}, reason};
    for (uint32_t p : staged_parts) {
      be.retire(p, f);
      retired_.insert(p);
    }
    for (const auto& kv : reservation_)
      if (!staged_parts.count(kv.first)) {
        be.release(kv.first);
        released_.insert(kv.first);
      }
    failure_ = f;
    state_ = State::Aborted;
    decision_ = 2;
    finalize_ns_ = elapsed(t0);
    return {};
  }

  // The receipt's figures (receipt.rs): decision, ordinal, write-set and
  // executed totals, events, teardown masks and timings.
  void receipt(FaberTxnReceiptV1& r) const {
    r = FaberTxnReceiptV1{};
    r.decision = decision_;
    r.state = (int32_t)state_;
    r.failure_kind = (int32_t)failure_.kind;
    const bool be = failure_.kind == FailKind::Backend || failure_.kind == FailKind::PublishFailed;
    r.failure_class = be ? (int32_t)failure_.error.cls : 0;
    r.failure_partition = be ? failure_.error.partition : 0;
    r.published = published_ ? 1 : 0;
    r.publication_ordinal = ordinal_;
    r.declared_write_bytes = declared_write_bytes();
    r.executed_operations = executed_.size();
    r.executed_bytes = executed_bytes_;
    r.completed_events = events_.size();
    r.staged_bytes = published_staged_;
    r.published_bytes = published_bytes_;
    for (uint32_t p : released_) r.released_partitions |= 1ull << p;
    for (uint32_t p : retired_) r.retired_partitions |= 1ull << p;
    r.partial_publication = 0;  // publication is all or nothing
    r.prepare_ns = prepare_ns_;
    r.execute_ns = execute_ns_;
    r.finalize_ns = finalize_ns_;
  }

 private:
  std::map<uint32_t, BoundPartition> plan_;
  std::vector<Op> ops_;
  std::vector<uint64_t> barriers_, launches_;
  std::map<OpKey, size_t> keys_;
  State state_ = State::New;
  std::map<uint32_t, Reservation> reservation_;
  std::map<WriteKey, Write> declared_, staged_;
  std::vector<Op> executed_;
  uint64_t executed_bytes_ = 0;
  std::set<Event> events_;
  Failure failure_;
  int32_t decision_ = 0;  // 1 committed, 2 aborted
  uint64_t ordinal_ = 0;
  bool published_ = false;
  uint64_t published_staged_ = 0, published_bytes_ = 0;
  std::set<uint32_t> released_, retired_;
  uint64_t prepare_ns_ = 0, execute_ns_ = 0, finalize_ns_ = 0;

  static uint64_t elapsed(std::chrono::steady_clock::time_point t0) {
    return (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0)
        .count();
  }
  const Op* find_op(OpKind k, uint64_t ref) const {
    for (const Op& op : ops_)
      if (op.kind == k && op.ref == ref) return &op;
    return nullptr;
  }
  Outcome invalid_state(const char* call) const {
    return fail_with(kTxnInvalidState, std::string("InvalidState: ") + call + " in state " + state_name(state_));
  }
  static Outcome backend_outcome(int32_t kind, const BackendError& e) {
    Outcome o = fail_with(kind, std::string(kind == kTxnPublishFailed ? "PublishFailed: " : "Backend: ") + e.detail);
    o.backend = e;
    o.partition = e.partition;
    return o;
  }
  // the first failure wins (transaction.rs:530-540)
  void fail_backend(const BackendError& e) {
    if (state_ == State::New || state_ == State::Prepared || state_ == State::Executing) {
      failure_ = {FailKind::Backend, e, e.detail};
      state_ = State::Failed;
    }
  }
  // boundary refs whose completion events have not all arrived: a barrier
  // needs every participant, a launch its partition (transaction.rs:554-608)
  uint64_t missing_boundary() const {
    uint64_t missing = 0;
    auto check = [&](OpKind k, uint64_t ref) {
      const Op* op = find_op(k, ref);
      bool ok = op != nullptr;
      if (op)
        for (const Event& e : op_events(*op))
          if (!events_.count(e)) ok = false;
      if (!ok) ++missing;
    };
    for (uint64_t b : barriers_) check(OpKind::Barrier, b);
    for (uint64_t l : launches_) check(OpKind::Launch, l);
    return missing;
  }
};

}  // namespace txn
}  // namespace faber
