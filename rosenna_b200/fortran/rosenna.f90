! module rosenna -- Fortran binding of the B200 engine (librosenna_b200.so).
!
! Keeps roseNNa's solver-side calls (fLibrary/rosenna.f90, README "Hello
! RoseNNa"): `use rosenna`, `call initialize()`, `call use_model(inputs..., output)`,
! now with a leading batch dimension of independent samples.  initialize() is
! the library's bind(c) symbol itself (as reader.f90:38); use_model is a generic
! over fp32 and fp64 arrays of any rank (assumed rank, Fortran 2018) for models
! with one, three or five inputs (MLP/CNN; LSTM with h0,c0; two LSTMs) and one
! output.  Arrays are the reference layout: the ONNX shape with its batch
! dimension widened to n, contiguous.  An optional `stat` receives the status
! (0 = OK); without it a failure stops the program, as the reference does.
!
! Not compiled in this repository's build: the image carries no Fortran compiler.
module rosenna
    use iso_c_binding
    implicit none
    private
    public :: initialize, use_model, rosenna_finalize_f

    interface
        subroutine initialize() bind(c, name="initialize")
        end subroutine initialize
        integer(c_int) function c_last_status() bind(c, name="rosenna_last_status")
            import :: c_int
        end function c_last_status
        integer(c_int) function c_use_f32(n, ins, outs) bind(c, name="rosenna_use_model_f32")
            import :: c_int, c_int64_t, c_ptr
            integer(c_int64_t), value :: n
            type(c_ptr), value :: ins, outs
        end function c_use_f32
        integer(c_int) function c_use_f64(n, ins, outs) bind(c, name="rosenna_use_model_f64")
            import :: c_int, c_int64_t, c_ptr
            integer(c_int64_t), value :: n
            type(c_ptr), value :: ins, outs
        end function c_use_f64
        integer(c_int) function c_input_shape(i, dims, maxd, bdim) bind(c, name="rosenna_input_shape")
            import :: c_int, c_int64_t
            integer(c_int), value :: i, maxd
            integer(c_int64_t) :: dims(*)
            integer(c_int) :: bdim
        end function c_input_shape
        integer(c_int) function c_finalize() bind(c, name="rosenna_finalize")
            import :: c_int
        end function c_finalize
    end interface

    interface use_model
        module procedure use_model_1_f32, use_model_1_f64, use_model_3_f32, use_model_3_f64, &
                         use_model_5_f32, use_model_5_f64
    end interface use_model

contains

    subroutine rosenna_finalize_f()
        integer(c_int) :: rc
        rc = c_finalize()
    end subroutine rosenna_finalize_f

    ! batch size: the extent of input 0 along its batch dimension
    integer(c_int64_t) function batch_of(x) result(n)
        class(*), intent(in) :: x(..)
        integer(c_int64_t) :: dims(8)
        integer(c_int) :: bdim, r
        r = c_input_shape(0_c_int, dims, 8_c_int, bdim)
        n = size(x, bdim + 1, kind=c_int64_t)
    end function batch_of

    subroutine finish(rc, stat)
        integer(c_int), intent(in) :: rc
        integer, intent(out), optional :: stat
        if (present(stat)) then
            stat = rc
        else if (rc /= 0) then
            error stop "rosenna: use_model failed (see rosenna_last_error)"
        end if
    end subroutine finish

    subroutine use_model_1_f32(i0, o0, stat)
        real(c_float), intent(in), target, contiguous :: i0(..)
        real(c_float), intent(out), target, contiguous :: o0(..)
        integer, intent(out), optional :: stat
        type(c_ptr), target :: ins(1), outs(1)
        ins(1) = c_loc(i0); outs(1) = c_loc(o0)
        call finish(c_use_f32(batch_of(i0), c_loc(ins), c_loc(outs)), stat)
    end subroutine use_model_1_f32

    subroutine use_model_1_f64(i0, o0, stat)
        real(c_double), intent(in), target, contiguous :: i0(..)
        real(c_double), intent(out), target, contiguous :: o0(..)
        integer, intent(out), optional :: stat
        type(c_ptr), target :: ins(1), outs(1)
        ins(1) = c_loc(i0); outs(1) = c_loc(o0)
        call finish(c_use_f64(batch_of(i0), c_loc(ins), c_loc(outs)), stat)
    end subroutine use_model_1_f64

    subroutine use_model_3_f32(i0, i1, i2, o0, stat)
        real(c_float), intent(in), target, contiguous :: i0(..), i1(..), i2(..)
        real(c_float), intent(out), target, contiguous :: o0(..)
        integer, intent(out), optional :: stat
        type(c_ptr), target :: ins(3), outs(1)
        ins = [c_loc(i0), c_loc(i1), c_loc(i2)]; outs(1) = c_loc(o0)
        call finish(c_use_f32(batch_of(i0), c_loc(ins), c_loc(outs)), stat)
    end subroutine use_model_3_f32

    subroutine use_model_3_f64(i0, i1, i2, o0, stat)
        real(c_double), intent(in), target, contiguous :: i0(..), i1(..), i2(..)
        real(c_double), intent(out), target, contiguous :: o0(..)
        integer, intent(out), optional :: stat
        type(c_ptr), target :: ins(3), outs(1)
        ins = [c_loc(i0), c_loc(i1), c_loc(i2)]; outs(1) = c_loc(o0)
        call finish(c_use_f64(batch_of(i0), c_loc(ins), c_loc(outs)), stat)
    end subroutine use_model_3_f64

    subroutine use_model_5_f32(i0, i1, i2, i3, i4, o0, stat)
        real(c_float), intent(in), target, contiguous :: i0(..), i1(..), i2(..), i3(..), i4(..)
        real(c_float), intent(out), target, contiguous :: o0(..)
        integer, intent(out), optional :: stat
        type(c_ptr), target :: ins(5), outs(1)
        ins = [c_loc(i0), c_loc(i1), c_loc(i2), c_loc(i3), c_loc(i4)]; outs(1) = c_loc(o0)
        call finish(c_use_f32(batch_of(i0), c_loc(ins), c_loc(outs)), stat)
    end subroutine use_model_5_f32

    subroutine use_model_5_f64(i0, i1, i2, i3, i4, o0, stat)
        real(c_double), intent(in), target, contiguous :: i0(..), i1(..), i2(..), i3(..), i4(..)
        real(c_double), intent(out), target, contiguous :: o0(..)
        integer, intent(out), optional :: stat
        type(c_ptr), target :: ins(5), outs(1)
        ins = [c_loc(i0), c_loc(i1), c_loc(i2), c_loc(i3), c_loc(i4)]; outs(1) = c_loc(o0)
        call finish(c_use_f64(batch_of(i0), c_loc(ins), c_loc(outs)), stat)
    end subroutine use_model_5_f64

end module rosenna
